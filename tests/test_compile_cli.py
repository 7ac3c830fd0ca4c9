"""compile.py keeps the reference's contract (compile.py:9-19 and
scripts/check_all.py:39-46 of the reference): PTX on stdout, starting with
.version, ASCII, entry named after the IR kernel, parameters in meta.json's
arg_order; failures exit non-zero with nothing on stdout.  Every module
assembles for sm_100a with ptxas (a CPU-side check)."""

import json
import re
import shutil
import subprocess
import sys

import pytest

from conftest import GOLDEN, PACKAGES, ROOT

IRS = sorted(p for d in PACKAGES for p in (GOLDEN / d).glob("*.ir.json"))
PTXAS = shutil.which("ptxas")


def run_compile(path, *flags):
    return subprocess.run([sys.executable, str(ROOT / "compile.py"), *flags, str(path)], capture_output=True,
                          text=True)


@pytest.mark.parametrize("mode", ["tuned", "generic"])
@pytest.mark.parametrize("path", IRS, ids=lambda p: f"{p.parent.name}/{p.stem}")
def test_compile_contract(path, mode, tmp_path):
    r = run_compile(path, *(["--generic"] if mode == "generic" else []))
    assert r.returncode == 0, r.stderr
    ptx = r.stdout
    assert ptx.startswith(".version") and ptx.isascii()
    assert ".target sm_100a" in ptx
    meta = json.loads((path.parent / "meta.json").read_text())
    entry = path.name[: -len(".ir.json")]
    k = next(k for k in meta["kernels"] if k["entry"] == entry)
    sig = re.search(r"\.entry\s+(\w+)\s*\(([^)]*)\)", ptx)
    assert sig.group(1) == entry
    params = re.findall(r"\.param\s+\.u64\s+(\w+)", sig.group(2))
    assert params == [f"p_{a}" for a in k["arg_order"]]
    if PTXAS:
        f = tmp_path / "k.ptx"
        f.write_text(ptx)
        a = subprocess.run([PTXAS, "-arch=sm_100a", str(f), "-o", str(tmp_path / "k.cubin")],
                           capture_output=True, text=True)
        assert a.returncode == 0, a.stderr


def test_unsupported_statement_fails_loudly(tmp_path):
    src = GOLDEN / "p00_scalar_add"
    g = json.loads((src / "k_add_pointwise.ir.json").read_text())
    node = next(n for n in g["nodes"].values() if n["op"] == "KernelOp")
    node["op_fields"]["body"] = ["Tile(axes=(Axis(name='a0', extent=Dim(64), window=None),), "
                                 "body=(TensorMapPrefetch(desc='d', src_buffer='x'),), block_threads=64, aux_threads=0, "
                                 "raster_axes=None, raster_group=None, raster_orient='m')"]
    (tmp_path / "k_add_pointwise.ir.json").write_text(json.dumps(g))
    shutil.copy(src / "meta.json", tmp_path / "meta.json")
    r = run_compile(tmp_path / "k_add_pointwise.ir.json")
    assert r.returncode != 0 and r.stdout == ""
    assert "TensorMapPrefetch" in r.stderr and "NotImplementedError" in r.stderr


def test_missing_meta_entry_fails(tmp_path):
    src = GOLDEN / "p00_scalar_add"
    shutil.copy(src / "k_add_pointwise.ir.json", tmp_path / "k_add_pointwise.ir.json")
    meta = json.loads((src / "meta.json").read_text())
    meta["kernels"][0]["entry"] = "other"
    (tmp_path / "meta.json").write_text(json.dumps(meta))
    r = run_compile(tmp_path / "k_add_pointwise.ir.json")
    assert r.returncode != 0 and r.stdout == ""
