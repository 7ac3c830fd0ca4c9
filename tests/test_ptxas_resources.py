"""ptxas resource checks of the tuned families (CPU: ptxas assembles sm_100a without a GPU):
at the benchmark shapes and the edge shapes, every tuned module assembles with no spill
stores or loads and no stack frame, and its tuned CTA fits one SM's register file -- a spill
or an over-budget launch would be a silent performance loss (or a launch failure) that the
GPU parity tests would not name."""

import json
import re
import shutil
import subprocess

import pytest

from thompiler import load, synth
from thompiler.compiler import compile_kernel
from thompiler.emitter import read_sidecar

PTXAS = shutil.which("ptxas")
pytestmark = pytest.mark.skipif(PTXAS is None, reason="ptxas not on PATH")

CASES = [
    ("attention", synth.attention_package, (8, 16, 2048, 128), {}),
    ("attention", synth.attention_package, (1, 2, 384, 128), {}),
    ("attention", synth.attention_package, (2, 2, 512, 64), {}),
    ("attention", synth.attention_package, (1, 1, 128, 64), {}),
    ("matmul single CTA", synth.matmul_package, (4096, 4096, 4096), {"matmul_pair": False}),
    ("matmul", synth.matmul_package, (4096, 4096, 4096), {}),
    ("matmul", synth.matmul_package, (8192, 3072, 1024), {}),
    ("matmul", synth.matmul_package, (384, 320, 512), {}),
    ("matmul f16 out", synth.matmul_package, (2048, 2048, 1024, "col", "f16"), {}),
    ("matmul row-major B", synth.matmul_package, (1024, 1024, 1024, "row"), {}),
    ("row softmax", synth.row_package, ("softmax", 8192, 4096), {}),
    ("rmsnorm", synth.row_package, ("rmsnorm", 8192, 4096), {}),
    ("sum", synth.sum_package, (1 << 20,), {}),
    ("big sum", synth.sum_package, (1 << 30,), {}),
    ("pointwise", synth.pointwise_package, (1 << 28, "relu_mul"), {}),
]


def _ptxas_info(ptx: str, tmp_path) -> dict:
    f = tmp_path / "k.ptx"
    f.write_text(ptx)
    r = subprocess.run([PTXAS, "-arch=sm_100a", "-O3", "-v", str(f), "-o", str(tmp_path / "k.cubin")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = r.stderr
    return {"regs": int(re.search(r"Used (\d+) registers", out).group(1)),
            "stack": int(re.search(r"(\d+) bytes stack frame", out).group(1)),
            "spill_st": int(re.search(r"(\d+) bytes spill stores", out).group(1)),
            "spill_ld": int(re.search(r"(\d+) bytes spill loads", out).group(1))}


@pytest.mark.parametrize("what,builder,args,tuning", CASES,
                         ids=[f"{c[0]}-{'x'.join(map(str, c[2][:4]))}" for c in CASES])
def test_tuned_module_has_no_spills(tmp_path, monkeypatch, what, builder, args, tuning):
    from thompiler.families.tuning import TUNING
    for k, v in tuning.items():
        monkeypatch.setattr(TUNING, k, v)
    d = builder(tmp_path / "p", *args)
    ir = next(d.glob("*.ir.json"))
    ptx = compile_kernel(load.load(str(ir)))
    fam = re.search(r"// family: ([\w-]+)", ptx)
    assert fam and fam.group(1) != "generic", f"{what}: no tuned family recognised"
    info = _ptxas_info(ptx, tmp_path)
    assert info["spill_st"] == 0 and info["spill_ld"] == 0 and info["stack"] == 0, (what, info)
    side = read_sidecar(ptx) or {}
    block = side.get("block") or json.loads((d / "meta.json").read_text())["kernels"][0]["block"]
    threads = block[0] * block[1] * block[2]
    warps = -(-threads // 32)
    # the tuned CTA's registers fit one SM (65,536), allocated per warp in units of 256
    per_warp = -(-info["regs"] * 32 // 256) * 256
    assert per_warp * warps <= 65536, (what, info, threads)
