"""Programmatic dependent launch, on the CPU: a tuned module whose launch record says ``pdl``
may begin while the stream's previous kernel still runs, so in its tuned body no access to
global data (loads, stores, atomics, TMA and bulk copies) may come before
``griddepcontrol.wait`` -- only the guard's reads of the module's own tensor-map tables, which
the host alone writes.  The generic path of the same module waits first thing."""

import re

import pytest

from conftest import GOLDEN
from thompiler import load, synth
from thompiler.compiler import compile_kernel
from thompiler.emitter import read_sidecar

GLOBAL = re.compile(r"^\s*(@!?%\w+\s+)?(ld\.global|st\.global|atom\.|red\.|cp\.async\.bulk|cp\.reduce\.async|"
                    r"ld\.(relaxed|acquire|volatile)|st\.(relaxed|release|volatile)|prefetch)")
HOST_TABLES = ("thc_tmap_ptr", "thc_tmap_ring")

CASES = [
    ("rows", lambda d: synth.row_package(d, "softmax", 256, 4096)),
    ("sum", lambda d: synth.sum_package(d, 1 << 20)),
    ("pointwise", lambda d: synth.pointwise_package(d, 1 << 20, "relu_mul")),
    ("matmul pair", lambda d: synth.matmul_package(d, 1024, 1024, 512)),
    ("matmul", lambda d: synth.matmul_package(d, 384, 320, 512)),
    ("attention", lambda d: synth.attention_package(d, 1, 2, 512, 128)),
    ("f32 matmul", lambda d: GOLDEN / "m01_matmul_512"),
]


def _body(ptx: str) -> list[str]:
    start = ptx.index("{", ptx.index(".entry"))
    return ptx[start:].splitlines()


@pytest.mark.parametrize("name,make", CASES, ids=[c[0] for c in CASES])
def test_no_global_access_before_the_wait(tmp_path, name, make):
    d = make(tmp_path / "p")
    ir = sorted(d.glob("*.ir.json"))[0]
    ptx = compile_kernel(load.load(str(ir)))
    side = read_sidecar(ptx) or {}
    assert side.get("pdl") is True, (name, side.get("family"))
    lines = _body(ptx)
    waits = [i for i, ln in enumerate(lines) if "griddepcontrol.wait" in ln]
    assert len(waits) >= 2                                 # the tuned body and the generic path
    for ln in lines[:waits[0]]:
        if GLOBAL.match(ln):
            assert any(t in ln for t in HOST_TABLES), (name, ln)
    assert "griddepcontrol.launch_dependents" in "\n".join(lines[:waits[0]])
    generic = next(i for i, ln in enumerate(lines) if "generic lowering of the same IR" in ln)
    first = next(ln for ln in lines[generic + 1:] if ln.strip() and not ln.strip().startswith("//"))
    assert "griddepcontrol.wait" in first


def test_generic_compile_has_no_pdl(tmp_path):
    """``compile.py --generic`` output (the reference-equivalent lowering) is unchanged: no
    griddepcontrol and no pdl launch record."""
    d = synth.sum_package(tmp_path / "s", 1 << 20)
    ptx = compile_kernel(load.load(str(next(d.glob("*.ir.json")))), tuned=False)
    assert "griddepcontrol" not in ptx and not (read_sidecar(ptx) or {}).get("pdl")
