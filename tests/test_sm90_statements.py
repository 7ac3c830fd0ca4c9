"""The IR statements the reference compiler does not lower (TASK.md's * entries), on the CPU:
they parse, lower to PTX that ptxas accepts for sm_100a, record their tensor maps in the
launch sidecar, and refuse at compile time the tensor maps the TMA unit would reject."""

import re
import shutil
import subprocess

import pytest

from sm90_ir import N, TILE, scan_package, select_package, tma_transpose_package, window_package
from thompiler import ir, load, synth
from thompiler.compiler import compile_kernel
from thompiler.emitter import read_sidecar


def _ptx(d):
    return compile_kernel(load.load(str(next(d.glob("*.ir.json")))))


def _ptxas(ptx, tmp_path):
    if shutil.which("ptxas") is None:
        pytest.skip("ptxas not on PATH")
    f = tmp_path / "k.ptx"
    f.write_text(ptx)
    r = subprocess.run(["ptxas", "-arch=sm_100a", str(f), "-o", str(tmp_path / "k.cubin")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_statements_parse_from_repr():
    stmts = [ir.TmaDescriptor("d", "x", (8, 16), (8, 16), "B64", synth.F32T),
             ir.TmaLoad("buf", (synth.L(0),), "d", (synth.L(0), synth.L(0)), "bar", synth.L(1)),
             ir.MbarrierInit("bar", synth.L(1), synth.L(0)), ir.MbarrierArriveExpectTx("bar", synth.L(512), None),
             ir.MbarrierArrive("bar", None), ir.MbarrierWait("bar", synth.V("ph"), None), ir.SetMaxNReg(232, "inc"),
             ir.Select("s", (ir.Branch("a", synth.B("<", synth.V("i"), synth.L(3))), ir.Branch("b", None))),
             ir.ZeroPrologue("z", synth.L(8)), ir.Pre("p", "c", (synth.L(0),)),
             ir.Carry("c", "v", (synth.L(0),), synth.L(0), synth.F32T)]
    for s in stmts:
        assert ir.parse_stmt(synth.to_repr(s)) == s
    # an arm written with another constructor name keeps its fields
    sel = ir.parse_stmt("Select(name='s', branches=(SelectBranch(value='a', select=None),))")
    assert isinstance(sel, ir.Select) and isinstance(sel.branches[0], ir.Opaque)


def test_tma_transpose_lowers(tmp_path):
    ptx = _ptx(tma_transpose_package(tmp_path / "t"))
    side = read_sidecar(ptx)
    assert side["error_word"] == "thc_error" and "grid" not in side          # meta.json's launch
    (m,) = side["ir_tmaps"]
    assert m == {"global": "thc_tmap_dx", "param": "x", "dtype": "f32", "dims": [N, N], "strides": [N * 4],
                 "box": [TILE, TILE], "swizzle": 0}
    assert "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes" in ptx
    assert "mbarrier.init.shared::cta.b64" in ptx and "fence.mbarrier_init.release.cluster" in ptx
    assert "mbarrier.arrive.expect_tx.shared::cta.b64" in ptx and "mbarrier.try_wait.parity" in ptx
    assert re.search(r"setp\.lt\.u32 [^,]+, [^,]+, 262144", ptx)                 # the wait is bounded
    _ptxas(ptx, tmp_path)


def test_select_zero_prologue_builtins_lower(tmp_path):
    ptx = _ptx(select_package(tmp_path / "s"))
    for s in ("%ctaid.x", "%tid.x", "min.s32", "selp.f32", "st.global.u32"):
        assert s in ptx, s
    _ptxas(ptx, tmp_path)


@pytest.mark.parametrize("box,swizzle,why", [((64, 2), None, "not a multiple of 16"),
                                            ((300, 64), None, "outside 1..256"),
                                            ((64, 64), "B128", "wider than the 128-byte swizzle"),
                                            ((64, 32), "B7", "swizzle")])
def test_bad_tensor_maps_refused(tmp_path, box, swizzle, why):
    d = tma_transpose_package(tmp_path / "t")
    f = next(d.glob("*.ir.json"))
    txt = f.read_text().replace("box_extents=(64, 64)", f"box_extents={box}")
    txt = txt.replace("swizzle=None, dtype=DataType", f"swizzle={swizzle!r}, dtype=DataType")
    f.write_text(txt)
    with pytest.raises((ValueError, NotImplementedError), match=why):
        _ptx(d)


def test_set_max_nreg_and_checks(tmp_path):
    from thompiler.emitter import Emitter
    from thompiler.handlers.async_copy import emit_set_max_nreg
    from thompiler.walk import Walker
    k = load.load(str(next(select_package(tmp_path / "s").glob("*.ir.json"))))
    w = Walker(Emitter(), k)
    emit_set_max_nreg(w, ir.SetMaxNReg(232, "inc"))
    emit_set_max_nreg(w, ir.SetMaxNReg(40, "dec"))
    text = "\n".join(w.em.lines)
    assert "setmaxnreg.inc.sync.aligned.u32 232" in text and "setmaxnreg.dec.sync.aligned.u32 40" in text
    for bad in (ir.SetMaxNReg(230, "inc"), ir.SetMaxNReg(16, "dec"), ir.SetMaxNReg(64, "sideways")):
        with pytest.raises(ValueError):
            emit_set_max_nreg(w, bad)


def test_unbuilt_vocabulary_fails_loudly(tmp_path):
    """A statement this reader does not model fails at lowering, naming the statement, as the
    reference does for every statement it lacks; a BlockScaleLoad into an undeclared fragment
    and a Wgmma statement in a kernel with no WgmmaMma are refused."""
    d = select_package(tmp_path / "s")
    f = next(d.glob("*.ir.json"))
    text = f.read_text()
    zp = "ZeroPrologue(dst='z', words=Literal(value=64, dtype='int'))"
    f.write_text(text.replace(zp, "TensorMapPrefetch(desc='d')"))
    with pytest.raises(NotImplementedError, match="TensorMapPrefetch"):
        _ptx(d)
    f.write_text(text.replace(zp, "BlockScaleLoad(frag='sf', src_buffer='x', src_index=(Var(name='a0'), "
                                  "Literal(value=0, dtype='int')), role='a')"))
    with pytest.raises(KeyError, match="used before its RegFragment"):
        _ptx(d)
    f.write_text(text.replace(zp, "WgmmaFence()"))
    with pytest.raises(ValueError, match="WgmmaFence in a kernel without a WgmmaMma"):
        _ptx(d)


def test_carried_state_lowers(tmp_path):
    """Carry / Pre: each cell is seeded before its loop, copied at each step's start, replaced at
    its end; a Pre inside the loop reads the previous step's value, after the loop the final one."""
    ptx = _ptx(scan_package(tmp_path / "c"))
    for cell, seed in (("acc__cell_s", "0f00000000"), ("fib__cell_0", "0f00000000"), ("fib__cell_1", "0f3F800000")):
        assert f"mov.f32 %n_{cell}, {seed};" in ptx, cell
    loop = ptx[ptx.index("$L_loop_2:"):ptx.index("$L_loop_end_3:")]
    assert "mov.f32 %n_fa, %n_fib__cell_0;" in loop            # cell 0 as the step began
    tail = ptx[ptx.index("$L_loop_end_3:"):]
    assert "mov.f32 %n_tot, %n_acc__cell_s;" in tail
    _ptxas(ptx, tmp_path)


def test_carried_state_run_time_cells(tmp_path):
    """A carrier indexed at run time keeps its cells in per-thread .local arrays over the range
    its indices reach: here j % 4 for the loop variable j, so 4 cells (16 bytes) per array."""
    ptx = _ptx(window_package(tmp_path / "w", 4))
    assert ".local .align 8 .b8 thl_win_cur[16];" in ptx and ".local .align 8 .b8 thl_win_next[16];" in ptx
    assert "st.local.f32" in ptx and "ld.local.f32" in ptx
    _ptxas(ptx, tmp_path)


def test_carried_state_index_must_be_bounded(tmp_path):
    """A run-time cell index with no bound from the axes (a value loaded from data) is refused."""
    d = scan_package(tmp_path / "c")
    f = next(d.glob("*.ir.json"))
    text = f.read_text().replace("Carry(name='fib', value='fs', index=(Literal(value=1, dtype='int'),)",
                                 "Carry(name='fib', value='fs', index=(CastExpr(dtype='int', expr=Var(name='fs')),)")
    f.write_text(text)
    with pytest.raises(NotImplementedError, match="must be bounded by axis extents"):
        _ptx(d)


def _lower_body(tmp_path, stmts, inputs=(("x", (1024,)),), out=("y", (1024,)), T=128):
    """Lower a one-axis Tile of ``stmts`` (a ragged probe kernel) and assemble it."""
    from sm90_ir import _graph, _write, axis
    tile = ir.Tile((axis("a0", out[1][0]),), tuple(stmts), T, 0, None, None, "m")
    g = _graph({n: (s, "f32") for n, s in inputs}, {}, out[0], out[1], "k_probe", tile)
    args = [{"name": n, "dtype": "f32", "shape": list(s), "seed": i} for i, (n, s) in enumerate(inputs)]
    args.append({"name": out[0], "dtype": "f32", "shape": list(out[1]), "output": True})
    kmeta = {"node": out[0], "arg_order": [n for n, _ in inputs] + [out[0]], "grid": [out[1][0] // T, 1, 1],
             "block": [T, 1, 1], "smem_bytes": 0, "zero_outputs": [], "args": args}
    d = _write(tmp_path / "k", "probe", "probe", "k_probe", g, kmeta, 0, 0)
    ptx = _ptx(d)
    _ptxas(ptx, tmp_path)
    return ptx


def test_runtime_forms_lower(tmp_path):
    """Run-time operands take the checked paths: a TMA destination chosen at run time gets the
    bound check that skips an overrunning box, a wait takes its phase from a register, a
    ZeroPrologue its word count from an index expression, a Select mixes literal and named arms."""
    L, V, B = synth.L, synth.V, synth.B
    stmts = [
        ir.Smem("buf", (4, 32, 32), "float", 1024),
        ir.Smem("bar", (2,), "uint64_t", 8),
        ir.TmaDescriptor("dx", "x", (32, 32), (32, 32), None, synth.F32T),
        ir.MbarrierInit("bar", L(1), B("%", V("a0"), L(2))),
        ir.Sync(0, None, False),
        ir.Let("slot", B("/", V("a0"), L(256)), ir.DataType("i32", "int32", 4)),
        ir.Cond(B("==", B("%", V("a0"), L(128)), L(0)), (
            ir.MbarrierArriveExpectTx("bar", L(4096), B("%", V("slot"), L(2))),
            ir.TmaLoad("buf", (V("slot"), L(0), L(0)), "dx", (L(0), L(0)), "bar", B("%", V("slot"), L(2))),
        ), ()),
        ir.MbarrierWait("bar", V("slot"), B("%", V("slot"), L(2))),
        ir.ZeroPrologue("z", B("*", V("slot"), L(0))),
        ir.Load(("v",), "x", (V("a0"),), synth.F32T),
        ir.Select("s", (ir.Branch(L(2.5, "float"), B(">", V("a0"), L(1000))), ir.Branch("v", None))),
        ir.Write("y", (V("a0"),), ("s",), synth.F32T, False, "NONE"),
    ]
    ptx = _lower_body(tmp_path, stmts, inputs=(("x", (1024,)), ("z", (1024,))))
    assert "setp.gt.u32" in ptx                        # the run-time destination bound
    assert "mbarrier.try_wait.parity.shared::cta.b64" in ptx and "selp.f32" in ptx


def test_carried_state_in_unrolled_inner_loop(tmp_path):
    """A carrier owned by an unrolled inner loop, its cells indexed by the outer unrolled
    variable -- cell indices fold to constants."""
    L, V = synth.L, synth.V
    inner = ir.Loop(synth.axis("k", 4), (
        ir.Pre("p", "acc", (V("c"),)),
        ir.Load(("v",), "x", (V("a0"),), synth.F32T),
        synth.assign("s", "add", "p", "v"),
        ir.Carry("acc", "s", (V("c"),), L(0.0, "float"), synth.F32T),
    ), True, False)
    outer = ir.Loop(synth.axis("c", 2), (inner, ir.Pre("fin", "acc", (V("c"),)),
                                         ir.Write("y", (V("a0"),), ("fin",), synth.F32T, False, "NONE")),
                    True, False)
    ptx = _lower_body(tmp_path, [outer])
    assert "%n_acc__cell_0" in ptx and "%n_acc__cell_1" in ptx
