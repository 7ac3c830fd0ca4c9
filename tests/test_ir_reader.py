"""The IR reader: every shipped Kernel IR parses, without eval, into the
statement classes the walker dispatches on."""

import json

import pytest

from conftest import GOLDEN, PACKAGES
from thompiler import ir
from thompiler.load import load


def all_ir_files():
    return sorted(p for d in PACKAGES for p in (GOLDEN / d).glob("*.ir.json"))


@pytest.mark.parametrize("path", all_ir_files(), ids=lambda p: f"{p.parent.name}/{p.stem}")
def test_parses(path):
    g = ir.Graph.from_dict(json.loads(path.read_text()))
    assert len(g.kernels) == 1
    k = g.kernels[0]
    assert isinstance(k.body[0], ir.Tile)
    kinds = {type(s).__name__ for s in ir.walk_stmts(k.body)}
    assert "Opaque" not in kinds


def test_kernel_info_follows_arg_order():
    info = load(GOLDEN / "m01_matmul_512" / "k_matmul_2967be.ir.json")
    assert [p.name for p in info.params] == ["x1", "x0", "matmul"]     # meta order, not IR order
    assert info.dynamic_smem_bytes == 73728
    assert info.param("matmul").written and not info.param("x0").written
    assert info.grid == (128, 1, 1) and info.block == (512, 1, 1)


def test_unknown_constructor_is_kept_opaque():
    s = ir.parse_stmt("TensorMapPrefetch(desc='d', src_buffer='x', index=(Var(name='i'),))")
    assert isinstance(s, ir.Opaque) and s.kind == "TensorMapPrefetch"
    assert dict(s.fields)["src_buffer"] == "x"


def test_block_scale_load_is_read():
    s = ir.parse_stmt("BlockScaleLoad(frag='sf', src_buffer='x', src_index=(Var(name='i'), Literal(value=0, "
                      "dtype='int')), role='a', ldm=64)")
    assert isinstance(s, ir.BlockScaleLoad) and (s.frag, s.src_buffer, s.role, s.ldm) == ("sf", "x", "a", 64)
    assert s.src_index == (ir.Var("i"), ir.Literal(0, "int"))


def test_rejects_non_constructor_syntax():
    with pytest.raises(ir.IRSyntaxError):
        ir.parse_stmt("__import__('os').system('true')")
    with pytest.raises(ir.IRSyntaxError):
        ir.parse_stmt("Var(name=x)")


def test_elementwise_identities():
    assert ir.ElementwiseImpl("add").identity == 0.0
    assert ir.ElementwiseImpl("multiply").identity == 1.0
    assert ir.ElementwiseImpl("maximum").identity == -1e30
    assert ir.ElementwiseImpl("exp").arity == 1


def test_records_behave_as_frozen_dataclasses():
    """The IR's node classes are frozen records: positional or keyword construction with the
    declared defaults, field-wise equality and hash, the dataclass repr, no assignment, and
    construction errors that name the class (the reader turns them into IRSyntaxError)."""
    import dataclasses

    from thompiler.synth import F32T, L, V
    a = ir.Load(("v",), "x", (V("i"),), F32T)
    b = ir.Load(names=("v",), input="x", index=(V("i"),), dtype=F32T)
    assert a == b and hash(a) == hash(b) and a != ir.Load(("w",), "x", (V("i"),), F32T)
    assert ir.field_names(a) == ("names", "input", "index", "dtype") and ir.is_record(a)
    assert not ir.is_record(ir.Load)
    assert repr(L(3)) == "Literal(value=3, dtype='int')"
    st = ir.RegStore("y", (L(0), L(0)), "c", (16, 8, 16))
    assert (st.ldm, st.epilogue, st.extra_frags, st.atomic, st.swizzle) == (0, None, (), False, "NONE")
    assert ir.Opaque("K").fields == ()
    assert ir.Tile.extents.fget is not None                     # properties survive
    with pytest.raises(dataclasses.FrozenInstanceError):
        a.input = "y"
    with pytest.raises(TypeError, match="Load.__init__\\(\\) got an unexpected keyword argument 'bogus'"):
        ir.Load(("v",), "x", (), F32T, bogus=1)
    with pytest.raises(TypeError, match="missing 1 required positional argument: 'input'"):
        ir.Load(("v",))
    with pytest.raises(TypeError, match="multiple values for argument 'names'"):
        ir.Load(("v",), names=("w",), input="x", index=())
    with pytest.raises(ir.IRSyntaxError, match="Write: "):
        ir.parse_stmt("Write(output='y', index=(), values=(), dtype=None)")
