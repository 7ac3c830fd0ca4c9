"""Bulk tensor copies and mbarriers: TmaDescriptor, TmaLoad, Mbarrier*, SetMaxNReg.

The IR reference (TASK.md:120-128 of the reference) defines these for sm_90 and newer; the
reference compiler has no handler for them.  Here they lower onto sm_100a directly:

* ``TmaDescriptor`` renders no code: it declares a 128-byte module global ``thc_tmap_<name>``
  and records, in the module's launch sidecar (``ir_tmaps``), the tensor map the runner encodes
  into it before every launch from the buffer's device pointer: the IR's row-major
  ``src_shape`` / ``box_extents`` become innermost-first dims / box, byte strides of the outer
  dims, and the swizzle (none / 32 / 64 / 128 bytes).  What the TMA unit rejects or faults on
  is refused at compile time: a box side above 256, an inner box or row not a multiple of
  16 bytes, an inner box wider than its swizzle span.
* ``TmaLoad`` is one ``cp.async.bulk.tensor`` (the thread that executes the statement issues
  it) into the Smem element at ``smem_index``, completing on the mbarrier slot.  Coordinates
  are the IR's row-major order, reversed for the instruction.  The copy is skipped, and bit
  0 of the module's error word ``thc_error`` set, when its innermost coordinate is not a
  16-byte multiple, its destination not 128-byte aligned, or its box would run past the Smem
  array (the forms that fault): the consumer's bounded wait then runs out instead of the GPU
  faulting.
* ``MbarrierInit`` is executed by thread (0, 0, 0) only ("once in the kernel prologue"),
  followed by ``fence.mbarrier_init``; ``MbarrierArriveExpectTx`` / ``MbarrierArrive`` arrive
  on the slot; ``MbarrierWait`` polls ``mbarrier.try_wait.parity`` for ``phase & 1`` at most
  ``WAIT_LIMIT`` times, then sets bit 1 of ``thc_error`` and goes on -- no wait can hang.
* ``SetMaxNReg`` is ``setmaxnreg.{inc,dec}.sync.aligned.u32`` (a multiple of 8 in 24..256).

An mbarrier array is an Smem array of 8-byte elements; a slot is an index into it.
"""

from __future__ import annotations

from math import prod
from typing import TYPE_CHECKING

from thompiler import ir
from thompiler.lowering import expr
from thompiler.lowering.address import SharedArray, flat_index, shared_element_address
from thompiler.lowering.types import dtype_of

if TYPE_CHECKING:
    from thompiler.walk import Walker

WAIT_LIMIT = 1 << 18          # try_wait rounds (~4 us each while the phase is open): ~1 s
ERROR_WORD = "thc_error"
ERR_TMA_SKIPPED = 1
ERR_WAIT_TIMEOUT = 2
TMAP_DTYPES = {"f16": "f16", "bf16": "bf16", "f32": "f32"}
_SWIZZLE = {None: 0, "": 0, "NONE": 0, 0: 0, "B32": 1, 32: 1, "B64": 2, 64: 2, "B128": 3, 128: 3}
_SWIZZLE_SPAN = {0: None, 1: 32, 2: 64, 3: 128}


def _error_word(w: "Walker") -> str:
    w.em.module(f".global .align 4 .u32 {ERROR_WORD}")
    side = w.em.sidecar if w.em.sidecar is not None else {}
    side["error_word"] = ERROR_WORD
    w.em.sidecar = side
    r = w.em.tmp("b64")
    w.em.ins(f"mov.u64 {r}, {ERROR_WORD}")
    return r


def _flag(w: "Walker", bit: int, pred: str | None = None) -> None:
    """Set ``bit`` of the error word (under ``pred`` when given)."""
    r = _error_word(w)
    g = f"@{pred} " if pred else ""
    w.em.ins(f"{g}red.global.or.b32 [{r}], {bit}")


def _mbar_address(w: "Walker", name: str, slot) -> str:
    arr = w.smem.get(name)
    if arr is None:
        raise ValueError(f"mbarrier {name} is not a declared Smem array")
    if arr.ty.nbytes != 8:
        raise TypeError(f"mbarrier array {name} has {arr.ty.nbytes}-byte elements, not 8")
    idx = (0,) * len(arr.extents) if slot is None else (slot if isinstance(slot, tuple) else (slot,))
    if len(idx) != len(arr.extents):
        idx = (0,) * (len(arr.extents) - len(idx)) + tuple(idx)
    return shared_element_address(w, arr, flat_index(w, arr.extents, tuple(idx), name))


def _tmap_global(name: str) -> str:
    return f"thc_tmap_{name}"


def emit_tma_descriptor(w: "Walker", d: ir.TmaDescriptor) -> None:
    em = w.em
    em.note(d.pretty())
    p = w.kernel.param(d.src_buf)
    if p is None:
        raise ValueError(f"TmaDescriptor {d.name}: {d.src_buf} is not a kernel buffer")
    ty = dtype_of(d.dtype if d.dtype is not None else p.ty.name, f"TmaDescriptor {d.name}")
    if ty.name not in TMAP_DTYPES or ty is not p.ty:
        raise NotImplementedError(f"TmaDescriptor {d.name}: {ty.name} tensor maps of a {p.ty.name} buffer")
    shape = tuple(int(x) for x in d.src_shape)
    box = tuple(int(x) for x in d.box_extents)
    if not 1 <= len(shape) <= 5 or len(box) != len(shape):
        raise ValueError(f"TmaDescriptor {d.name}: rank {len(shape)} shape with a rank {len(box)} box")
    if prod(shape) != p.nelems:
        raise ValueError(f"TmaDescriptor {d.name}: shape {shape} does not cover {d.src_buf} ({p.nelems} elements)")
    swz = _SWIZZLE.get(d.swizzle if not isinstance(d.swizzle, str) else d.swizzle.upper())
    if swz is None:
        raise NotImplementedError(f"TmaDescriptor {d.name}: swizzle {d.swizzle!r}")
    esz = ty.nbytes
    if any(not 1 <= b <= 256 for b in box):
        raise ValueError(f"TmaDescriptor {d.name}: box {box} has a side outside 1..256")
    if (box[-1] * esz) % 16:
        raise ValueError(f"TmaDescriptor {d.name}: inner box of {box[-1] * esz} bytes is not a multiple of 16")
    span = _SWIZZLE_SPAN[swz]
    if span is not None and box[-1] * esz > span:
        raise ValueError(f"TmaDescriptor {d.name}: inner box of {box[-1] * esz} bytes is wider than the "
                         f"{span}-byte swizzle")
    if len(shape) > 1 and (shape[-1] * esz) % 16:
        raise ValueError(f"TmaDescriptor {d.name}: rows of {shape[-1] * esz} bytes are not a multiple of 16")
    dims = list(reversed(shape))
    strides, acc = [], esz
    for n in dims[:-1]:
        acc *= n
        strides.append(acc)
    spec = {"global": _tmap_global(d.name), "param": d.src_buf, "dtype": TMAP_DTYPES[ty.name], "dims": dims,
            "strides": strides, "box": list(reversed(box)), "swizzle": swz}
    em.module(f".global .align 64 .b8 {spec['global']}[128]")
    side = em.sidecar if em.sidecar is not None else {}
    maps = side.setdefault("ir_tmaps", [])
    if any(m["global"] == spec["global"] for m in maps):
        raise ValueError(f"TmaDescriptor {d.name} declared twice")
    maps.append(spec)
    em.sidecar = side
    w.tma_descs = getattr(w, "tma_descs", {})
    w.tma_descs[d.name] = (spec, ty, box)


def emit_tma_load(w: "Walker", t: ir.TmaLoad) -> None:
    em = w.em
    em.note(t.pretty())
    descs = getattr(w, "tma_descs", {})
    if t.desc not in descs:
        raise ValueError(f"TmaLoad: descriptor {t.desc} is not declared before use")
    spec, ty, box = descs[t.desc]
    arr: SharedArray | None = w.smem.get(t.smem)
    if arr is None:
        raise ValueError(f"TmaLoad: {t.smem} is not a declared Smem array")
    coords = tuple(t.coords)
    if len(coords) != len(box):
        raise ValueError(f"TmaLoad: {len(coords)} coordinates for a rank {len(box)} descriptor")
    box_bytes = prod(box) * ty.nbytes
    if box_bytes > arr.nbytes:
        raise ValueError(f"TmaLoad: a {box_bytes}-byte box does not fit Smem {t.smem} ({arr.nbytes} bytes)")
    dst_flat = flat_index(w, arr.extents, tuple(t.smem_index), t.smem)
    last = arr.nbytes - box_bytes                 # the last byte offset a box may start at
    if expr.is_imm(dst_flat) and int(dst_flat) * arr.ty.nbytes > last:
        raise ValueError(f"TmaLoad: a {box_bytes}-byte box at element {dst_flat} overruns Smem {t.smem}")
    dst = shared_element_address(w, arr, dst_flat)
    mbar = _mbar_address(w, t.mbar, t.mbar_slot)
    ops = [expr.int_operand(w, c) for c in reversed(coords)]
    # the forms that fault: an innermost coordinate off a 16-byte boundary, a destination off 128
    bad = em.tmp("pred")
    x = ops[0]
    inner_mask = (16 // ty.nbytes) - 1 if ty.nbytes < 16 else 0
    if expr.is_imm(x):
        if int(x) & inner_mask:
            raise ValueError(f"TmaLoad: innermost coordinate {x} is not a multiple of {inner_mask + 1} elements")
        em.ins(f"setp.ne.u32 {bad}, 0, 0")
    else:
        m = em.tmp("b32")
        em.ins(f"and.b32 {m}, {x}, {inner_mask}")
        em.ins(f"setp.ne.u32 {bad}, {m}, 0")
    da = em.tmp("b32")
    dst_base, _, dst_off = dst.partition("+")
    if dst_base.startswith("%"):
        em.ins(f"add.u32 {da}, {dst_base}, {dst_off or 0}")
    else:
        em.ins(f"mov.u32 {da}, {dst_base}")
        if dst_off:
            em.ins(f"add.u32 {da}, {da}, {dst_off}")
    al, bad2 = em.tmp("b32"), em.tmp("pred")
    em.ins(f"and.b32 {al}, {da}, 127")
    em.ins(f"setp.ne.u32 {bad2}, {al}, 0")
    em.ins(f"or.pred {bad}, {bad}, {bad2}")
    if not expr.is_imm(dst_flat):                 # a run-time index: the box must stay inside the array
        off = em.tmp("b32")
        em.ins(f"mul.lo.s32 {off}, {dst_flat}, {arr.ty.nbytes}")
        em.ins(f"setp.gt.u32 {bad2}, {off}, {last}")
        em.ins(f"or.pred {bad}, {bad}, {bad2}")
    _flag(w, ERR_TMA_SKIPPED, bad)
    tm = em.tmp("b64")
    em.ins(f"mov.u64 {tm}, {spec['global']}")
    em.ins(f"cvta.global.u64 {tm}, {tm}")
    em.ins(f"@!{bad} cp.async.bulk.tensor.{len(box)}d.shared::cluster.global.mbarrier::complete_tx::bytes "
           f"[{da}], [{tm}, {{{', '.join(ops)}}}], [{mbar}]")


def _first_thread(w: "Walker") -> str:
    em = w.em
    t, p = em.tmp("b32"), em.tmp("pred")
    em.ins(f"mov.u32 {t}, %tid.x")
    u = em.tmp("b32")
    em.ins(f"mov.u32 {u}, %tid.y")
    em.ins(f"or.b32 {t}, {t}, {u}")
    em.ins(f"mov.u32 {u}, %tid.z")
    em.ins(f"or.b32 {t}, {t}, {u}")
    em.ins(f"setp.eq.u32 {p}, {t}, 0")
    return p


def emit_mbarrier_init(w: "Walker", s: ir.MbarrierInit) -> None:
    em = w.em
    em.note(s.pretty())
    addr = _mbar_address(w, s.mbar, s.slot)
    count = expr.int_operand(w, s.count)
    if expr.is_imm(count) and not 1 <= int(count) < (1 << 20):
        raise ValueError(f"MbarrierInit {s.mbar}: arrival count {count} outside 1..2^20-1")
    p = _first_thread(w)
    em.ins(f"@{p} mbarrier.init.shared::cta.b64 [{addr}], {count}")
    em.ins(f"@{p} fence.mbarrier_init.release.cluster")


def emit_mbarrier_arrive_expect_tx(w: "Walker", s: ir.MbarrierArriveExpectTx) -> None:
    em = w.em
    em.note(s.pretty())
    addr = _mbar_address(w, s.mbar, s.slot)
    nbytes = expr.int_operand(w, s.bytes_)
    if expr.is_imm(nbytes) and not 0 <= int(nbytes) < (1 << 20):
        raise ValueError(f"MbarrierArriveExpectTx {s.mbar}: {nbytes} bytes outside the transaction range")
    em.ins(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [{addr}], {nbytes}")


def emit_mbarrier_arrive(w: "Walker", s: ir.MbarrierArrive) -> None:
    em = w.em
    em.note(s.pretty())
    em.ins(f"mbarrier.arrive.shared::cta.b64 _, [{_mbar_address(w, s.mbar, s.slot)}]")


def emit_mbarrier_wait(w: "Walker", s: ir.MbarrierWait) -> None:
    em = w.em
    em.note(s.pretty())
    addr = _mbar_address(w, s.mbar, s.slot)
    phase = expr.int_operand(w, s.phase)
    par = em.tmp("b32")
    if expr.is_imm(phase):
        em.ins(f"mov.u32 {par}, {int(phase) & 1}")
    else:
        em.ins(f"and.b32 {par}, {phase}, 1")
    top, done = em.label("mbw"), em.label("mbw_done")
    n, ok, more = em.tmp("b32"), em.tmp("pred"), em.tmp("pred")
    em.ins(f"mov.u32 {n}, 0")
    em.place(top)
    em.ins(f"mbarrier.try_wait.parity.shared::cta.b64 {ok}, [{addr}], {par}")
    em.ins(f"@{ok} bra {done}")
    em.ins(f"add.u32 {n}, {n}, 1")
    em.ins(f"setp.lt.u32 {more}, {n}, {WAIT_LIMIT}")
    em.ins(f"@{more} bra {top}")
    _flag(w, ERR_WAIT_TIMEOUT)
    em.place(done)


def emit_set_max_nreg(w: "Walker", s: ir.SetMaxNReg) -> None:
    em = w.em
    em.note(s.pretty())
    n = int(s.count)
    if n % 8 or not 24 <= n <= 256:
        raise ValueError(f"SetMaxNReg: {n} registers (a multiple of 8 in 24..256)")
    d = s.direction
    if isinstance(d, str):
        d = d.lower()
    if d in ("inc", "increase", "up", 1, True):
        op = "inc"
    elif d in ("dec", "decrease", "down", -1, False):
        op = "dec"
    else:
        raise ValueError(f"SetMaxNReg: direction {s.direction!r}")
    em.ins(f"setmaxnreg.{op}.sync.aligned.u32 {n}")
