"""PTX text builder for one kernel.

The emitter knows PTX syntax, nothing about the IR: it hands out registers
and labels, collects instruction lines and module-scope declarations, and
renders the file at the end (``.reg`` declarations need final counts, so
the text is produced last).

Registers
  * temporaries: ``%p7`` (pred), ``%h3`` (b16), ``%r12`` (b32), ``%rd4``
    (b64), ``%f9`` (f32), ``%fd2`` (f64);
  * IR values: ``%n_<name>``; the same IR name always maps to the same
    register (accumulators and loop counters are rewritten in place) and a
    name keeps one register class for the whole kernel;
  * buffer base addresses: ``%g_<buffer>``.
``lane`` and ``warp`` (the thread's lane and warp within its CTA) are IR
builtins; they are computed once at kernel entry when the body reads them.
"""

from __future__ import annotations

import json

REG_CLASSES = ("pred", "b16", "b32", "b64", "f32", "f64")
_TEMP_PREFIX = {"pred": "%p", "b16": "%h", "b32": "%r", "b64": "%rd", "f32": "%f", "f64": "%fd"}

SIDECAR_TAG = "// @thompiler-launch "


class Emitter:
    def __init__(self) -> None:
        self.lines: list[str] = []
        self.module_decls: list[str] = []
        self.counts = {k: 0 for k in REG_CLASSES}
        self.named: dict[str, str] = {}        # register -> class
        self.nlabels = 0
        self.builtins: set[str] = set()        # "lane", "warp" when read
        self.sidecar: dict | None = None       # tuned launch, rendered as a comment
        self.entry_attrs: list[str] = []       # .maxntid / .minnctapersm ...
        self.local_decls: list[str] = []       # per-thread .local arrays, declared in the entry

    # ---- registers --------------------------------------------------------

    def tmp(self, cls: str) -> str:
        if cls not in _TEMP_PREFIX:
            raise NotImplementedError(f"register class {cls!r}")
        self.counts[cls] += 1
        return f"{_TEMP_PREFIX[cls]}{self.counts[cls]}"

    def tmps(self, cls: str, n: int) -> list[str]:
        return [self.tmp(cls) for _ in range(n)]

    def declare(self, reg: str, cls: str) -> str:
        if cls not in _TEMP_PREFIX:
            raise NotImplementedError(f"register class {cls!r}")
        have = self.named.setdefault(reg, cls)
        if have != cls:
            raise TypeError(f"{reg} is a .{have} register, used here as .{cls}")
        return reg

    def value(self, name: str, cls: str) -> str:
        """Register of IR value ``name`` (declared on first use)."""
        return self.declare(f"%n_{name}", cls)

    def has_value(self, name: str) -> bool:
        return f"%n_{name}" in self.named or name in ("lane", "warp")

    def get(self, name: str) -> str:
        """Register of an IR value that must already exist."""
        if name in ("lane", "warp"):
            self.builtins.add(name)
            return self.declare(f"%n_{name}", "b32")
        reg = f"%n_{name}"
        if reg not in self.named:
            raise KeyError(f"IR value {name!r} is read before it is defined")
        return reg

    def cls_of(self, name: str) -> str:
        return self.named[self.get(name)]

    def buffer_reg(self, buffer: str) -> str:
        return self.declare(f"%g_{buffer}", "b64")

    # ---- text ------------------------------------------------------------

    def ins(self, text: str) -> None:
        self.lines.append(f"\t{text};")

    def raw(self, text: str) -> None:
        self.lines.append(text)

    def note(self, text: str) -> None:
        clean = text.encode("ascii", "replace").decode("ascii").replace("\n", " ")
        self.lines.append(f"\t// {clean}")

    def label(self, hint: str) -> str:
        self.nlabels += 1
        return f"$L_{hint}_{self.nlabels}"

    def place(self, label: str) -> None:
        self.lines.append(f"{label}:")

    def local(self, decl: str) -> None:
        """A declaration at the top of the entry's body (a per-thread .local array)."""
        line = decl if decl.rstrip().endswith(";") else f"{decl};"
        if line not in self.local_decls:
            self.local_decls.append(line)

    def module(self, decl: str) -> None:
        line = decl if decl.rstrip().endswith(";") else f"{decl};"
        if line not in self.module_decls:
            self.module_decls.append(line)

    # ---- output ----------------------------------------------------------

    def render(self, header: list[str], entry: str, params: list[str]) -> str:
        prologue = []
        if "lane" in self.builtins:
            prologue += ["\tmov.u32 %n_lane, %tid.x;", "\tand.b32 %n_lane, %n_lane, 31;"]
        if "warp" in self.builtins:
            prologue += ["\tmov.u32 %n_warp, %tid.x;", "\tshr.u32 %n_warp, %n_warp, 5;"]
        decls = [f"\t.reg .{cls} {_TEMP_PREFIX[cls]}<{n + 1}>;"
                 for cls, n in self.counts.items() if n]
        for cls in REG_CLASSES:
            regs = [r for r, c in self.named.items() if c == cls]
            for i in range(0, len(regs), 16):
                decls.append(f"\t.reg .{cls} {', '.join(regs[i:i + 16])};")
        side = []
        if self.sidecar is not None:
            side = [SIDECAR_TAG + json.dumps(self.sidecar, sort_keys=True, separators=(",", ":"))]
        sig = [f".visible .entry {entry}(", ",\n".join(f"\t{p}" for p in params), ")"]
        text = "\n".join([*header, *side, "", *self.module_decls, "", *sig, *self.entry_attrs,
                          "{", *decls, *(f"\t{d}" for d in self.local_decls), "", *prologue, *self.lines, "}", ""])
        if not text.isascii():
            raise ValueError("PTX must be ASCII")
        return text


def read_sidecar(ptx: str) -> dict | None:
    """The tuned-launch record a PTX file carries, or None."""
    for line in ptx.splitlines()[:8]:
        if line.startswith(SIDECAR_TAG):
            return json.loads(line[len(SIDECAR_TAG):])
    return None
