"""Problem packages: compile, run on the local B200 and check -- the local
counterpart of the reference's submit.py and scripts/check_all.py.

A package is a folder with ``meta.json`` (launch contract, args, tolerance),
one ``<entry>.ir.json`` per kernel and, for open problems, ``expected.npz``.
Kernels run in meta.json order; a buffer marked ``intermediate`` is the
output of an earlier kernel (submit.py:112-122).  Inputs are
``default_rng(seed).standard_normal(shape)`` in the arg's dtype, constants
come from ``data``, outputs start at zero and ``zero_outputs`` are re-zeroed
before every launch (docs/API.md:44-52).

Unlike submit.py, which casts every output to f32 before ``allclose``
(submit.py:148), outputs are compared in their own dtype, so f64 results
are checked to f64 precision.

    python -m thompiler.problems <package dir>... [--meta-launch] [--generic]
"""

from __future__ import annotations

import argparse
import json
import sys
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from thompiler import runner
from thompiler.compiler import compile_kernel
from thompiler.load import load

NP_DTYPES = {"f32": np.float32, "f16": np.float16, "f64": np.float64, "i32": np.int32, "i64": np.int64,
             "u8": np.uint8}


@dataclass
class Package:
    dir: Path
    meta: dict
    expected: dict | None

    @property
    def name(self) -> str:
        return self.meta.get("id", self.dir.name)

    def ir_path(self, entry: str) -> Path:
        return self.dir / f"{entry}.ir.json"


def load_package(pdir: str | Path) -> Package:
    pdir = Path(pdir)
    meta = json.loads((pdir / "meta.json").read_text())
    exp = pdir / "expected.npz"
    return Package(pdir, meta, dict(np.load(exp)) if exp.exists() else None)


def seeded_input(shape, seed: int, dtype: str, init: dict | None = None) -> np.ndarray:
    """The runner's seeded input (standard normal), or the distribution an
    ``init`` record names (synthetic packages: ``uniform`` low/high,
    ``normal`` mean/std, ``integers`` low..high inclusive)."""
    shape = list(shape) or [1]
    if init is None:
        return np.random.default_rng(seed).standard_normal(shape).astype(NP_DTYPES[dtype])
    rng = np.random.default_rng(init.get("seed", seed))
    if init["dist"] == "uniform":
        return rng.uniform(init.get("low", 0.0), init.get("high", 1.0), shape).astype(NP_DTYPES[dtype])
    if init["dist"] == "integers":
        return rng.integers(init.get("low", -2), init.get("high", 2) + 1, shape).astype(NP_DTYPES[dtype])
    if init["dist"] == "normal":
        return (rng.standard_normal(shape) * init.get("std", 1.0) + init.get("mean", 0.0)).astype(NP_DTYPES[dtype])
    raise ValueError(f"input distribution {init['dist']!r}")


def make_inputs(pkg: Package) -> dict[str, np.ndarray]:
    """Every seeded / constant input of the package, by buffer name."""
    out: dict[str, np.ndarray] = {}
    for k in pkg.meta["kernels"]:
        for a in k["args"]:
            if a.get("output") or a.get("intermediate") or a["name"] in out:
                continue
            if "data" in a:
                out[a["name"]] = np.asarray(a["data"], dtype=NP_DTYPES[a["dtype"]]).reshape(a["shape"])
            else:
                out[a["name"]] = seeded_input(a["shape"], a.get("seed", 0), a["dtype"], a.get("init"))
    return out


def compile_package(pkg: Package, tuned: bool = True) -> dict[str, str]:
    """entry -> PTX for every kernel of the package (this compiler)."""
    return {k["entry"]: compile_kernel(load(pkg.ir_path(k["entry"])), tuned=tuned) for k in pkg.meta["kernels"]}


def run_package(pkg: Package, ptx: dict[str, str], inputs: dict | None = None, honour_meta: bool = False,
                warmup: int = 0, iters: int = 1, device: int = 0) -> dict:
    """Run every kernel through the runner's host-buffer call (thr_run).
    Returns {"outputs": {name: array}, "median_us": {entry: us}, "launch": {entry: plan}}."""
    runner.init(device)
    inputs = dict(make_inputs(pkg) if inputs is None else inputs)
    produced: dict[str, np.ndarray] = {}
    times, plans = {}, {}
    for k in pkg.meta["kernels"]:
        mod = runner.load_module(ptx[k["entry"]], device)
        try:
            fn = mod.function(k["entry"])
            plan = runner.plan_launch(mod, k, honour_meta=honour_meta)
            recs = {a["name"]: a for a in k["args"]}
            args = []
            for name in k["arg_order"]:
                a = recs[name]
                dt = NP_DTYPES[a["dtype"]]
                if a.get("output"):
                    arr = np.zeros(a["shape"], dtype=dt)
                    args.append({"array": arr, "output": True, "zero_each": name in k.get("zero_outputs", [])})
                elif a.get("intermediate"):
                    args.append({"array": np.ascontiguousarray(produced[name], dtype=dt)})
                else:
                    args.append({"array": np.ascontiguousarray(inputs[name], dtype=dt)})
            res = runner.run(fn, plan, args, warmup=warmup, iters=iters, arg_order=list(k["arg_order"]))
            if not res["ok"]:
                raise runner.RunnerError(res["stage"], res["stderr"])
            for name, a in zip(k["arg_order"], args):
                if a.get("output"):
                    produced[name] = a["array"]
            times[k["entry"]] = res["median_us"]
            plans[k["entry"]] = plan
        finally:
            mod.unload()
    return {"outputs": produced, "median_us": times, "launch": plans}


def compare(got: np.ndarray, want: np.ndarray, rtol: float, atol: float) -> tuple[bool, float]:
    got = np.asarray(got).reshape(want.shape)
    ok = bool(np.allclose(got, want, rtol=rtol, atol=atol, equal_nan=False))
    err = float(np.max(np.abs(got.astype(np.float64) - want.astype(np.float64)))) if want.size else 0.0
    return ok, err


def check_package(pkg: Package, result: dict) -> list[tuple[str, bool, float]]:
    rows = []
    for name, want in (pkg.expected or {}).items():
        ok, err = compare(result["outputs"][name], want, pkg.meta["rtol"], pkg.meta["atol"])
        rows.append((name, ok, err))
    return rows


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description="compile, run and check problem packages on the local GPU")
    ap.add_argument("packages", nargs="+")
    ap.add_argument("--meta-launch", action="store_true", help="ignore tuned launches; use meta.json's")
    ap.add_argument("--generic", action="store_true", help="generic lowering only (no tuned families)")
    args = ap.parse_args(argv)
    failed = 0
    for d in args.packages:
        pkg = load_package(d)
        try:
            res = run_package(pkg, compile_package(pkg, tuned=not args.generic), honour_meta=args.meta_launch)
        except Exception as e:  # report and continue
            print(f"FAIL  {pkg.name}: {e}")
            failed += 1
            continue
        for name, ok, err in check_package(pkg, res):
            print(f"{'PASS' if ok else 'FAIL'}  {pkg.name:24s} {name:12s} max abs err {err:.3e}  "
                  f"{sum(res['median_us'].values()):.1f} us")
            failed += not ok
    return 1 if failed else 0


if __name__ == "__main__":
    sys.exit(main())
