"""Compile latency of ``compile.py``, this backend against the reference (a side metric).

Run in a container that has the reference checkout (its compile.py runs unmodified, with the
clean-room emmy stand-in oracle/emmy_shim on the path, as tests/golden/make_golden.py runs it):

    python oracle/compile_latency.py --reference <reference checkout> [--repeat 3]

For every kernel of the 19 golden packages it reports the median wall time of one
``python3 compile.py <kernel>.ir.json`` process for each compiler (interpreter start-up
included, as a runner calling the compiler pays it), twice: with Python's bytecode cache
(warmed once, kept under a temporary PYTHONPYCACHEPREFIX so nothing is written beside either
compiler's sources) and without one (every import compiles its source); and, for this backend,
the median time of the compile call alone inside one process.  Test infrastructure: it
measures, it ships nothing.
"""

from __future__ import annotations

import argparse
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden" / "packages"


def _proc_ms(cmd: list[str], env: dict, repeat: int) -> float:
    ts = []
    for _ in range(repeat):
        t = time.perf_counter()
        subprocess.run(cmd, capture_output=True, env=env, check=True)
        ts.append((time.perf_counter() - t) * 1e3)
    return statistics.median(ts)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="a checkout of the reference repository")
    ap.add_argument("--repeat", type=int, default=3)
    args = ap.parse_args()
    sys.path.insert(0, str(REPO / "thompiler-emmy-hackathon_b200"))
    from thompiler.compiler import compile_kernel
    from thompiler.load import load
    base = {k: v for k, v in os.environ.items() if k not in ("PYTHONDONTWRITEBYTECODE", "PYTHONPYCACHEPREFIX")}
    cache = tempfile.mkdtemp(prefix="pycache_")
    envs = {"cached": dict(base, PYTHONPYCACHEPREFIX=cache), "uncached": dict(base, PYTHONDONTWRITEBYTECODE="1")}
    ref_py = str(REPO / "oracle" / "emmy_shim")
    ours_cmd = [sys.executable, str(REPO / "compile.py")]
    ref_cmd = [sys.executable, str(Path(args.reference) / "compile.py")]
    rows = []
    for d in sorted(p for p in GOLDEN.iterdir() if (p / "meta.json").exists()):
        for ir in sorted(d.glob("*.ir.json")):
            row = [f"{d.name}/{ir.name.removesuffix('.ir.json')}"]
            for mode in ("cached", "uncached"):
                env = envs[mode]
                renv = dict(env, PYTHONPATH=ref_py)
                if mode == "cached":                    # warm both caches once
                    subprocess.run(ours_cmd + [str(ir)], capture_output=True, env=env, check=True)
                    subprocess.run(ref_cmd + [str(ir)], capture_output=True, env=renv, check=True)
                row += [_proc_ms(ours_cmd + [str(ir)], env, args.repeat), _proc_ms(ref_cmd + [str(ir)], renv, args.repeat)]
            ts = []
            for _ in range(args.repeat):
                t = time.perf_counter()
                compile_kernel(load(str(ir)))
                ts.append((time.perf_counter() - t) * 1e3)
            rows.append((*row, statistics.median(ts)))
    print("| kernel | ours, cached (ms) | reference, cached (ms) | ours, no cache (ms) | reference, no cache (ms) "
          "| ours, compile call (ms) |")
    print("|---|---|---|---|---|---|")
    for name, *v in rows:
        print(f"| {name} | {v[0]:.0f} | {v[1]:.0f} | {v[2]:.0f} | {v[3]:.0f} | {v[4]:.1f} |")
    med = [statistics.median(col) for col in zip(*[r[1:] for r in rows])]
    print(f"| median of {len(rows)} kernels | {med[0]:.0f} | {med[1]:.0f} | {med[2]:.0f} | {med[3]:.0f} | {med[4]:.1f} |")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
