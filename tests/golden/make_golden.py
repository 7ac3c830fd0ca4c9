"""Build the golden fixtures under tests/golden/packages/ from the reference.

Run where the reference checkout is present (the fixtures it writes are
all the tests need; nothing reads the checkout at test time):

    python tests/golden/make_golden.py --reference <reference checkout>

For every problem package of the reference (problems/ and tests/problems/)
it writes, into tests/golden/packages/<id>/:

  * meta.json, <entry>.ir.json, expected.npz -- copied byte for byte: the
    reference's own launch contracts, Kernel IR and golden outputs;
  * <entry>.ref.ptx -- the reference compiler's own PTX for the kernel,
    produced by running the reference's unmodified compile.py with the
    clean-room emmy stand-in (oracle/emmy_shim) on the path;
  * oracle.npz -- every buffer the oracle interpreter (oracle/interp.py)
    produces for the package's seeded inputs; the script checks it against
    expected.npz with the package's tolerance before writing it.

MANIFEST.json records the sha256 of each copied file and the generator.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle.interp import run_package  # noqa: E402


def sha(p: Path) -> str:
    return hashlib.sha256(p.read_bytes()).hexdigest()


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="a checkout of the reference repository")
    args = ap.parse_args()
    ref = Path(args.reference)
    out_root = HERE / "packages"
    out_root.mkdir(exist_ok=True)
    manifest = {"generator": "tests/golden/make_golden.py", "packages": {}}
    env = dict(os.environ, PYTHONPATH=str(REPO / "oracle" / "emmy_shim"))
    dirs = sorted(d for root in (ref / "problems", ref / "tests" / "problems") for d in root.iterdir()
                  if (d / "meta.json").exists())
    for d in dirs:
        dst = out_root / d.name
        if dst.exists():
            shutil.rmtree(dst)
        dst.mkdir()
        files = {}
        for f in [d / "meta.json", d / "expected.npz", *sorted(d.glob("*.ir.json"))]:
            shutil.copyfile(f, dst / f.name)
            files[f.name] = sha(f)
        meta = json.loads((d / "meta.json").read_text())
        for k in meta["kernels"]:
            r = subprocess.run([sys.executable, str(ref / "compile.py"), str(d / f"{k['entry']}.ir.json")],
                               capture_output=True, text=True, env=env, check=True)
            (dst / f"{k['entry']}.ref.ptx").write_text(r.stdout)
        produced = run_package(dst)
        exp = dict(np.load(d / "expected.npz"))
        for name, want in exp.items():
            got = produced[name].reshape(want.shape)
            if not np.allclose(got, want, rtol=meta["rtol"], atol=meta["atol"]):
                raise SystemExit(f"oracle disagrees with expected.npz on {d.name}/{name}")
        np.savez_compressed(dst / "oracle.npz", **produced)
        manifest["packages"][d.name] = {"source": str(d.relative_to(ref)), "files": files}
        print(f"ok  {d.name}")
    (HERE / "MANIFEST.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    return 0


if __name__ == "__main__":
    sys.exit(main())
