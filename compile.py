"""Kernel IR in, sm_100a PTX out.

    python3 compile.py <kernel>.ir.json > out.ptx
    python3 compile.py --generic <kernel>.ir.json > out.ptx   # statement-by-statement lowering only

Reads one Emmy Kernel IR file and the meta.json launch contract next to it,
and prints one PTX module on stdout (nothing else goes to stdout).  Any
failure raises: a non-zero exit with a traceback on stderr and no partial
PTX -- the contract of the reference's compile.py:9-19.  Without flags the
output depends on the IR and meta.json alone (no environment variable is
read).
"""

import os
import sys

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "thompiler-emmy-hackathon_b200"))

from thompiler.compiler import compile_kernel  # noqa: E402
from thompiler.load import load  # noqa: E402


def main() -> None:
    args = sys.argv[1:]
    generic = args[:1] == ["--generic"]
    if generic:
        args = args[1:]
    if len(args) != 1:
        sys.exit("usage: python3 compile.py [--generic] <kernel>.ir.json > out.ptx")
    ptx = compile_kernel(load(args[0]), tuned=not generic)
    sys.stdout.write(ptx)


if __name__ == "__main__":
    main()
