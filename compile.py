"""Kernel IR in, sm_100a PTX out.

    python3 compile.py <kernel>.ir.json > out.ptx

Reads one Emmy Kernel IR file and the meta.json launch contract next to it,
and prints one PTX module on stdout (nothing else goes to stdout).  Any
failure raises: a non-zero exit with a traceback on stderr and no partial
PTX -- the contract of the reference's compile.py:9-19.
"""

import os
import sys

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "thompiler-emmy-hackathon_b200"))

from thompiler.compiler import compile_kernel  # noqa: E402
from thompiler.load import load  # noqa: E402


def main() -> None:
    if len(sys.argv) != 2:
        sys.exit("usage: python3 compile.py <kernel>.ir.json > out.ptx")
    ptx = compile_kernel(load(sys.argv[1]))
    sys.stdout.write(ptx)


if __name__ == "__main__":
    main()
