"""Hand-tuned sm_100a kernel families, chosen by recognising the IR's shape.

``recognise(kernel)`` returns an object with ``emit() -> str`` for a kernel
this backend has a tuned body for, else None (generic lowering).
"""

from __future__ import annotations

from thompiler.load import KernelInfo


def recognise(kernel: KernelInfo):
    from thompiler.families import attention, attention_pair, matmul, matmul_pair, pointwise, strided
    for fam in (strided, matmul_pair, matmul, attention_pair, attention, pointwise):
        k = fam.recognise(kernel)
        if k is not None:
            return k
    return None
