"""Tuning switches of the tuned families, set from Python only.

The compiler reads no environment variable: ``compile.py`` with no flags emits
the same PTX for the same IR wherever it runs.  Tests and experiments change
these attributes in-process (for example pytest's
``monkeypatch.setattr(TUNING, "matmul_pair", False)``); the defaults are the
measured best choices.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass
class Tuning:
    # f16 matmul: CTA pairs (cta_group::2) where the shape allows; False: the single-CTA kernel
    matmul_pair: bool = True
    # force the matmul tile width (0: chosen per shape)
    matmul_bn: int = 0
    # force the number of matmul K stages (0: as many as shared memory holds)
    matmul_stages: int = 0
    # cut a partial last wave of matmul tiles along K
    matmul_split_tail: bool = True
    # attention: P handed to the MMA warp in this many parts along the keys (1, 2 or 4)
    attention_p_parts: int = 2
    # attention: of every 8 score pairs, this many take 2^x from a polynomial on the FMA pipe
    attention_poly_pairs: int = 0


TUNING = Tuning()
