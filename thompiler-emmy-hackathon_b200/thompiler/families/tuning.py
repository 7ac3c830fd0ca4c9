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
    # the fewest 64-deep K blocks a part of a split tile keeps (CTA-pair kernel)
    matmul_tail_kblocks: int = 16
    # CTA-pair kernel: a partial last wave whose tiles, halved, fit one wave of pairs has its
    # 256-wide tiles cut along N into two 256 x 128 units (else, or when False, the K split)
    matmul_half_tail: bool = True
    # programmatic dependent launch: tuned bodies signal griddepcontrol.launch_dependents and wait
    # (griddepcontrol.wait) before global accesses, and their launches may overlap the previous kernel
    pdl: bool = True
    # attention: of every 8 score pairs, this many take 2^x from a polynomial on the FMA pipe
    # instead of the exponential unit (0 .. 8)
    attention_poly_pairs: int = 1


TUNING = Tuning()
