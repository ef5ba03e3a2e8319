"""The scoring kernels scale bf16 logits by sqrt(128) with a multiply by the
correctly rounded reciprocal instead of a division (``scale_by_recip`` in
``csrc/score_select.cu``).  The reference divides the bf16 logits
(``heterocache/cache_utils.py:814``: ``/ math.sqrt(head_dim)``, computed in
fp32 and rounded to bf16).  The two agree only if, for every finite bf16
value x, rounding x * RN(1 / c) and RN(x / c) to bf16 gives the same bits,
c = fp32(sqrt(128)).  This checks all 2^16 bit patterns, and that the same
does not hold for fp16 (which keeps the division).
"""
import math

import numpy as np


def _bf16_round(a):
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    return ((u + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32).view(np.float32)


def _mismatches(kind):
    c = np.float32(math.sqrt(128.0))
    r = np.float32(1.0) / c
    bits = np.arange(1 << 16, dtype=np.uint32)
    if kind == "bf16":
        x = (bits << 16).view(np.float32)
        rnd = _bf16_round
    else:
        x = bits.astype(np.uint16).view(np.float16).astype(np.float32)
        rnd = lambda a: a.astype(np.float16).astype(np.float32)  # noqa: E731
    x = x[np.isfinite(x)]
    with np.errstate(all="ignore"):
        by_div = rnd((x / c).astype(np.float32))
        by_mul = rnd((x * r).astype(np.float32))
    return int((by_div.view(np.uint32) != by_mul.view(np.uint32)).sum()), x.size


def test_bf16_scale_by_reciprocal_is_exact():
    bad, n = _mismatches("bf16")
    assert n == 65280 and bad == 0


def test_fp16_needs_the_division():
    bad, _ = _mismatches("f16")
    assert bad > 0
