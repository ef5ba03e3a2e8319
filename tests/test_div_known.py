"""Division by a known divisor (``div_known`` in hc_common.cuh) is correctly rounded.

The kernels replace IEEE division by a fixed divisor y with Markstein's
residual correction: q = RN(x*r), e = RN(x - q*y) (one fused multiply-add,
exact), result RN(q + e*r), with r = RN(1/y).  The reference divides
logits by sqrt(head_dim) and pooled sums by the kernel size with ordinary
IEEE division, so the replacement must agree bit for bit on the operands the
kernels feed it:

* logits of 16-bit models: every bf16 and f16 value divided by
  float32(sqrt(128)), the quotient's sign then copied from the operand (which
  only matters for -0); nonzero operands with |x| < 2^-120 (quotient near or
  below the subnormal range) are sent to IEEE division by the kernel, so they
  are excluded here;
* pooled sums: fp32 values divided by the kernel size 3, 5 or 7 (half-widths
  1..3).  The quotient of a normal x depends only on its significand, so one
  full binade stands for all normal operands; two more binades and every
  subnormal are checked as well.

The emulation is exact: products of two fp32 values are exact in float64, the
residual is exact by Sterbenz's lemma, and the one sum that float64 may round
is checked for landing on an fp32 rounding midpoint (then the double
rounding could differ; the test asserts it never happens).
"""
import numpy as np
import pytest


def _markstein(x32: np.ndarray, y32: np.float32):
    r = np.float32(1) / y32
    x = x32.astype(np.float64)
    q = (x * np.float64(r)).astype(np.float32)
    e = (x - q.astype(np.float64) * np.float64(y32)).astype(np.float32)
    s = q.astype(np.float64) + e.astype(np.float64) * np.float64(r)
    res = s.astype(np.float32)
    lo = np.nextafter(res, np.float32(-np.inf))
    hi = np.nextafter(res, np.float32(np.inf))
    mid = (s == (lo.astype(np.float64) + res) / 2) | (s == (hi.astype(np.float64) + res) / 2)
    return res, mid


def _check(x32: np.ndarray, y: float, copysign: bool = False) -> None:
    y32 = np.float32(y)
    res, mid = _markstein(x32, y32)
    if copysign:
        res = np.copysign(res, x32)
    assert not mid.any(), "float64 emulation hit an fp32 midpoint"
    want = x32 / y32
    bad = res.view(np.uint32) != want.view(np.uint32)
    assert not bad.any(), (x32[bad][:5], res[bad][:5], want[bad][:5])


def _logit_operands(kind: str) -> np.ndarray:
    if kind == "bf16":
        x = (np.arange(1 << 16, dtype=np.uint32) << 16).view(np.float32)
    else:
        x = np.arange(1 << 16, dtype=np.uint16).view(np.float16).astype(np.float32)
    return x[np.isfinite(x) & ((np.abs(x) >= np.float32(2.0 ** -120)) | (x == 0))]


@pytest.mark.parametrize("kind", ["bf16", "f16"])
def test_logit_scaling_matches_ieee_division(kind):
    x = _logit_operands(kind)
    assert np.signbit(x[x == 0]).any() and not np.signbit(x[x == 0]).all()  # both zeros are covered
    _check(x, float(np.float32(np.sqrt(128.0))), copysign=True)


@pytest.mark.parametrize("ks", [3.0, 5.0, 7.0])
def test_pooling_division_matches_ieee_division(ks):
    for e in (0, 2, -60):
        xs = (np.uint32((e + 127) << 23) + np.arange(1 << 23, dtype=np.uint32)).view(np.float32)
        _check(xs, ks)
    _check(np.arange(1, 1 << 23, dtype=np.uint32).view(np.float32), ks)  # subnormals
    _check(np.zeros(1, np.float32), ks)

