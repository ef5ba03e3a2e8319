"""Parity rules shared by the GPU tests.

Selections (top-k position sets) are compared with the rule the target
states: indices must agree wherever the reference's scores are separated by
more than ``rtol`` relative.  Concretely, for oracle scores ``ref`` and device
scores ``dev`` of the same positions:

* a position is *flipped* when its device score differs from the oracle's by
  more than ``value_tol`` relative (0 for 16-bit dtypes: any bit differs);
  flips come from fp32 accumulation order inside the dot products and the
  softmax sum, and their count is reported and bounded separately;
* positions within ``rtol`` relative of the oracle's k-th score or of the
  device's k-th score are ties at the boundary (either choice is valid: the
  reference's ``torch.topk`` order among equal values is unspecified);
* every other position must be selected by both or by neither.
"""
from __future__ import annotations

from typing import Dict, Iterable, Optional

import numpy as np

# bf16 / fp16: a device score either matches the oracle bit for bit or it is a
# flip.  fp32: the reference's own CPU softmax carries ~1e-6 relative error
# at L = 32K (measured against fp64), so values within 1e-6 count as equal.
VALUE_TOL = {"float32": 1e-6, "bfloat16": 0.0, "float16": 0.0}
SEL_RTOL = 1e-6
# Bound on the device scores themselves.  16-bit: at most 1% of positions may
# differ from the oracle (each by one rounding step).  fp32: every position
# within 1e-5 relative (exp implementation and summation order differ between
# the CPU reference and the device; each contributes ~1e-6).
FLIP_FRAC_16 = 0.01
FP32_MAX_REL = 1e-5


def scores_close(res: Dict, dtype: str) -> bool:
    if dtype == "float32":
        return res["max_rel"] <= FP32_MAX_REL
    return res["flips"] <= FLIP_FRAC_16 * res["L"]


def kth_largest(x: np.ndarray, k: int) -> float:
    if k <= 0:
        return np.inf
    if k >= x.size:
        return float(x.min())
    return float(np.partition(x, x.size - k)[x.size - k])


def compare_selection(ref: np.ndarray, dev: Optional[np.ndarray], sel: Iterable[int], k: int, dtype: str,
                      rtol: float = SEL_RTOL) -> Dict:
    ref = np.asarray(ref, dtype=np.float64)
    sel = np.asarray(sorted(set(int(i) for i in sel)), dtype=np.int64)
    L = ref.size
    out = {"k": k, "n_selected": int(sel.size), "L": L}
    mask = np.zeros(L, dtype=bool)
    mask[sel] = True
    t_ref = kth_largest(ref, k)
    if dev is not None:
        dev = np.asarray(dev, dtype=np.float64)
        tol = VALUE_TOL[dtype]
        flips = np.abs(dev - ref) > tol * np.abs(ref)
        t_dev = kth_largest(dev, k)
        nz = ref != 0
        out["max_rel"] = float(np.max(np.abs(dev - ref)[nz] / np.abs(ref[nz]))) if nz.any() else 0.0
    else:
        flips = np.zeros(L, dtype=bool)
        t_dev = t_ref
        out["max_rel"] = 0.0
    band = (np.abs(ref - t_ref) <= rtol * abs(t_ref)) | (np.abs(ref - t_dev) <= rtol * abs(t_dev))
    exempt = flips | band
    must_in = (ref > t_ref) & ~exempt
    must_out = (ref < t_ref) & ~exempt
    out["missing"] = int(np.count_nonzero(must_in & ~mask))
    out["extra"] = int(np.count_nonzero(must_out & mask))
    out["flips"] = int(np.count_nonzero(flips))
    out["boundary"] = int(np.count_nonzero(band))
    ref_set = np.zeros(L, dtype=bool)
    if k > 0:
        ref_set[np.argsort(-ref, kind="stable")[:k]] = True
    out["set_diff"] = int(np.count_nonzero(ref_set != mask))
    out["ok"] = out["missing"] == 0 and out["extra"] == 0 and sel.size == min(k, L)
    return out
