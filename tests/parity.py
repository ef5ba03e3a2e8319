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
* a flipped position is exempt only when the oracle's score at it lies within
  one rounding step of the dtype of the k-th score (a flip moves a score by
  one step, so only there can it change the selection);
* every other position must be selected by both or by neither.

Every comparison is also recorded (``RECORDS``); with ``HC_PARITY_REPORT``
set, the test session writes them, per test, as JSON to that path.
"""
from __future__ import annotations

import math
import os
from typing import Dict, Iterable, List, Optional

import numpy as np

# bf16 / fp16: a device score either matches the oracle bit for bit or it is a
# flip.  fp32: the reference's own CPU softmax carries ~1e-6 relative error
# at L = 32K (measured against fp64), so values within 1e-6 count as equal.
VALUE_TOL = {"float32": 1e-6, "bfloat16": 0.0, "float16": 0.0}
SEL_RTOL = 1e-6
# Bound on the device scores themselves.  16-bit: at most 0.1% of positions
# (or 12, at short lengths) may differ from the oracle, each by one rounding
# step; the aggregate rate is reported.  fp32: every
# position within 1e-5 relative (exp implementation and summation order
# differ between the CPU reference and the device; each contributes ~1e-6).
FLIP_FRAC_16 = 0.001
FLIP_FLOOR_16 = 12  # ... or up to this many, at short lengths (measured: 9 of 3000 in one fp16 drift step)
FP32_MAX_REL = 1e-5
MANTISSA = {"bfloat16": 7, "float16": 10}

RECORDS: List[Dict] = []


def rounding_step(x: float, dtype: str) -> float:
    """Spacing of the dtype's values at |x|: one rounding step (fp32: the
    score tolerance, relative)."""
    if not math.isfinite(x):
        return 0.0
    if dtype == "float32":
        return FP32_MAX_REL * abs(x)
    m = MANTISSA[dtype]
    if x == 0.0:
        return 2.0 ** (-133 if dtype == "bfloat16" else -24)
    e = math.floor(math.log2(abs(x)))
    if dtype == "float16":
        e = max(e, -14)
    return 2.0 ** (e - m)


def scores_close(res: Dict, dtype: str, terms: int = 1) -> bool:
    """``terms``: rounded probabilities summed into each score (the
    observation window); a flip of any one of them can flip the sum, so the
    16-bit bound scales with it."""
    if dtype == "float32":
        return res["max_rel"] <= FP32_MAX_REL
    return res["flips"] <= max(FLIP_FRAC_16 * res["L"] * terms, FLIP_FLOOR_16)


def kth_largest(x: np.ndarray, k: int) -> float:
    if k <= 0:
        return np.inf
    if k >= x.size:
        return float(x.min())
    return float(np.partition(x, x.size - k)[x.size - k])


def exempt_mask(ref: np.ndarray, dev: Optional[np.ndarray], k: int, dtype: str, rtol: float = SEL_RTOL,
                with_near: bool = False):
    """(exempt, flips, band, t_ref, t_dev) for oracle scores ``ref`` and device
    scores ``dev`` of a top-k selection (and the flips within one rounding
    step of the k-th score, with_near)."""
    ref = np.asarray(ref, dtype=np.float64)
    t_ref = kth_largest(ref, k)
    if dev is not None:
        dev = np.asarray(dev, dtype=np.float64)
        flips = np.abs(dev - ref) > VALUE_TOL[dtype] * np.abs(ref)
        t_dev = kth_largest(dev, k)
    else:
        flips = np.zeros(ref.size, dtype=bool)
        t_dev = t_ref
    band = (np.abs(ref - t_ref) <= rtol * abs(t_ref)) | (np.abs(ref - t_dev) <= rtol * abs(t_dev))
    near = (np.abs(ref - t_ref) <= rounding_step(t_ref, dtype)) | (np.abs(ref - t_dev) <= rounding_step(t_dev, dtype))
    if with_near:
        return (flips & near) | band, flips, band, t_ref, t_dev, flips & near
    return (flips & near) | band, flips, band, t_ref, t_dev


def compare_selection(ref: np.ndarray, dev: Optional[np.ndarray], sel: Iterable[int], k: int, dtype: str,
                      rtol: float = SEL_RTOL, scores_only: bool = False) -> Dict:
    """The tie-aware rule above.  scores_only: the caller compares the scores
    alone (no selection to check); the record says so."""
    ref = np.asarray(ref, dtype=np.float64)
    sel = np.asarray(sorted(set(int(i) for i in sel)), dtype=np.int64)
    L = ref.size
    out = {"k": k, "n_selected": int(sel.size), "L": L}
    mask = np.zeros(L, dtype=bool)
    mask[sel] = True
    exempt, flips, band, t_ref, _ = exempt_mask(ref, dev, k, dtype, rtol)
    if dev is not None:
        dev = np.asarray(dev, dtype=np.float64)
        nz = ref != 0
        out["max_rel"] = float(np.max(np.abs(dev - ref)[nz] / np.abs(ref[nz]))) if nz.any() else 0.0
    else:
        out["max_rel"] = 0.0
    must_in = (ref > t_ref) & ~exempt
    must_out = (ref < t_ref) & ~exempt
    out["missing"] = int(np.count_nonzero(must_in & ~mask))
    out["extra"] = int(np.count_nonzero(must_out & mask))
    out["flips"] = int(np.count_nonzero(flips))
    out["flips_near_boundary"] = int(np.count_nonzero(flips & exempt & ~band))
    out["boundary"] = int(np.count_nonzero(band))
    ref_set = np.zeros(L, dtype=bool)
    if k > 0:
        ref_set[np.argsort(-ref, kind="stable")[:k]] = True
    out["set_diff"] = int(np.count_nonzero(ref_set != mask))
    out["ok"] = out["missing"] == 0 and out["extra"] == 0 and sel.size == min(k, L)
    rec = {"test": os.environ.get("PYTEST_CURRENT_TEST", "").split(" ")[0], "dtype": dtype,
           **{key: out[key] for key in ("L", "k", "flips", "flips_near_boundary", "boundary", "set_diff",
                                         "max_rel", "ok")}}
    if scores_only:
        rec.update(scores_only=True, ok=None, set_diff=None)
    RECORDS.append(rec)
    return out


def compare_exact(ref: np.ndarray, dev: Optional[np.ndarray], sel: Iterable[int], k: int, dtype: str) -> Dict:
    """Selections under one tie rule on both sides (equal scores go to the
    lowest positions, the oracle run with ties="lowest"): the device's set
    must be the oracle's stable top-k, except that each device score that
    flipped within one rounding step of the k-th score may change two
    memberships (itself, and the tie it displaces)."""
    ref = np.asarray(ref, dtype=np.float64)
    sel = set(int(i) for i in sel)
    L = ref.size
    ref_set = set(np.argsort(-ref, kind="stable")[:k].tolist()) if k > 0 else set()
    _, flips, band, _, _, near = exempt_mask(ref, dev, k, dtype, with_near=True)
    out = {"k": k, "L": L, "n_selected": len(sel), "set_diff": len(ref_set ^ sel),
           "flips": int(np.count_nonzero(flips)), "flips_near_boundary": int(np.count_nonzero(near)),
           "boundary": int(np.count_nonzero(band)), "max_rel": 0.0}
    if dev is not None:
        dev = np.asarray(dev, dtype=np.float64)
        nz = ref != 0
        out["max_rel"] = float(np.max(np.abs(dev - ref)[nz] / np.abs(ref[nz]))) if nz.any() else 0.0
    out["ok"] = out["set_diff"] <= 2 * out["flips_near_boundary"] and len(sel) == min(k, L)
    RECORDS.append({"test": os.environ.get("PYTEST_CURRENT_TEST", "").split(" ")[0], "dtype": dtype,
                    "exact": True, **{key: out[key] for key in ("L", "k", "flips", "flips_near_boundary",
                                                               "boundary", "set_diff", "max_rel", "ok")}})
    return out


def near_flip_count(ref: np.ndarray, dev: Optional[np.ndarray], k: int, dtype: str) -> int:
    """Device scores that flipped within one rounding step of the k-th score."""
    return int(np.count_nonzero(exempt_mask(ref, dev, k, dtype, with_near=True)[5]))


def exempt_count(ref: np.ndarray, dev: Optional[np.ndarray], k: int, dtype: str) -> int:
    """Positions whose membership in a top-k the parity rule leaves open."""
    return int(np.count_nonzero(exempt_mask(ref, dev, k, dtype)[0]))


def summary() -> Dict:
    """Per test: comparisons, worst flip fraction, total flips / boundary ties."""
    out: Dict[str, Dict] = {}
    for r in RECORDS:
        s = out.setdefault(r["test"], {"comparisons": 0, "positions": 0, "flips": 0, "flips_near_boundary": 0,
                                       "boundary": 0, "set_diff": 0, "max_flip_frac": 0.0, "dtype": r["dtype"]})
        s["comparisons"] += 1
        s["positions"] += r["L"]
        for key in ("flips", "flips_near_boundary", "boundary", "set_diff"):
            s[key] += r[key] or 0
        s["max_flip_frac"] = max(s["max_flip_frac"], r["flips"] / max(r["L"], 1))
    for s in out.values():
        s["flip_frac"] = s["flips"] / max(s["positions"], 1)
    return out
