"""Row-by-row comparison of the CUDA sampler against the oracle.

Rule (the benchmark's parity criterion): ids identical, except rows whose draw
lies within 1e-5 (relative to the renormalisation sum) of a CDF boundary or
whose nucleus cut lies within 1e-5 of top_p -- there the device expf (<= 2 ulp
from glibc's) may legitimately move the boundary.  Probabilities of matching
rows agree within 1e-5 relative.
"""
from __future__ import annotations

import numpy as np

TOL = 1e-5


def compare(ids, probs, ref_ids, ref_probs, ref_res, tol: float = TOL) -> dict:
    ids = np.asarray(ids)
    ref_ids = np.asarray(ref_ids)
    same = ids == ref_ids
    near = (ref_res["r_margin"] <= tol) | (ref_res["cut_margin"] <= tol)
    bad = ~same & ~near
    pr_bad = np.zeros_like(same)
    if probs is not None:
        p = np.asarray(probs, np.float64)
        q = np.asarray(ref_probs, np.float64)
        both_nan = np.isnan(p) & np.isnan(q)
        rel = np.abs(p - q) / np.maximum(np.abs(q), 1e-30)
        pr_bad = same & ~both_nan & ~(rel <= tol)
    return {
        "rows": int(ids.size),
        "exact": int(same.sum()),
        "exempt_mismatch": int((~same & near).sum()),
        "bad": int(bad.sum()),
        "bad_rows": np.nonzero(bad)[0][:20].tolist(),
        "prob_bad": int(pr_bad.sum()),
        "prob_bad_rows": np.nonzero(pr_bad)[0][:20].tolist(),
        "near": int(near.sum()),
    }
