"""Parity comparators: the CUDA path's results against the oracle's.

TEST INFRASTRUCTURE ONLY (the checker side): used by tests/ and by bench.py's
parity leg, never by the product path.

Each function returns a small dict (the `parity` object of a bench line) with
the counts it checked and `pass`, applying the bar the backend promises for
that precision class:

  * fp16 / bf16: recall >= 0.99 against the oracle's top-k on the same rounded
    values, rank-wise distances within 1e-2 relative (1e-4 absolute floor);
  * fp32 (3xTF32): identical rows except where distances tie within 1e-5
    relative, distances within 1e-5 relative;
  * int8 and PQ codes: identical rows and identical distance bits.
"""
from __future__ import annotations

import numpy as np


def recall(rows, ref_rows) -> float:
    hits = total = 0
    for a, b in zip(rows, ref_rows):
        b = b[b >= 0]
        total += len(b)
        hits += len(np.intersect1d(a[a >= 0], b, assume_unique=False))
    return hits / max(total, 1)


def _dist_err(dist, ref_dist):
    valid = np.isfinite(ref_dist)
    if not valid.any():
        return 0.0, 0.0
    diff = np.abs(dist[valid].astype(np.float64) - ref_dist[valid].astype(np.float64))
    rel = diff / np.maximum(np.abs(ref_dist[valid].astype(np.float64)), 1e-30)
    return float(diff.max()), float(rel.max())


def low_precision(dist, rows, ref_dist, ref_rows, rtol=1e-2, atol=1e-4, min_recall=0.99) -> dict:
    """fp16 / bf16 class."""
    rec = recall(rows, ref_rows)
    max_abs, max_rel = _dist_err(dist, ref_dist)
    valid = np.isfinite(ref_dist)
    within = bool((np.abs(dist[valid].astype(np.float64) - ref_dist[valid])
                   <= rtol * np.abs(ref_dist[valid].astype(np.float64)) + atol).all())
    return {"queries": int(rows.shape[0]), "k": int(rows.shape[1]), "recall": round(rec, 6),
            "max_abs_dist_err": max_abs, "max_rel_dist_err": max_rel,
            "criterion": f"recall >= {min_recall}, |d - d_ref| <= {rtol} |d_ref| + {atol}",
            "pass": bool(rec >= min_recall and within)}


def fp32_exact(dist, rows, ref_dist, ref_rows, true_dist, rtol=1e-5, atol=0.0) -> dict:
    """fp32-exact class: differing rows must be ties. true_dist(q, row) is the
    oracle's distance of any (query, row) pair."""
    valid = ref_rows >= 0
    same_count = bool(np.array_equal(rows >= 0, valid))
    tol = rtol * np.maximum(np.abs(ref_dist), 1e-30) + atol
    dist_ok = bool(not (valid & (np.abs(dist - ref_dist) > tol)).any())
    diff = valid & (rows != ref_rows)
    unexplained = 0
    for q, i in zip(*np.nonzero(diff)):
        if abs(true_dist(int(q), int(rows[q, i])) - ref_dist[q, i]) > tol[q, i]:
            unexplained += 1
    max_abs, max_rel = _dist_err(dist, ref_dist)
    return {"queries": int(rows.shape[0]), "k": int(rows.shape[1]),
            "rows_equal": int((~diff & valid).sum()), "rows_checked": int(valid.sum()),
            "rows_differing_as_ties": int(diff.sum()) - unexplained, "rows_differing_not_ties": unexplained,
            "recall": round(recall(rows, ref_rows), 6), "max_abs_dist_err": max_abs, "max_rel_dist_err": max_rel,
            "criterion": f"identical rows except ties within {rtol} relative; distances within {rtol} relative",
            "pass": bool(same_count and dist_ok and unexplained == 0)}


def bit_exact(dist, rows, ref_dist, ref_rows) -> dict:
    """int8 / PQ class: ids and distance bits identical."""
    rows_eq = rows == ref_rows
    bits_eq = np.ascontiguousarray(dist, np.float32).view(np.uint32) == \
        np.ascontiguousarray(ref_dist, np.float32).view(np.uint32)
    q_eq = rows_eq.all(axis=1) & bits_eq.all(axis=1)
    return {"queries": int(rows.shape[0]), "k": int(rows.shape[1]),
            "queries_identical": int(q_eq.sum()), "rows_equal": int(rows_eq.sum()),
            "dist_bits_equal": int(bits_eq.sum()), "entries": int(rows.size),
            "criterion": "identical ids and distance bits", "pass": bool(q_eq.all())}


def against_reference_with_ties(dist, rows, ref_dist, ref_rows, gap) -> dict:
    """IVF-PQ against the reference's own GpuIVFPQIndex::search: a query may
    differ only where the reference's rerank boundary is an exact tie (gap 0),
    whose resolution std::partial_sort leaves unspecified."""
    same = (rows == ref_rows).all(axis=1) & \
        (np.ascontiguousarray(dist, np.float32).view(np.uint32) ==
         np.ascontiguousarray(ref_dist, np.float32).view(np.uint32)).all(axis=1)
    differ = np.nonzero(~same)[0]
    untied = [int(q) for q in differ if gap[q] != 0]
    return {"queries": int(rows.shape[0]), "queries_identical": int(same.sum()),
            "queries_differing_at_a_tied_boundary": int(len(differ) - len(untied)),
            "queries_differing_untied": len(untied),
            "criterion": "identical to the reference except queries whose rerank boundary is an exact tie",
            "pass": not untied}
