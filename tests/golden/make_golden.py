"""Regenerates tests/golden/reference_outputs.npz by running the reference's
own compiled code (oracle/_ref/libelips_ref.so, built from the reference
sources by oracle/Makefile) on small seeded inputs.

    python tests/golden/make_golden.py

Every array in the file is either a seeded input or an output of the
reference itself: ExactIndex::search (3 metrics), ExactIndex with
ScalarQuantizer / ProductQuantizer / OPQ, quant::detail::kmeans,
train_pq_codebook, encode_pq, and GpuIVFPQIndex::search on a CPU GpuPort.
"""
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
import oracle as O  # noqa: E402

METRICS = ["cosine", "euclidean", "dot_product"]


def main():
    rng = np.random.default_rng(20261201)
    out = {}
    base = rng.standard_normal((600, 24)).astype(np.float32)
    queries = rng.standard_normal((12, 24)).astype(np.float32)
    unit_base = (base / np.linalg.norm(base, axis=1, keepdims=True)).astype(np.float32)
    unit_q = (queries / np.linalg.norm(queries, axis=1, keepdims=True)).astype(np.float32)
    out["base"], out["queries"], out["unit_base"], out["unit_queries"] = base, queries, unit_base, unit_q
    for m in METRICS:
        b, q = (unit_base, unit_q) if m == "cosine" else (base, queries)
        d, r = O.RefExactIndex(m, b).search(q, 7, 1)
        out[f"exact_{m}_dist"], out[f"exact_{m}_rows"] = d, r
    # sq8: trained on the first 300 rows, so later rows exercise the clamp
    mins, scales = O.ref_sq8_train("euclidean", base[:300])
    out["sq8_mins"], out["sq8_scales"] = mins, scales
    out["sq8_codes"] = O.ref_sq8_encode("euclidean", mins, scales, base)
    for m in METRICS:
        d, r = O.RefExactIndex(m, base, codec="sq8", mins=mins, scales=scales).search(queries, 5, 1)
        out[f"sq8_{m}_dist"], out[f"sq8_{m}_rows"] = d, r
    # pq: 8 subspaces x 16 codewords (4 bits)
    cb = O.ref_train_pq_codebook(base, 8, 16, 6)
    out["pq_codebook"] = cb
    out["pq_codes"] = O.ref_encode_pq(cb, base)
    for m in METRICS:
        d, r = O.RefExactIndex(m, base, codec="pq", codebook=cb, pq_bits=4).search(queries, 5, 1)
        out[f"pq_{m}_dist"], out[f"pq_{m}_rows"] = d, r
    # opq: a seeded orthonormal rotation
    rot, _ = np.linalg.qr(rng.standard_normal((24, 24)))
    rot = rot.astype(np.float32)
    out["opq_rotation"] = rot
    for m in METRICS:
        d, r = O.RefExactIndex(m, base, codec="opq", codebook=cb, pq_bits=4, rotation=rot).search(queries, 5, 1)
        out[f"opq_{m}_dist"], out[f"opq_{m}_rows"] = d, r
    # k-means
    out["kmeans_centroids"] = O.ref_kmeans(base, 10, 8)
    # ivf-pq: 12 lists, residual PQ 8 x 16, nprobe 3, k 4 (R = 16)
    cent = O.ref_kmeans(base, 12, 8)
    asg = O.ivf_assign("euclidean", base, cent)
    res = base - cent[asg]
    icb = O.ref_train_pq_codebook(res, 8, 16, 6)
    icodes = O.ref_encode_pq(icb, res)
    d, r = O.RefIvfPqIndex("euclidean", cent, asg, icb, icodes, base, 3, pq_bits=4).search(queries, 4, 1)
    out.update(ivf_centroids=cent, ivf_assignments=asg, ivf_codebook=icb, ivf_codes=icodes,
               ivf_dist=d, ivf_rows=r)
    path = Path(__file__).resolve().parent / "reference_outputs.npz"
    np.savez_compressed(path, **out)
    print(path, sum(v.nbytes for v in out.values()), "bytes")


if __name__ == "__main__":
    main()
