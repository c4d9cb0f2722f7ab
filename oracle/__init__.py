"""CPU checkers for the parity tests. TEST INFRASTRUCTURE ONLY.

Libraries built by oracle/Makefile:
  * liboracle.so             -- oracle.c, a C restatement of the reference's
                                search arithmetic (each function cites the
                                reference file:line it follows);
  * _ref/libelips_ref.so     -- the reference's own sources compiled in place
                                plus ref_driver.cpp, used to pin the
                                restatement and as the timed CPU baseline;
  * _ref/libelips_ref_b200.so -- the same reference classes able to run on
                                the B200 CudaBackend adapter
                                (elips_b200/integration), for the drop-in check
                                of the GpuPort boundary (GPU tests only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs may import this package; the product path (elips_b200/) never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, c_float, c_int, c_int64, c_size_t, c_uint8, c_uint32, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libelips_ref.so"
REF_B200_SO = HERE / "_ref" / "libelips_ref_b200.so"
PRODUCT_SO = HERE.parent / "elips_b200" / "libelips_b200.so"
# The reference tree: ELIPS_REF_ROOT, else a checkout named `reference` beside
# this repository.
REF_ROOT = Path(os.environ.get("ELIPS_REF_ROOT", str(HERE.parent.parent / "reference")))

METRIC = {"cosine": 0, "euclidean": 1, "dot_product": 2}


def build(ref: bool = True) -> None:
    """Builds liboracle.so and, when the reference sources are present, _ref."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    if ref and REF_ROOT.exists():
        targets = ["ref", "ref_b200"] if PRODUCT_SO.exists() else ["ref"]
        subprocess.run(["make", "-s", "-j8", "-C", str(HERE), *targets, f"REF_ROOT={REF_ROOT}"], check=True)


_orc = None
_ref = None
_ref_b200 = None


def orc() -> ctypes.CDLL:
    global _orc
    if _orc is None:
        if not ORACLE_SO.exists():
            build(ref=False)
        _orc = ctypes.CDLL(str(ORACLE_SO))
        _orc.orc_distance.restype = c_float
        _orc.orc_distance.argtypes = [c_int, c_void_p, c_void_p, c_size_t]
        _orc.orc_sq8_lut_distance.restype = c_float
        _orc.orc_pq_lut_distance.restype = c_float
        _orc.orc_nearest_centroid.restype = c_uint8
    return _orc


def ref_available() -> bool:
    return REF_SO.exists() or REF_ROOT.exists()


def _declare(lib: ctypes.CDLL) -> ctypes.CDLL:
    lib.ref_distance.restype = c_float
    lib.ref_distance.argtypes = [c_int, c_void_p, c_void_p, c_size_t]
    for name in ("ref_exact_create", "ref_sq8_exact_create", "ref_pq_exact_create", "ref_opq_exact_create",
                 "ref_ivfpq_create", "ref_ivfflat_create", "ref_brute_create"):
        getattr(lib, name).restype = c_void_p
    return lib


def ref() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not REF_SO.exists():
            build(ref=True)
        _ref = _declare(ctypes.CDLL(str(REF_SO)))
    return _ref


def ref_b200() -> ctypes.CDLL:
    """The reference classes on the B200 CudaBackend (needs a GPU to run)."""
    global _ref_b200
    if _ref_b200 is None:
        if not REF_B200_SO.exists():
            build(ref=True)
        _ref_b200 = _declare(ctypes.CDLL(str(REF_B200_SO)))
    return _ref_b200


def _port_lib(port: str) -> ctypes.CDLL:
    """Library whose next index handle is built on `port` ("cpu" or "b200")."""
    if port == "cpu":
        return ref()
    if port != "b200":
        raise ValueError(f"unknown port {port!r}")
    lib = ref_b200()
    if lib.ref_use_b200_port(1) != 1:
        raise RuntimeError("reference driver built without the B200 port")
    return lib


def _p(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _threads(n):
    return int(n) if n else (os.cpu_count() or 1)


# ------------------------------------------------------------- restatement

def distance(metric: str, a, b) -> float:
    a, b = _f32(a), _f32(b)
    return float(orc().orc_distance(METRIC[metric], _p(a), _p(b), a.size))


def exact_search(metric, base, queries, k, nthreads=None, mask=None):
    base, queries = _f32(base), _f32(queries)
    n, d = base.shape
    nq = queries.shape[0]
    dist = np.empty((nq, k), np.float32)
    rows = np.empty((nq, k), np.int64)
    if mask is None:
        orc().orc_exact_search(METRIC[metric], _p(base), c_size_t(n), c_size_t(d), _p(queries),
                               c_size_t(nq), c_size_t(k), c_int(_threads(nthreads)), _p(dist), _p(rows))
    else:
        m = np.ascontiguousarray(mask, np.uint32)
        orc().orc_exact_search_masked(METRIC[metric], _p(base), c_size_t(n), c_size_t(d), _p(m),
                                      _p(queries), c_size_t(nq), c_size_t(k), c_int(_threads(nthreads)),
                                      _p(dist), _p(rows))
    return dist, rows


def int8_ip_search(base, queries, k, nthreads=None):
    base = np.ascontiguousarray(base, np.int8)
    queries = np.ascontiguousarray(queries, np.int8)
    n, d = base.shape
    nq = queries.shape[0]
    dist = np.empty((nq, k), np.float32)
    rows = np.empty((nq, k), np.int64)
    orc().orc_int8_ip_search(_p(base), c_size_t(n), c_size_t(d), _p(queries), c_size_t(nq), c_size_t(k),
                             c_int(_threads(nthreads)), _p(dist), _p(rows))
    return dist, rows


def exact_search_fast(metric, base, queries, k, nthreads=None, mask=None):
    """exact_search's results (bit for bit) from the blocked, vectorised scan
    of oracle_fast.c: each pair's sum is still the sequential single-precision
    loop, 16 queries share a vector. For large bases (2M x 768)."""
    base, queries = _f32(base), _f32(queries)
    n, d = base.shape
    nq = queries.shape[0]
    dist = np.empty((nq, k), np.float32)
    rows = np.empty((nq, k), np.int64)
    m = None if mask is None else np.ascontiguousarray(mask, np.uint32)
    orc().orc_exact_search_fast(METRIC[metric], _p(base), c_size_t(n), c_size_t(d),
                                None if m is None else _p(m), _p(queries), c_size_t(nq), c_size_t(k),
                                c_int(_threads(nthreads)), _p(dist), _p(rows))
    return dist, rows


def int8_ip_search_fast(base, queries, k, nthreads=None):
    """int8_ip_search's results (bit for bit) from oracle_fast.c's blocked scan."""
    base = np.ascontiguousarray(base, np.int8)
    queries = np.ascontiguousarray(queries, np.int8)
    n, d = base.shape
    nq = queries.shape[0]
    dist = np.empty((nq, k), np.float32)
    rows = np.empty((nq, k), np.int64)
    orc().orc_int8_ip_search_fast(_p(base), c_size_t(n), c_size_t(d), _p(queries), c_size_t(nq), c_size_t(k),
                                  c_int(_threads(nthreads)), _p(dist), _p(rows))
    return dist, rows


def sq8_train(rows):
    rows = _f32(rows)
    n, d = rows.shape
    mins = np.empty(d, np.float32)
    scales = np.empty(d, np.float32)
    orc().orc_sq8_train(c_size_t(d), _p(rows), c_size_t(n), _p(mins), _p(scales))
    return mins, scales


def sq8_encode(mins, scales, rows):
    rows = _f32(rows)
    n, d = rows.shape
    codes = np.empty((n, d), np.uint8)
    orc().orc_sq8_encode(c_size_t(d), _p(_f32(mins)), _p(_f32(scales)), _p(rows), c_size_t(n), _p(codes))
    return codes


def sq8_search(metric, mins, scales, codes, queries, k, nthreads=None):
    codes = np.ascontiguousarray(codes, np.uint8)
    queries = _f32(queries)
    n, d = codes.shape
    nq = queries.shape[0]
    dist = np.empty((nq, k), np.float32)
    rows = np.empty((nq, k), np.int64)
    orc().orc_sq8_search(METRIC[metric], c_size_t(d), _p(_f32(mins)), _p(_f32(scales)), _p(codes),
                         c_size_t(n), _p(queries), c_size_t(nq), c_size_t(k), c_int(_threads(nthreads)),
                         _p(dist), _p(rows))
    return dist, rows


def pq_search(metric, codebook, codes, queries, k, nthreads=None):
    codebook = _f32(codebook)
    m, ksub, sub = codebook.shape
    codes = np.ascontiguousarray(codes, np.uint8)
    queries = _f32(queries)
    n = codes.shape[0]
    nq, d = queries.shape
    dist = np.empty((nq, k), np.float32)
    rows = np.empty((nq, k), np.int64)
    orc().orc_pq_search(METRIC[metric], c_size_t(d), c_size_t(m), c_size_t(ksub), _p(codebook), _p(codes),
                        c_size_t(n), _p(queries), c_size_t(nq), c_size_t(k), c_int(_threads(nthreads)),
                        _p(dist), _p(rows))
    return dist, rows


def encode_pq(codebook, rows):
    codebook = _f32(codebook)
    m, ksub, sub = codebook.shape
    rows = _f32(rows)
    n, d = rows.shape
    codes = np.empty((n, m), np.uint8)
    orc().orc_encode_pq(_p(rows), _p(codebook), c_size_t(n), c_size_t(d), c_size_t(m), c_size_t(ksub),
                        _p(codes))
    return codes


def rotate_rows(rotation, rows):
    """apply_matrix on every row (KMeans.cpp:295-305)."""
    rotation, rows = _f32(rotation), _f32(rows)
    n, d = rows.shape
    out = np.empty_like(rows)
    orc().orc_rotate_rows(_p(rotation), _p(rows), c_size_t(n), c_size_t(d), _p(out))
    return out


def kmeans(rows, k, iters):
    rows = _f32(rows)
    n, d = rows.shape
    cent = np.empty((k, d), np.float32)
    orc().orc_kmeans(_p(rows), c_size_t(n), c_size_t(d), c_size_t(k), c_size_t(iters), _p(cent))
    return cent


def ivf_train(metric, rows, nlist, iters):
    """IvfIndexState::train_centroids then the final assignment (C restatement)."""
    rows = _f32(rows)
    n, d = rows.shape
    cent = np.empty((nlist, d), np.float32)
    asg = np.empty(n, np.uint32)
    orc().orc_ivf_train(METRIC[metric], _p(rows), c_size_t(n), c_size_t(d), c_size_t(nlist), c_size_t(iters),
                        _p(cent), _p(asg))
    return cent, asg


def ref_ivf_train(metric, rows, nlist, iters):
    """The same through the reference's GpuIVFFlatIndex::build_from_batch."""
    rows = _f32(rows)
    n, d = rows.shape
    cent = np.empty((nlist, d), np.float32)
    asg = np.empty(n, np.uint32)
    rc = ref().ref_ivf_train(METRIC[metric], c_uint32(d), _p(rows), c_size_t(n), c_size_t(nlist), c_size_t(iters),
                             _p(cent), _p(asg))
    if rc != 0:
        raise RuntimeError(f"reference IVF training failed ({rc})")
    return cent, asg


def train_pq_codebook(rows, m, ksub, iters):
    """train_pq_codebook (C restatement): codebook [m][ksub][d/m]."""
    rows = _f32(rows)
    n, d = rows.shape
    cb = np.empty((m, ksub, d // m), np.float32)
    orc().orc_train_pq_codebook(_p(rows), c_size_t(n), c_size_t(d), c_size_t(m), c_size_t(ksub), c_size_t(iters),
                                _p(cb))
    return cb


def ivf_probe(metric, queries, centroids, nprobe):
    """IvfIndexState::probe_lists restated: [nq][nprobe] nearest list ids, ties by id."""
    queries, centroids = _f32(queries), _f32(centroids)
    nq, d = queries.shape
    out = np.empty((nq, nprobe), np.uint32)
    for q in range(nq):
        orc().orc_ivf_probe(METRIC[metric], _p(queries[q]), c_size_t(d), _p(centroids), c_size_t(centroids.shape[0]),
                            c_size_t(nprobe), _p(out[q]), None)
    return out


def ivf_assign(metric, rows, centroids):
    rows, centroids = _f32(rows), _f32(centroids)
    out = np.empty(rows.shape[0], np.uint32)
    orc().orc_ivf_assign(METRIC[metric], _p(rows), c_size_t(rows.shape[0]), c_size_t(rows.shape[1]),
                         _p(centroids), c_size_t(centroids.shape[0]), _p(out))
    return out


def lists_csr(assignments, nlist):
    """Members of each list in ascending row order (IvfIndexState.cpp:75-83)."""
    assignments = np.asarray(assignments, np.uint32)
    order = np.argsort(assignments, kind="stable").astype(np.uint32)
    counts = np.bincount(assignments, minlength=nlist)
    offsets = np.zeros(nlist + 1, np.uint32)
    offsets[1:] = np.cumsum(counts)
    return offsets, order


def ivfpq_search(metric, centroids, codebook, codes, vectors, assignments, queries, nprobe, k, nthreads=None,
                 order="reference", with_gap=False):
    """GpuIVFPQIndex::search. order="reference": the reference's own tie order
    (libstdc++ partial_sort for the rerank set, rerank position for exact
    ties); order="device": subspace-grouped approximate sums and ties by slot,
    the device path's documented order. with_gap also returns, per query, the
    relative gap between the R-th approximate distance and the first one left
    out (0 = tied at the rerank boundary)."""
    centroids, codebook, vectors, queries = _f32(centroids), _f32(codebook), _f32(vectors), _f32(queries)
    nlist, d = centroids.shape
    m, ksub, sub = codebook.shape
    offsets, order_rows = lists_csr(assignments, nlist)
    codes = np.ascontiguousarray(codes, np.uint8)
    nq = queries.shape[0]
    dist = np.empty((nq, k), np.float32)
    rows = np.empty((nq, k), np.int64)
    gap = np.empty(nq, np.float32)
    mode = {"reference": 0, "device": 1}[order]
    orc().orc_ivfpq_search(METRIC[metric], c_size_t(d), c_size_t(m), c_size_t(ksub), c_size_t(nlist),
                           c_size_t(nprobe), _p(centroids), _p(codebook), _p(codes), _p(vectors), _p(offsets),
                           _p(order_rows), _p(queries), c_size_t(nq), c_size_t(k), c_int(mode),
                           c_int(_threads(nthreads)), _p(dist), _p(rows), _p(gap))
    return (dist, rows, gap) if with_gap else (dist, rows)


def normalize_rows(rows):
    """Vector::normalized of every row (C restatement)."""
    x = _f32(rows)
    out = np.empty_like(x)
    orc().orc_normalize_rows(_p(x), _p(out), c_size_t(x.shape[0]), c_size_t(x.shape[1]))
    return out


def ref_normalize_rows(rows):
    """Vector::normalized of every row (the reference's own code)."""
    x = _f32(rows)
    out = np.empty_like(x)
    ref().ref_normalize_rows(_p(x), _p(out), c_size_t(x.shape[0]), c_size_t(x.shape[1]))
    return out


def ivfflat_search(metric, centroids, vectors, assignments, queries, nprobe, k, nthreads=None):
    """GpuIVFFlatIndex::search: probe, gather (probe order, member order), exact
    distances, top-k with ties by gather position."""
    centroids, vectors, queries = _f32(centroids), _f32(vectors), _f32(queries)
    nlist, d = centroids.shape
    offsets, order_rows = lists_csr(assignments, nlist)
    nq = queries.shape[0]
    dist = np.empty((nq, k), np.float32)
    rows = np.empty((nq, k), np.int64)
    orc().orc_ivfflat_search(METRIC[metric], c_size_t(d), c_size_t(nlist), c_size_t(nprobe), _p(centroids),
                             _p(vectors), _p(offsets), _p(order_rows), _p(queries), c_size_t(nq), c_size_t(k),
                             c_int(_threads(nthreads)), _p(dist), _p(rows))
    return dist, rows


# --------------------------------------------------- reference, compiled

class RefExactIndex:
    """The reference's ExactIndex (optionally with its sq8 or PQ codec)."""

    def __init__(self, metric, base, codec=None, mins=None, scales=None, codebook=None, pq_bits=8, rotation=None):
        base = _f32(base)
        self.dim = base.shape[1]
        lib = ref()
        if codec is None:
            self.h = lib.ref_exact_create(METRIC[metric], c_uint32(self.dim), _p(base), c_size_t(base.shape[0]))
        elif codec == "sq8":
            self.h = lib.ref_sq8_exact_create(METRIC[metric], c_uint32(self.dim), _p(_f32(mins)),
                                              _p(_f32(scales)), _p(base), c_size_t(base.shape[0]))
        elif codec == "pq":
            cb = _f32(codebook)
            self.h = lib.ref_pq_exact_create(METRIC[metric], c_uint32(self.dim), c_uint32(cb.shape[0]),
                                             c_uint32(pq_bits), _p(cb), _p(base), c_size_t(base.shape[0]))
        elif codec == "opq":
            cb = _f32(codebook)
            rot = _f32(rotation)
            self.h = lib.ref_opq_exact_create(METRIC[metric], c_uint32(self.dim), c_uint32(cb.shape[0]),
                                              c_uint32(pq_bits), _p(cb), _p(rot), _p(base), c_size_t(base.shape[0]))
        else:
            raise ValueError(codec)
        self.h = c_void_p(self.h)

    def _l(self):
        return getattr(self, "_lib", None) or ref()

    def search(self, queries, k, nthreads=None):
        queries = _f32(queries)
        nq = queries.shape[0]
        dist = np.empty((nq, k), np.float32)
        rows = np.empty((nq, k), np.int64)
        self._l().ref_exact_search(self.h, c_uint32(self.dim), _p(queries), c_size_t(nq), c_size_t(k),
                                   c_int(_threads(nthreads)), _p(dist), _p(rows))
        return dist, rows

    def insert(self, rows, first):
        """ExactIndex::insert of rows with ids row_id(first + i)."""
        rows = _f32(rows)
        self._l().ref_exact_insert(self.h, _p(rows), c_size_t(rows.shape[0]), c_uint32(self.dim), c_size_t(first))

    def remove(self, row):
        self._l().ref_exact_remove(self.h, c_size_t(row))

    def size(self):
        self._l().ref_exact_size.restype = c_size_t
        return int(self._l().ref_exact_size(self.h))

    def __del__(self):
        try:
            self._l().ref_exact_destroy(self.h)
        except Exception:
            pass


class RefBruteForceIndex:
    """The reference's GpuBruteForceIndex (build_from_batch) on a GpuPort."""

    def __init__(self, metric, base, port="cpu"):
        base = _f32(base)
        self.dim = base.shape[1]
        self.lib = _port_lib(port)
        h = self.lib.ref_brute_create(METRIC[metric], c_uint32(self.dim), _p(base), c_size_t(base.shape[0]))
        if not h:
            raise RuntimeError("reference brute-force build failed")
        self.h = c_void_p(h)

    def search(self, queries, k, nthreads=None):
        queries = _f32(queries)
        nq = queries.shape[0]
        dist = np.empty((nq, k), np.float32)
        rows = np.empty((nq, k), np.int64)
        self.lib.ref_brute_search(self.h, c_uint32(self.dim), _p(queries), c_size_t(nq), c_size_t(k),
                                  c_int(_threads(nthreads)), _p(dist), _p(rows))
        return dist, rows

    def search_batch(self, queries, k):
        queries = _f32(queries)
        nq = queries.shape[0]
        dist = np.empty((nq, k), np.float32)
        rows = np.empty((nq, k), np.int64)
        rc = self.lib.ref_brute_search_batch(self.h, c_uint32(self.dim), _p(queries), c_size_t(nq), c_size_t(k),
                                             _p(dist), _p(rows))
        if rc != 0:
            raise RuntimeError(f"reference brute-force search_batch failed ({rc})")
        return dist, rows

    def __del__(self):
        try:
            self.lib.ref_brute_destroy(self.h)
        except Exception:
            pass


class B200PortIndex:
    """One of the B200 index adapters (elips_b200/integration/B200Indexes.cpp),
    selected by make_b200_index from an elips::Config and driven through the
    reference's own IndexPort / GpuIndexPort / IndexTransferPort calls (GPU
    only). Row i has RecordID row_id(i); results come back as rows.

    kind "brute_force" (precision "fp32" / "fp16" / "bf16"), "ivf_pq", or
    "quantized" (codec "sq8" with params = mins ++ scales, "pq" / "opq" with
    params = codebook)."""

    ALGO = {"brute_force": 4, "ivf_pq": 3}
    PRECISION = {"fp32": 0, "fp16": 1, "int8": 2, "auto": 3, "bf16": 4}
    CODEC = {"pq": 1, "opq": 2, "sq8": 3}

    def __init__(self, kind, metric, dim, precision="fp32", n_lists=1024, nprobe=64, pq_dim=0, pq_bits=8,
                 kmeans_iters=20, codec=None, params=None, rotation=None):
        self.lib = ref_b200()
        self.dim = int(dim)
        if kind == "quantized":
            params = _f32(params)
            rot = None if rotation is None else _f32(rotation)
            h = self.lib.ref_b200_quant_index_create(METRIC[metric], c_uint32(dim), c_int(self.CODEC[codec]),
                                                     c_uint32(pq_dim), c_uint32(pq_bits), _p(params),
                                                     None if rot is None else _p(rot))
        else:
            h = self.lib.ref_b200_index_create(METRIC[metric], c_uint32(dim), c_int(self.ALGO[kind]),
                                               c_int(self.PRECISION[precision]), c_size_t(n_lists),
                                               c_size_t(nprobe), c_uint32(pq_dim), c_uint32(pq_bits),
                                               c_size_t(kmeans_iters))
        if not h:
            raise RuntimeError("make_b200_index returned no index")
        self.h = c_void_p(h)

    def insert(self, rows, first=0):
        """IndexPort::insert of every row; returns False when it threw DimensionMismatch."""
        rows = _f32(rows)
        return self.lib.ref_b200_index_insert(self.h, _p(rows), c_size_t(rows.shape[0]), c_size_t(rows.shape[1]),
                                              c_size_t(first)) == 0

    def remove(self, row):
        self.lib.ref_b200_index_remove(self.h, c_size_t(row))

    def build(self, rows):
        rows = _f32(rows)
        return self.lib.ref_b200_index_build(self.h, _p(rows), c_size_t(rows.shape[0]), c_uint32(rows.shape[1]))

    def search(self, queries, k, nthreads=4):
        """IndexPort::search per query; (dist, rows, threw DimensionMismatch)."""
        queries = _f32(queries)
        nq = queries.shape[0]
        dist = np.zeros((nq, k), np.float32)
        rows = np.full((nq, k), -1, np.int64)
        rc = self.lib.ref_b200_index_search(self.h, c_uint32(queries.shape[1]), _p(queries), c_size_t(nq),
                                            c_size_t(k), c_int(nthreads), _p(dist), _p(rows))
        return dist, rows, rc == 1

    def search_batch(self, queries, k, candidates=None):
        """GpuIndexPort::search_batch (or the filtered form over candidate rows):
        (status 0 or 1 + GpuError, dist, rows)."""
        queries = _f32(queries)
        nq = queries.shape[0]
        dist = np.zeros((nq, k), np.float32)
        rows = np.full((nq, k), -1, np.int64)
        cand = None if candidates is None else np.ascontiguousarray(candidates, np.int64)
        rc = self.lib.ref_b200_index_search_batch(self.h, c_uint32(self.dim), _p(queries), c_size_t(nq), c_size_t(k),
                                                  None if cand is None else _p(cand),
                                                  c_size_t(0 if cand is None else cand.size), _p(dist), _p(rows))
        return rc, dist, rows

    def size(self):
        self.lib.ref_b200_index_size.restype = c_size_t
        return int(self.lib.ref_b200_index_size(self.h))

    def type_name(self):
        buf = ctypes.create_string_buffer(64)
        self.lib.ref_b200_index_type_name(self.h, buf, c_size_t(64))
        return buf.value.decode()

    def device_bytes(self):
        self.lib.ref_b200_index_device_bytes.restype = c_size_t
        return int(self.lib.ref_b200_index_device_bytes(self.h))

    def copy_snapshot_to(self, other):
        """export_snapshot of this index imported into `other`; 0 on success."""
        return self.lib.ref_b200_index_snapshot_copy(self.h, other.h)

    def export_to_cpu(self, metric):
        """export_to_cpu_index into a new CPU ExactIndex (a RefExactIndex)."""
        self.lib.ref_b200_index_export_to_cpu.restype = c_void_p
        h = self.lib.ref_b200_index_export_to_cpu(self.h, METRIC[metric], c_uint32(self.dim))
        if not h:
            raise RuntimeError("export_to_cpu_index failed")
        out = RefExactIndex.__new__(RefExactIndex)
        out.dim, out.h, out._lib = self.dim, c_void_p(h), self.lib
        return out

    def import_from_cpu(self, exact):
        return self.lib.ref_b200_index_import_from_cpu(self.h, exact.h)

    def centroids(self, n_lists):
        out = np.zeros((n_lists, self.dim), np.float32)
        self.lib.ref_b200_index_centroids.restype = c_size_t
        got = self.lib.ref_b200_index_centroids(self.h, _p(out), c_size_t(out.size))
        return out[:got]

    def export(self, n, pq_dim, ksub):
        """An IVF-PQ index's export_snapshot: (rows, vectors, assignments, codebook, codes)."""
        rows = np.empty(n, np.int64)
        vec = np.empty((n, self.dim), np.float32)
        asg = np.empty(n, np.uint32)
        cb = np.empty((pq_dim, ksub, self.dim // pq_dim), np.float32)
        codes = np.empty((n, pq_dim), np.uint8)
        rc = self.lib.ref_b200_index_export(self.h, c_size_t(n), c_uint32(self.dim), _p(rows), _p(vec), _p(asg),
                                            _p(cb), c_size_t(cb.size), _p(codes), c_size_t(codes.size))
        if rc != 0:
            raise RuntimeError(f"export_snapshot failed ({rc})")
        return rows, vec, asg, cb, codes

    def __del__(self):
        try:
            self.lib.ref_b200_index_destroy(self.h)
        except Exception:
            pass


class RefIvfFlatIndex:
    """The reference's GpuIVFFlatIndex on a CPU GpuPort, loaded via import_snapshot."""

    def __init__(self, metric, centroids, assignments, vectors, nprobe, port="cpu"):
        centroids, vectors = _f32(centroids), _f32(vectors)
        assignments = np.ascontiguousarray(assignments, np.uint32)
        self.dim = vectors.shape[1]
        self.lib = _port_lib(port)
        h = self.lib.ref_ivfflat_create(METRIC[metric], c_uint32(self.dim), c_size_t(centroids.shape[0]),
                                     c_size_t(nprobe), _p(centroids), _p(assignments), _p(vectors),
                                     c_size_t(vectors.shape[0]))
        if not h:
            raise RuntimeError("reference IVF-Flat import_snapshot failed")
        self.h = c_void_p(h)

    def search(self, queries, k, nthreads=None):
        queries = _f32(queries)
        nq = queries.shape[0]
        dist = np.empty((nq, k), np.float32)
        rows = np.empty((nq, k), np.int64)
        self.lib.ref_ivfflat_search(self.h, c_uint32(self.dim), _p(queries), c_size_t(nq), c_size_t(k),
                                 c_int(_threads(nthreads)), _p(dist), _p(rows))
        return dist, rows

    def search_batch(self, queries, k):
        queries = _f32(queries)
        nq = queries.shape[0]
        dist = np.empty((nq, k), np.float32)
        rows = np.empty((nq, k), np.int64)
        rc = self.lib.ref_ivfflat_search_batch(self.h, c_uint32(self.dim), _p(queries), c_size_t(nq), c_size_t(k),
                                            _p(dist), _p(rows))
        if rc != 0:
            raise RuntimeError(f"reference IVF-Flat search_batch failed ({rc})")
        return dist, rows

    def __del__(self):
        try:
            self.lib.ref_ivfflat_destroy(self.h)
        except Exception:
            pass


class RefIvfPqEmpty:
    """The reference's GpuIVFPQIndex on the CPU port, created empty (its own
    config: n_lists, nprobe, pq_dim, pq_bits, kmeans rounds), filled by
    insert or build_from_batch; search / remove / export as RefIvfPqIndex."""

    def __init__(self, metric, dim, n_lists, nprobe, pq_dim, pq_bits=8, kmeans_iters=20):
        self.lib = ref()
        self.dim = int(dim)
        self.lib.ref_ivfpq_create_empty.restype = c_void_p
        self.h = c_void_p(self.lib.ref_ivfpq_create_empty(METRIC[metric], c_uint32(dim), c_size_t(n_lists),
                                                          c_size_t(nprobe), c_uint32(pq_dim), c_uint32(pq_bits),
                                                          c_size_t(kmeans_iters)))

    def insert(self, rows, first=0):
        rows = _f32(rows)
        self.lib.ref_ivfpq_insert(self.h, _p(rows), c_size_t(rows.shape[0]), c_uint32(self.dim), c_size_t(first))

    def build(self, rows):
        rows = _f32(rows)
        return self.lib.ref_ivfpq_build(self.h, _p(rows), c_size_t(rows.shape[0]), c_uint32(self.dim))

    def size(self):
        self.lib.ref_ivfpq_size.restype = c_size_t
        return int(self.lib.ref_ivfpq_size(self.h))

    def centroids(self, n_lists):
        out = np.zeros((n_lists, self.dim), np.float32)
        self.lib.ref_ivfpq_centroids.restype = c_size_t
        got = self.lib.ref_ivfpq_centroids(self.h, _p(out), c_size_t(out.size))
        return out[:got]

    search = lambda self, *a, **kw: RefIvfPqIndex.search(self, *a, **kw)
    remove = lambda self, row: RefIvfPqIndex.remove(self, row)
    export = lambda self, *a: RefIvfPqIndex.export(self, *a)

    def __del__(self):
        try:
            self.lib.ref_ivfpq_destroy(self.h)
        except Exception:
            pass


class RefIvfPqIndex:
    """The reference's GpuIVFPQIndex on a CPU GpuPort, loaded via import_snapshot."""

    def __init__(self, metric, centroids, assignments, codebook, codes, vectors, nprobe, pq_bits=8, port="cpu"):
        centroids, codebook, vectors = _f32(centroids), _f32(codebook), _f32(vectors)
        assignments = np.ascontiguousarray(assignments, np.uint32)
        codes = np.ascontiguousarray(codes, np.uint8)
        self.dim = vectors.shape[1]
        self.lib = _port_lib(port)
        h = self.lib.ref_ivfpq_create(METRIC[metric], c_uint32(self.dim), c_size_t(centroids.shape[0]),
                                   c_size_t(nprobe), c_uint32(codebook.shape[0]), c_uint32(pq_bits),
                                   _p(centroids), _p(assignments), _p(codebook), _p(codes), _p(vectors),
                                   c_size_t(vectors.shape[0]))
        if not h:
            raise RuntimeError("reference IVF-PQ import_snapshot failed")
        self.h = c_void_p(h)

    def search(self, queries, k, nthreads=None):
        queries = _f32(queries)
        nq = queries.shape[0]
        dist = np.empty((nq, k), np.float32)
        rows = np.empty((nq, k), np.int64)
        self.lib.ref_ivfpq_search(self.h, c_uint32(self.dim), _p(queries), c_size_t(nq), c_size_t(k),
                               c_int(_threads(nthreads)), _p(dist), _p(rows))
        return dist, rows

    def remove(self, row):
        """GpuIVFPQIndex::remove of the record added as `row` (rebuilds the codes)."""
        self.lib.ref_ivfpq_remove(self.h, c_size_t(row))

    def export(self, n, pq_dim, ksub):
        """export_snapshot: (original rows, vectors, assignments, codebook, codes)."""
        rows = np.empty(n, np.int64)
        vec = np.empty((n, self.dim), np.float32)
        asg = np.empty(n, np.uint32)
        cb = np.empty((pq_dim, ksub, self.dim // pq_dim), np.float32)
        codes = np.empty((n, pq_dim), np.uint8)
        rc = self.lib.ref_ivfpq_export(self.h, c_size_t(n), c_uint32(self.dim), _p(rows), _p(vec), _p(asg), _p(cb),
                                       c_size_t(cb.size), _p(codes), c_size_t(codes.size))
        if rc != 0:
            raise RuntimeError(f"reference export_snapshot failed ({rc})")
        return rows, vec, asg, cb, codes

    def __del__(self):
        try:
            self.lib.ref_ivfpq_destroy(self.h)
        except Exception:
            pass


def ref_distance(metric, a, b):
    a, b = _f32(a), _f32(b)
    return float(ref().ref_distance(METRIC[metric], _p(a), _p(b), a.size))


def ref_sq8_train(metric, rows):
    rows = _f32(rows)
    n, d = rows.shape
    mins = np.empty(d, np.float32)
    scales = np.empty(d, np.float32)
    ref().ref_sq8_train(METRIC[metric], c_uint32(d), _p(rows), c_size_t(n), _p(mins), _p(scales))
    return mins, scales


def ref_sq8_encode(metric, mins, scales, rows):
    rows = _f32(rows)
    n, d = rows.shape
    codes = np.empty((n, d), np.uint8)
    ref().ref_sq8_encode(METRIC[metric], c_uint32(d), _p(_f32(mins)), _p(_f32(scales)), _p(rows),
                         c_size_t(n), _p(codes))
    return codes


def ref_train_pq_codebook(rows, m, ksub, iters):
    rows = _f32(rows)
    n, d = rows.shape
    cb = np.empty((m, ksub, d // m), np.float32)
    ref().ref_train_pq_codebook(_p(rows), c_size_t(n), c_size_t(d), c_size_t(m), c_size_t(ksub),
                                c_size_t(iters), _p(cb))
    return cb


def ref_encode_pq(codebook, rows):
    codebook, rows = _f32(codebook), _f32(rows)
    m, ksub, sub = codebook.shape
    n, d = rows.shape
    codes = np.empty((n, m), np.uint8)
    ref().ref_encode_pq(_p(rows), _p(codebook), c_size_t(n), c_size_t(d), c_size_t(m), c_size_t(ksub),
                        _p(codes))
    return codes


def ref_kmeans(rows, k, iters):
    rows = _f32(rows)
    n, d = rows.shape
    cent = np.empty((k, d), np.float32)
    ref().ref_kmeans(_p(rows), c_size_t(n), c_size_t(d), c_size_t(k), c_size_t(iters), _p(cent))
    return cent
