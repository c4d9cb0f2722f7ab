/*
 * oracle.c -- CPU restatement of the reference's k-NN search arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker the parity tests compare
 * the CUDA kernels against; it is never linked into, loaded by, or called from
 * the product library (elips_b200/). Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline leg may load it.
 *
 * Every function cites the reference file:line it restates (paths relative to
 * the axiomchronicles/elips source tree). The arithmetic is single precision,
 * strictly sequential, with no fused multiply-add (built with
 * -ffp-contract=off, -mno-fma): that is what the reference's scalar loops
 * compile to on x86-64 with its default flags. Pinned against the reference's
 * own compiled code (oracle/_ref/libelips_ref.so, built by oracle/Makefile) by
 * tests/test_oracle_pin.py and against the committed golden fixtures in
 * tests/golden/.
 *
 * Ordering convention: results are sorted ascending by (distance, row). The
 * reference sorts by distance only with std::partial_sort (ExactIndex.cpp:
 * 81-84), which leaves the order of equal distances unspecified; (distance,
 * row) is one valid instance of it and is what the GPU path produces.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { ORC_COSINE = 0, ORC_EUCLIDEAN = 1, ORC_DOT = 2 }; /* elips::Metric, Config.hpp:27 */

/* ------------------------------------------------------------------------ */
/* Metrics.cpp                                                                */
/* ------------------------------------------------------------------------ */

/* dot_scalar, Metrics.cpp:20-27 */
static float dot_seq(const float* a, const float* b, size_t n) {
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) sum += a[i] * b[i];
    return sum;
}

/* sql2_scalar, Metrics.cpp:29-37 */
static float sql2_seq(const float* a, const float* b, size_t n) {
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        const float d = a[i] - b[i];
        sum += d * d;
    }
    return sum;
}

/* elips::distance, Metrics.cpp:104-115 */
float orc_distance(int metric, const float* a, const float* b, size_t n) {
    switch (metric) {
        case ORC_COSINE: return 1.0f - dot_seq(a, b, n);
        case ORC_EUCLIDEAN: return sqrtf(sql2_seq(a, b, n));
        case ORC_DOT: return -dot_seq(a, b, n);
    }
    return 0.0f;
}

/* Vector::normalized, include/elips/domain/Vector.hpp:25-44: magnitude =
 * sqrt(sequential sum of v*v); zero vectors unchanged; else v / magnitude. */
void orc_normalize_rows(const float* in, float* out, size_t n, size_t d) {
    for (size_t r = 0; r < n; ++r) {
        const float* x = in + r * d;
        float sum = 0.0f;
        for (size_t i = 0; i < d; ++i) sum += x[i] * x[i];
        const float mag = sqrtf(sum);
        for (size_t i = 0; i < d; ++i) out[r * d + i] = mag == 0.0f ? x[i] : x[i] / mag;
    }
}

/* ------------------------------------------------------------------------ */
/* k smallest by (distance, row): a bounded max-heap                          */
/* ------------------------------------------------------------------------ */

typedef struct { float d; int64_t r; } hit_t;

static int hit_less(hit_t a, hit_t b) { return a.d < b.d || (a.d == b.d && a.r < b.r); }

typedef struct { hit_t* h; size_t n, cap; } heap_t;

static void heap_push(heap_t* hp, hit_t x) {
    if (hp->cap == 0) return;
    if (hp->n < hp->cap) {
        size_t i = hp->n++;
        hp->h[i] = x;
        while (i > 0) {
            size_t p = (i - 1) / 2;
            if (!hit_less(hp->h[p], hp->h[i])) break;
            hit_t t = hp->h[p]; hp->h[p] = hp->h[i]; hp->h[i] = t;
            i = p;
        }
        return;
    }
    if (!hit_less(x, hp->h[0])) return;
    hp->h[0] = x;
    size_t i = 0;
    for (;;) {
        size_t l = 2 * i + 1, r = l + 1, m = i;
        if (l < hp->n && hit_less(hp->h[m], hp->h[l])) m = l;
        if (r < hp->n && hit_less(hp->h[m], hp->h[r])) m = r;
        if (m == i) break;
        hit_t t = hp->h[m]; hp->h[m] = hp->h[i]; hp->h[i] = t;
        i = m;
    }
}

static int hit_cmp(const void* a, const void* b) {
    const hit_t x = *(const hit_t*)a, y = *(const hit_t*)b;
    if (hit_less(x, y)) return -1;
    if (hit_less(y, x)) return 1;
    return 0;
}

/* Sorts the heap ascending and writes k slots; empty slots get row -1. */
static void heap_emit(heap_t* hp, size_t k, float* out_d, int64_t* out_r) {
    qsort(hp->h, hp->n, sizeof(hit_t), hit_cmp);
    for (size_t i = 0; i < k; ++i) {
        if (i < hp->n) { out_d[i] = hp->h[i].d; out_r[i] = hp->h[i].r; }
        else { out_d[i] = 0.0f; out_r[i] = -1; }
    }
}

/* ------------------------------------------------------------------------ */
/* query-parallel driver                                                      */
/* ------------------------------------------------------------------------ */

typedef void (*query_fn)(const void* ctx, size_t q, hit_t* scratch);

typedef struct {
    const void* ctx; query_fn fn; size_t nq, stride, first, scratch_n;
} worker_t;

static void* worker_main(void* arg) {
    worker_t* w = (worker_t*)arg;
    hit_t* scratch = (hit_t*)malloc(sizeof(hit_t) * (w->scratch_n ? w->scratch_n : 1));
    for (size_t q = w->first; q < w->nq; q += w->stride) w->fn(w->ctx, q, scratch);
    free(scratch);
    return NULL;
}

static void run_queries(const void* ctx, query_fn fn, size_t nq, int nthreads, size_t scratch_n) {
    size_t nt = nthreads < 1 ? 1 : (size_t)nthreads;
    if (nt > nq) nt = nq ? nq : 1;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nt);
    worker_t* ws = (worker_t*)malloc(sizeof(worker_t) * nt);
    for (size_t t = 0; t < nt; ++t) {
        ws[t].ctx = ctx; ws[t].fn = fn; ws[t].nq = nq; ws[t].stride = nt; ws[t].first = t;
        ws[t].scratch_n = scratch_n;
        if (nt == 1) worker_main(&ws[t]);
        else pthread_create(&th[t], NULL, worker_main, &ws[t]);
    }
    if (nt > 1) for (size_t t = 0; t < nt; ++t) pthread_join(th[t], NULL);
    free(th); free(ws);
}

/* ------------------------------------------------------------------------ */
/* ExactIndex::search over fp32 rows, ExactIndex.cpp:55-87 (plain branch     */
/* :72-78, then partial_sort :80-86).                                         */
/* ------------------------------------------------------------------------ */

typedef struct {
    int metric; const float* base; size_t n, d; const float* queries; size_t k;
    float* out_d; int64_t* out_r;
} exact_ctx;

static void exact_one(const void* c, size_t q, hit_t* scratch) {
    const exact_ctx* x = (const exact_ctx*)c;
    heap_t hp = { scratch, 0, x->k };
    const float* qv = x->queries + q * x->d;
    for (size_t i = 0; i < x->n; ++i) {
        hit_t h = { orc_distance(x->metric, qv, x->base + i * x->d, x->d), (int64_t)i };
        heap_push(&hp, h);
    }
    heap_emit(&hp, x->k, x->out_d + q * x->k, x->out_r + q * x->k);
}

void orc_exact_search(int metric, const float* base, size_t n, size_t d, const float* queries,
                      size_t nq, size_t k, int nthreads, float* out_d, int64_t* out_r) {
    exact_ctx c = { metric, base, n, d, queries, k, out_d, out_r };
    run_queries(&c, exact_one, nq, nthreads, k);
}

/* Filtered exact search: the ExactIndex scan restricted to the candidate row
 * set that MetadataIndex::exact_candidates returns (MetadataIndex.cpp:66-99),
 * as Vault::search_records does for a candidate subset (Database.cpp:
 * 1065-1126). The set is given as a bitmask over rows, bit (i & 31) of word
 * (i >> 5). */
typedef struct {
    exact_ctx e; const uint32_t* mask;
} masked_ctx;

static void masked_one(const void* c, size_t q, hit_t* scratch) {
    const masked_ctx* m = (const masked_ctx*)c;
    const exact_ctx* x = &m->e;
    heap_t hp = { scratch, 0, x->k };
    const float* qv = x->queries + q * x->d;
    for (size_t i = 0; i < x->n; ++i) {
        if (!((m->mask[i >> 5] >> (i & 31)) & 1u)) continue;
        hit_t h = { orc_distance(x->metric, qv, x->base + i * x->d, x->d), (int64_t)i };
        heap_push(&hp, h);
    }
    heap_emit(&hp, x->k, x->out_d + q * x->k, x->out_r + q * x->k);
}

void orc_exact_search_masked(int metric, const float* base, size_t n, size_t d,
                             const uint32_t* mask, const float* queries, size_t nq, size_t k,
                             int nthreads, float* out_d, int64_t* out_r) {
    masked_ctx c = { { metric, base, n, d, queries, k, out_d, out_r }, mask };
    run_queries(&c, masked_one, nq, nthreads, k);
}

/* ------------------------------------------------------------------------ */
/* Symmetric int8 inner-product codec. NO REFERENCE COUNTERPART: the         */
/* reference's only 8-bit codec is the unsigned affine sq8 below. The score   */
/* is -(float)(sum_i q_i * x_i) with the sum exact in int32 (|sum| <=        */
/* 1024*127*127 < 2^24, so the float conversion is exact too), ordered the    */
/* same way as the reference's dot_product metric (Metrics.cpp:111-112).     */
/* ------------------------------------------------------------------------ */

typedef struct {
    const int8_t* base; size_t n, d; const int8_t* queries; size_t k; float* out_d; int64_t* out_r;
} i8_ctx;

static void i8_one(const void* c, size_t q, hit_t* scratch) {
    const i8_ctx* x = (const i8_ctx*)c;
    heap_t hp = { scratch, 0, x->k };
    const int8_t* qv = x->queries + q * x->d;
    for (size_t i = 0; i < x->n; ++i) {
        const int8_t* r = x->base + i * x->d;
        int32_t acc = 0;
        for (size_t j = 0; j < x->d; ++j) acc += (int32_t)qv[j] * (int32_t)r[j];
        hit_t h = { -(float)acc, (int64_t)i };
        heap_push(&hp, h);
    }
    heap_emit(&hp, x->k, x->out_d + q * x->k, x->out_r + q * x->k);
}

void orc_int8_ip_search(const int8_t* base, size_t n, size_t d, const int8_t* queries, size_t nq,
                        size_t k, int nthreads, float* out_d, int64_t* out_r) {
    i8_ctx c = { base, n, d, queries, k, out_d, out_r };
    run_queries(&c, i8_one, nq, nthreads, k);
}

/* ------------------------------------------------------------------------ */
/* ScalarQuantizer (sq8), ScalarQuantizer.cpp                                */
/* ------------------------------------------------------------------------ */

/* ScalarQuantizer::train, ScalarQuantizer.cpp:26-50 */
void orc_sq8_train(size_t d, const float* rows, size_t n, float* mins, float* scales) {
    float* maxes = (float*)malloc(sizeof(float) * d);
    for (size_t i = 0; i < d; ++i) { mins[i] = 3.40282347e+38f; maxes[i] = -3.40282347e+38f; }
    for (size_t r = 0; r < n; ++r) {
        const float* v = rows + r * d;
        for (size_t i = 0; i < d; ++i) {
            if (v[i] < mins[i]) mins[i] = v[i];
            if (maxes[i] < v[i]) maxes[i] = v[i];
        }
    }
    for (size_t i = 0; i < d; ++i) {
        const float range = maxes[i] - mins[i];
        scales[i] = (range > 0.0f) ? (range / 255.0f) : 1.0f;
    }
    free(maxes);
}

/* ScalarQuantizer::encode, ScalarQuantizer.cpp:52-68: std::clamp then
 * std::lround (round half away from zero). */
void orc_sq8_encode(size_t d, const float* mins, const float* scales, const float* rows, size_t n,
                    uint8_t* codes) {
    for (size_t r = 0; r < n; ++r) {
        for (size_t i = 0; i < d; ++i) {
            const float level = (rows[r * d + i] - mins[i]) / scales[i];
            const float clamped = level < 0.0f ? 0.0f : (255.0f < level ? 255.0f : level);
            codes[r * d + i] = (uint8_t)lroundf(clamped);
        }
    }
}

/* ScalarQuantizer::make_lut, ScalarQuantizer.cpp:83-110: d x 256 table. */
void orc_sq8_make_lut(int metric, size_t d, const float* mins, const float* scales,
                      const float* query, float* lut) {
    const int use_dot = metric != ORC_EUCLIDEAN;
    for (size_t i = 0; i < d; ++i) {
        for (size_t level = 0; level < 256; ++level) {
            const float value = mins[i] + ((float)level * scales[i]);
            if (use_dot) {
                lut[i * 256 + level] = -(query[i] * value);
            } else {
                const float t = query[i] - value;
                lut[i * 256 + level] = t * t;
            }
        }
    }
}

/* ScalarQuantizer::lut_distance, ScalarQuantizer.cpp:112-128 */
float orc_sq8_lut_distance(int metric, size_t d, const float* lut, const uint8_t* code) {
    float sum = 0.0f;
    for (size_t i = 0; i < d; ++i) sum += lut[i * 256 + code[i]];
    switch (metric) {
        case ORC_COSINE: return 1.0f + sum;
        case ORC_DOT: return sum;
        case ORC_EUCLIDEAN: return sqrtf(0.0f < sum ? sum : 0.0f);
    }
    return sum;
}

/* ExactIndex::search, compressed branch, ExactIndex.cpp:62-71 */
typedef struct {
    int metric; size_t d; const float* mins; const float* scales; const uint8_t* codes; size_t n;
    const float* queries; size_t k; float* out_d; int64_t* out_r;
} sq8_ctx;

static void sq8_one(const void* c, size_t q, hit_t* scratch) {
    const sq8_ctx* x = (const sq8_ctx*)c;
    float* lut = (float*)malloc(sizeof(float) * x->d * 256);
    orc_sq8_make_lut(x->metric, x->d, x->mins, x->scales, x->queries + q * x->d, lut);
    heap_t hp = { scratch, 0, x->k };
    for (size_t i = 0; i < x->n; ++i) {
        hit_t h = { orc_sq8_lut_distance(x->metric, x->d, lut, x->codes + i * x->d), (int64_t)i };
        heap_push(&hp, h);
    }
    heap_emit(&hp, x->k, x->out_d + q * x->k, x->out_r + q * x->k);
    free(lut);
}

void orc_sq8_search(int metric, size_t d, const float* mins, const float* scales,
                    const uint8_t* codes, size_t n, const float* queries, size_t nq, size_t k,
                    int nthreads, float* out_d, int64_t* out_r) {
    sq8_ctx c = { metric, d, mins, scales, codes, n, queries, k, out_d, out_r };
    run_queries(&c, sq8_one, nq, nthreads, k);
}

/* ------------------------------------------------------------------------ */
/* ProductQuantizer (plain PQ, no rotation), ProductQuantizer.cpp            */
/* codebook layout [M][ksub][sub] (ProductQuantizer.hpp:102-104)             */
/* ------------------------------------------------------------------------ */

/* ProductQuantizer::make_lut, ProductQuantizer.cpp:118-160 */
void orc_pq_make_lut(int metric, size_t d, size_t m, size_t ksub, const float* codebook,
                     const float* query, float* lut) {
    const size_t sub = d / m;
    const int use_dot = metric != ORC_EUCLIDEAN;
    for (size_t s = 0; s < m; ++s) {
        const float* qs = query + s * sub;
        const float* cb = codebook + s * ksub * sub;
        for (size_t c = 0; c < ksub; ++c) {
            const float* cen = cb + c * sub;
            float acc = 0.0f;
            if (use_dot) {
                for (size_t i = 0; i < sub; ++i) acc += qs[i] * cen[i];
                lut[s * ksub + c] = -acc;
            } else {
                for (size_t i = 0; i < sub; ++i) {
                    const float t = qs[i] - cen[i];
                    acc += t * t;
                }
                lut[s * ksub + c] = acc;
            }
        }
    }
}

/* ProductQuantizer::lut_distance, ProductQuantizer.cpp:162-183 */
float orc_pq_lut_distance(int metric, size_t m, size_t ksub, const float* lut, const uint8_t* code) {
    float sum = 0.0f;
    for (size_t s = 0; s < m; ++s) sum += lut[s * ksub + code[s]];
    switch (metric) {
        case ORC_COSINE: return 1.0f + sum;
        case ORC_DOT: return sum;
        case ORC_EUCLIDEAN: return sqrtf(0.0f < sum ? sum : 0.0f);
    }
    return sum;
}

typedef struct {
    int metric; size_t d, m, ksub; const float* codebook; const uint8_t* codes; size_t n;
    const float* queries; size_t k; float* out_d; int64_t* out_r;
} pq_ctx;

static void pq_one(const void* c, size_t q, hit_t* scratch) {
    const pq_ctx* x = (const pq_ctx*)c;
    float* lut = (float*)malloc(sizeof(float) * x->m * x->ksub);
    orc_pq_make_lut(x->metric, x->d, x->m, x->ksub, x->codebook, x->queries + q * x->d, lut);
    heap_t hp = { scratch, 0, x->k };
    for (size_t i = 0; i < x->n; ++i) {
        hit_t h = { orc_pq_lut_distance(x->metric, x->m, x->ksub, lut, x->codes + i * x->m),
                    (int64_t)i };
        heap_push(&hp, h);
    }
    heap_emit(&hp, x->k, x->out_d + q * x->k, x->out_r + q * x->k);
    free(lut);
}

/* ExactIndex::search with a ProductQuantizer attached, ExactIndex.cpp:62-71 */
void orc_pq_search(int metric, size_t d, size_t m, size_t ksub, const float* codebook,
                   const uint8_t* codes, size_t n, const float* queries, size_t nq, size_t k,
                   int nthreads, float* out_d, int64_t* out_r) {
    pq_ctx c = { metric, d, m, ksub, codebook, codes, n, queries, k, out_d, out_r };
    run_queries(&c, pq_one, nq, nthreads, k);
}

/* ------------------------------------------------------------------------ */
/* k-means and PQ encode, KMeans.cpp                                         */
/* ------------------------------------------------------------------------ */

/* nearest_centroid, KMeans.cpp:166-180 (strict '<': lowest index wins) */
uint8_t orc_nearest_centroid(const float* v, const float* cb, size_t sub, size_t ksub) {
    float best = 3.40282347e+38f;
    size_t arg = 0;
    for (size_t c = 0; c < ksub; ++c) {
        const float dd = sql2_seq(v, cb + c * sub, sub);
        if (dd < best) { best = dd; arg = c; }
    }
    return (uint8_t)arg;
}

/* encode_pq, KMeans.cpp:270-285 */
void orc_encode_pq(const float* rows, const float* codebook, size_t n, size_t d, size_t m,
                   size_t ksub, uint8_t* codes) {
    const size_t sub = d / m;
    for (size_t r = 0; r < n; ++r)
        for (size_t s = 0; s < m; ++s)
            codes[r * m + s] = orc_nearest_centroid(rows + r * d + s * sub,
                                                    codebook + s * ksub * sub, sub, ksub);
}

/* kmeans, KMeans.cpp:182-247: strided seed, Lloyd, empty-cluster reseed,
 * early stop when no centroid component changes. */
void orc_kmeans(const float* rows, size_t n, size_t dim, size_t k, size_t iters, float* cent) {
    if (n == 0 || dim == 0 || k == 0) return;
    const size_t stride = (n / k) > 1 ? (n / k) : 1;
    for (size_t c = 0; c < k; ++c) {
        size_t sample = c * stride;
        if (sample > n - 1) sample = n - 1;
        memcpy(cent + c * dim, rows + sample * dim, sizeof(float) * dim);
    }
    float* sums = (float*)malloc(sizeof(float) * k * dim);
    size_t* counts = (size_t*)malloc(sizeof(size_t) * k);
    for (size_t it = 0; it < iters; ++it) {
        memset(sums, 0, sizeof(float) * k * dim);
        memset(counts, 0, sizeof(size_t) * k);
        for (size_t r = 0; r < n; ++r) {
            const float* v = rows + r * dim;
            float best = 3.40282347e+38f;
            size_t arg = 0;
            for (size_t c = 0; c < k; ++c) {
                const float dd = sql2_seq(v, cent + c * dim, dim);
                if (dd < best) { best = dd; arg = c; }
            }
            ++counts[arg];
            for (size_t i = 0; i < dim; ++i) sums[arg * dim + i] += v[i];
        }
        int moved = 0;
        for (size_t c = 0; c < k; ++c) {
            float* cc = cent + c * dim;
            if (counts[c] == 0) {
                memcpy(cc, rows + (c % n) * dim, sizeof(float) * dim);
                moved = 1;
                continue;
            }
            const float inv = 1.0f / (float)counts[c];
            for (size_t i = 0; i < dim; ++i) {
                const float upd = sums[c * dim + i] * inv;
                if (upd != cc[i]) moved = 1;
                cc[i] = upd;
            }
        }
        if (!moved) break;
    }
    free(sums); free(counts);
}

/* detail::apply_matrix, KMeans.cpp:295-305: out_i = sum_j R[i][j] * v[j],
 * sequential over j. OPQ rotates rows before encode and queries before
 * make_lut with it (ProductQuantizer.cpp:41-48, 79-85, 127-133). */
void orc_rotate_rows(const float* rot, const float* rows, size_t n, size_t d, float* out) {
    for (size_t r = 0; r < n; ++r) {
        for (size_t i = 0; i < d; ++i) {
            const float* m = rot + i * d;
            float sum = 0.0f;
            for (size_t j = 0; j < d; ++j) sum += m[j] * rows[r * d + j];
            out[r * d + i] = sum;
        }
    }
}

/* ------------------------------------------------------------------------ */
/* IVF coarse assignment and IVF-PQ search                                    */
/* ------------------------------------------------------------------------ */

/* IvfIndexState::assign_vectors_to_centroids, IvfIndexState.cpp:167-191
 * (elips::distance, strict '<': lowest list id wins). */
void orc_ivf_assign(int metric, const float* rows, size_t n, size_t d, const float* centroids,
                    size_t nlist, uint32_t* out) {
    for (size_t r = 0; r < n; ++r) {
        float best = 3.40282347e+38f;
        uint32_t arg = 0;
        for (size_t l = 0; l < nlist; ++l) {
            const float dd = orc_distance(metric, rows + r * d, centroids + l * d, d);
            if (dd < best) { best = dd; arg = (uint32_t)l; }
        }
        out[r] = arg;
    }
}

/* IvfIndexState::probe_lists, IvfIndexState.cpp:395-423: distances to every
 * centroid, then the nprobe smallest (ties by list id). */
/* IvfIndexState::train_centroids (IvfIndexState.cpp:118-165): strided seeds
 * (min(n-1, list*stride)), max(1, iters) Lloyd rounds with no early stop:
 * assign by elips::distance (strict '<', lowest list wins, :167-191), sums in
 * row order, centroid = sum / count (division), an empty list reseeded from
 * row min(n-1, list % n), then normalize_if_needed (cosine: divide by the
 * sequential magnitude when it is > 0, :20-35). Then the final assignment. */
void orc_ivf_train(int metric, const float* rows, size_t n, size_t d, size_t nlist, size_t iters,
                   float* cent, uint32_t* assign) {
    if (n == 0 || d == 0 || nlist == 0) return;
    const size_t stride = (n / nlist) > 1 ? (n / nlist) : 1;
    for (size_t l = 0; l < nlist; ++l) {
        size_t sample = l * stride;
        if (sample > n - 1) sample = n - 1;
        memcpy(cent + l * d, rows + sample * d, sizeof(float) * d);
    }
    float* sums = (float*)malloc(sizeof(float) * nlist * d);
    size_t* counts = (size_t*)malloc(sizeof(size_t) * nlist);
    const size_t rounds = iters > 0 ? iters : 1;
    for (size_t it = 0; it < rounds; ++it) {
        orc_ivf_assign(metric, rows, n, d, cent, nlist, assign);
        memset(sums, 0, sizeof(float) * nlist * d);
        memset(counts, 0, sizeof(size_t) * nlist);
        for (size_t r = 0; r < n; ++r) {
            const uint32_t l = assign[r];
            ++counts[l];
            for (size_t i = 0; i < d; ++i) sums[l * d + i] += rows[r * d + i];
        }
        for (size_t l = 0; l < nlist; ++l) {
            float* c = cent + l * d;
            if (counts[l] == 0) {
                size_t fb = l % n;
                if (fb > n - 1) fb = n - 1;
                memcpy(c, rows + fb * d, sizeof(float) * d);
            } else {
                for (size_t i = 0; i < d; ++i) c[i] = sums[l * d + i] / (float)counts[l];
            }
            if (metric == ORC_COSINE) {
                float norm = 0.0f;
                for (size_t i = 0; i < d; ++i) norm += c[i] * c[i];
                norm = sqrtf(norm);
                if (!(norm <= 0.0f))
                    for (size_t i = 0; i < d; ++i) c[i] /= norm;
            }
        }
    }
    orc_ivf_assign(metric, rows, n, d, cent, nlist, assign);
    free(sums); free(counts);
}

/* train_pq_codebook, KMeans.cpp:249-268: each subspace gathered into dense
 * rows, then kmeans (codebook [m][ksub][sub]). */
void orc_train_pq_codebook(const float* rows, size_t n, size_t d, size_t m, size_t ksub, size_t iters,
                           float* codebook) {
    if (n == 0 || m == 0 || d == 0 || d % m != 0 || ksub == 0) return;
    const size_t sub = d / m;
    float* scratch = (float*)malloc(sizeof(float) * n * sub);
    for (size_t s = 0; s < m; ++s) {
        for (size_t r = 0; r < n; ++r) memcpy(scratch + r * sub, rows + r * d + s * sub, sizeof(float) * sub);
        orc_kmeans(scratch, n, sub, ksub, iters, codebook + s * ksub * sub);
    }
    free(scratch);
}

void orc_ivf_probe(int metric, const float* query, size_t d, const float* centroids, size_t nlist,
                   size_t nprobe, uint32_t* out_lists, float* out_dist) {
    hit_t* scratch = (hit_t*)malloc(sizeof(hit_t) * (nprobe ? nprobe : 1));
    heap_t hp = { scratch, 0, nprobe };
    for (size_t l = 0; l < nlist; ++l) {
        hit_t h = { orc_distance(metric, query, centroids + l * d, d), (int64_t)l };
        heap_push(&hp, h);
    }
    qsort(hp.h, hp.n, sizeof(hit_t), hit_cmp);
    for (size_t i = 0; i < nprobe; ++i) {
        out_lists[i] = i < hp.n ? (uint32_t)hp.h[i].r : 0xFFFFFFFFu;
        if (out_dist) out_dist[i] = i < hp.n ? hp.h[i].d : 0.0f;
    }
    free(scratch);
}

typedef struct {
    int metric; size_t d, m, ksub, nlist, nprobe;
    const float* centroids; const float* codebook; const uint8_t* codes; const float* vectors;
    const uint32_t* list_offsets; const uint32_t* list_rows; /* CSR: members of each list */
    const float* queries; size_t k; int mode; float* out_d; int64_t* out_r; float* out_gap;
} ivfpq_ctx;

typedef struct { float d; uint32_t row; } cand_t;

/* std::partial_sort(first, middle, last, by distance) as GNU libstdc++
 * (bits/stl_algo.h, bits/stl_heap.h; GCC 13.3 here, unchanged for many
 * releases) implements it: heap-select (build a max-heap over [first, middle)
 * bottom-up, then every later element strictly below the root replaces it by
 * a pop), then heap-sort of [first, middle). The standard leaves the order of
 * equal distances unspecified; this restates the one the reference's build
 * actually produces, so that candidates tied at the rerank boundary are
 * chosen exactly as the reference chooses them. */
static int cand_less(const cand_t* a, const cand_t* b) { return a->d < b->d; }

/* Moves the hole at `hole` down to a leaf (always along the larger child,
 * the right one unless the left is strictly larger), then sifts `v` up from
 * there, no higher than `top`. */
static void heap_adjust(cand_t* a, size_t hole, size_t len, cand_t v) {
    const size_t top = hole;
    size_t child = hole;
    while (len > 2 && child < (len - 1) / 2) {
        child = 2 * (child + 1);
        if (cand_less(&a[child], &a[child - 1])) --child;
        a[hole] = a[child];
        hole = child;
    }
    if ((len & 1) == 0 && len >= 2 && child == (len - 2) / 2) {
        child = 2 * (child + 1);
        a[hole] = a[child - 1];
        hole = child - 1;
    }
    while (hole > top) {
        const size_t parent = (hole - 1) / 2;
        if (!cand_less(&a[parent], &v)) break;
        a[hole] = a[parent];
        hole = parent;
    }
    a[hole] = v;
}

static void partial_sort_libstdcxx(cand_t* a, size_t mid, size_t n) {
    if (mid < 2) {  /* one-element heap: replacement still follows the root test */
        for (size_t i = mid; mid == 1 && i < n; ++i)
            if (cand_less(&a[i], &a[0])) { cand_t t = a[0]; a[0] = a[i]; a[i] = t; }
        return;
    }
    for (size_t parent = (mid - 2) / 2;; --parent) {
        heap_adjust(a, parent, mid, a[parent]);
        if (parent == 0) break;
    }
    for (size_t i = mid; i < n; ++i) {
        if (cand_less(&a[i], &a[0])) {  /* pop: the root goes to i, a[i] re-enters */
            const cand_t v = a[i];
            a[i] = a[0];
            heap_adjust(a, 0, mid, v);
        }
    }
    for (size_t last = mid; last > 1;) {  /* sort_heap */
        --last;
        const cand_t v = a[last];
        a[last] = a[0];
        heap_adjust(a, 0, last, v);
    }
}

static int cand_slot_cmp(const void* a, const void* b) {
    const cand_t* x = (const cand_t*)a; const cand_t* y = (const cand_t*)b;
    if (x->d < y->d) return -1;
    if (y->d < x->d) return 1;
    return x->row < y->row ? -1 : (x->row > y->row);
}

/* Approximate distance of one candidate, decoded as centroid + codeword in
 * fp32 (decode_candidate_vector, GpuIVFPQIndex.cpp:132-148).
 * mode 0: elips::distance on the decoded vector, one sequential sum over all
 *         dimensions (GpuIVFPQIndex.cpp:204);
 * mode 1: the same per-dimension terms summed per subspace, then the subspace
 *         sums in order: the lookup-table grouping the device scan uses. */
static float ivfpq_approx(const ivfpq_ctx* x, const float* qv, const float* cen, const uint8_t* code, float* dec) {
    const size_t d = x->d, sub = d / x->m;
    if (x->mode == 0) {
        for (size_t s = 0; s < x->m; ++s) {
            const float* cw = x->codebook + (s * x->ksub + code[s]) * sub;
            for (size_t t = 0; t < sub; ++t) dec[s * sub + t] = cen[s * sub + t] + cw[t];
        }
        return orc_distance(x->metric, qv, dec, d);
    }
    float total = 0.0f;
    for (size_t s = 0; s < x->m; ++s) {
        const float* cw = x->codebook + (s * x->ksub + code[s]) * sub;
        float acc = 0.0f;
        for (size_t t = 0; t < sub; ++t) {
            const size_t i = s * sub + t;
            const float dv = cen[i] + cw[t];
            if (x->metric == ORC_EUCLIDEAN) { const float df = qv[i] - dv; acc += df * df; }
            else acc += qv[i] * dv;
        }
        total += acc;
    }
    if (x->metric == ORC_EUCLIDEAN) return sqrtf(total);
    return x->metric == ORC_COSINE ? 1.0f - total : -total;
}

/* GpuIVFPQIndex::search, GpuIVFPQIndex.cpp:161-237:
 *   probe_lists -> gather_candidates (probe order, then list member order,
 *   IvfIndexState.cpp:466-504) -> approximate distance per candidate
 *   (:190-206) -> keep R = max(4k, k) smallest (:208-218) -> exact_rank:
 *   exact elips::distance on the raw vectors and top-k (:37-71, :235-236).
 * mode 0 is the reference's own order: R chosen by libstdc++'s partial_sort,
 *   exact top-k ties broken by rerank position (GpuPort::top_k order);
 * mode 1 is the device path's documented order: approximate sums grouped by
 *   subspace, ties broken by slot in both stages.
 * out_gap[q] (optional): relative gap between the R-th smallest approximate
 *   distance and the smallest one left out (0 = tied at the boundary, +inf =
 *   nothing left out), in this mode's arithmetic. */
static void ivfpq_one(const void* c, size_t q, hit_t* scratch) {
    const ivfpq_ctx* x = (const ivfpq_ctx*)c;
    const size_t d = x->d;
    const float* qv = x->queries + q * d;
    uint32_t* lists = (uint32_t*)malloc(sizeof(uint32_t) * x->nprobe);
    orc_ivf_probe(x->metric, qv, d, x->centroids, x->nlist, x->nprobe, lists, NULL);
    size_t total = 0;
    for (size_t p = 0; p < x->nprobe; ++p)
        if (lists[p] < x->nlist) total += x->list_offsets[lists[p] + 1] - x->list_offsets[lists[p]];
    cand_t* cands = (cand_t*)malloc(sizeof(cand_t) * (total ? total : 1));
    float* dec = (float*)malloc(sizeof(float) * d);
    size_t nc = 0;
    for (size_t p = 0; p < x->nprobe; ++p) {
        const uint32_t l = lists[p];
        if (l >= x->nlist) continue;
        const float* cen = x->centroids + (size_t)l * d;
        for (uint32_t j = x->list_offsets[l]; j < x->list_offsets[l + 1]; ++j) {
            const uint32_t row = x->list_rows[j];
            cands[nc].d = ivfpq_approx(x, qv, cen, x->codes + (size_t)row * x->m, dec);
            cands[nc].row = row;
            ++nc;
        }
    }
    size_t rk = 4 * x->k > x->k ? 4 * x->k : x->k;
    if (rk > nc) rk = nc;
    if (x->mode == 0) partial_sort_libstdcxx(cands, rk, nc);
    else qsort(cands, nc, sizeof(cand_t), cand_slot_cmp);
    if (x->out_gap) {
        float g = INFINITY;
        if (rk > 0 && rk < nc) {
            float lo = cands[rk].d;
            for (size_t i = rk + 1; i < nc; ++i) if (cands[i].d < lo) lo = cands[i].d;
            const float hi = cands[rk - 1].d, mag = fmaxf(fabsf(hi), fabsf(lo));
            g = mag > 0.0f ? (lo - hi) / mag : lo - hi;
        }
        x->out_gap[q] = g;
    }
    heap_t hp = { scratch, 0, x->k };
    for (size_t i = 0; i < rk; ++i) {
        const uint32_t row = cands[i].row;
        hit_t h = { orc_distance(x->metric, qv, x->vectors + (size_t)row * d, d),
                    x->mode == 0 ? (int64_t)i : (int64_t)row };
        heap_push(&hp, h);
    }
    float* od = x->out_d + q * x->k;
    int64_t* orow = x->out_r + q * x->k;
    heap_emit(&hp, x->k, od, orow);
    if (x->mode == 0)
        for (size_t i = 0; i < x->k; ++i) if (orow[i] >= 0) orow[i] = cands[orow[i]].row;
    free(dec); free(cands); free(lists);
}

/* GpuIVFFlatIndex::search, GpuIVFFlatIndex.cpp:84-103 (search_batch,
 * :123-164, ranks each query the same way): probe_lists -> gather_candidates
 * (probe order, then list member order, IvfIndexState.cpp:466-504) ->
 * rank_candidates (:44-82): elips::distance to every candidate
 * (compute_distances_batch) and top_k, ties by gather position. */
typedef struct {
    int metric; size_t d, nlist, nprobe;
    const float* centroids; const float* vectors;
    const uint32_t* list_offsets; const uint32_t* list_rows;
    const float* queries; size_t k; float* out_d; int64_t* out_r;
} ivfflat_ctx;

static void ivfflat_one(const void* c, size_t q, hit_t* scratch) {
    const ivfflat_ctx* x = (const ivfflat_ctx*)c;
    const float* qv = x->queries + q * x->d;
    uint32_t* lists = (uint32_t*)malloc(sizeof(uint32_t) * x->nprobe);
    orc_ivf_probe(x->metric, qv, x->d, x->centroids, x->nlist, x->nprobe, lists, NULL);
    size_t total = 0;
    for (size_t p = 0; p < x->nprobe; ++p)
        if (lists[p] < x->nlist) total += x->list_offsets[lists[p] + 1] - x->list_offsets[lists[p]];
    uint32_t* rows = (uint32_t*)malloc(sizeof(uint32_t) * (total ? total : 1));
    heap_t hp = { scratch, 0, x->k };
    size_t pos = 0;
    for (size_t p = 0; p < x->nprobe; ++p) {
        const uint32_t l = lists[p];
        if (l >= x->nlist) continue;
        for (uint32_t j = x->list_offsets[l]; j < x->list_offsets[l + 1]; ++j, ++pos) {
            rows[pos] = x->list_rows[j];
            hit_t h = { orc_distance(x->metric, qv, x->vectors + (size_t)rows[pos] * x->d, x->d), (int64_t)pos };
            heap_push(&hp, h);
        }
    }
    float* od = x->out_d + q * x->k;
    int64_t* orow = x->out_r + q * x->k;
    heap_emit(&hp, x->k, od, orow);
    for (size_t i = 0; i < x->k; ++i) if (orow[i] >= 0) orow[i] = rows[orow[i]];
    free(rows); free(lists);
}

void orc_ivfflat_search(int metric, size_t d, size_t nlist, size_t nprobe, const float* centroids,
                        const float* vectors, const uint32_t* list_offsets, const uint32_t* list_rows,
                        const float* queries, size_t nq, size_t k, int nthreads, float* out_d, int64_t* out_r) {
    ivfflat_ctx c = { metric, d, nlist, nprobe, centroids, vectors, list_offsets, list_rows, queries, k,
                      out_d, out_r };
    run_queries(&c, ivfflat_one, nq, nthreads, k);
}

void orc_ivfpq_search(int metric, size_t d, size_t m, size_t ksub, size_t nlist, size_t nprobe,
                      const float* centroids, const float* codebook, const uint8_t* codes,
                      const float* vectors, const uint32_t* list_offsets,
                      const uint32_t* list_rows, const float* queries, size_t nq, size_t k,
                      int mode, int nthreads, float* out_d, int64_t* out_r, float* out_gap) {
    ivfpq_ctx c = { metric, d, m, ksub, nlist, nprobe, centroids, codebook, codes, vectors,
                    list_offsets, list_rows, queries, k, mode, out_d, out_r, out_gap };
    run_queries(&c, ivfpq_one, nq, nthreads, k);
}
