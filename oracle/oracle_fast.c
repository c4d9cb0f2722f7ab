/*
 * oracle_fast.c -- blocked, multi-threaded forms of the exact-search oracle.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.c): the checker the parity tests and
 * bench.py's parity leg compare the CUDA path with; never part of the product.
 *
 * These compute exactly what orc_exact_search / orc_exact_search_masked /
 * orc_int8_ip_search in oracle.c compute, bit for bit, at sizes where those
 * per-pair scalar loops take minutes (2,000,000 x 768 rows, 1,000 queries):
 *
 *  - fp32 metrics (elips::distance, Metrics.cpp:104-115): the sum of every
 *    (query, row) pair is still sequential over the dimensions in single
 *    precision with the product rounded before the add (no FMA), as
 *    dot_scalar / sql2_scalar (Metrics.cpp:20-37) compile to. The vector lanes
 *    hold 16 different QUERIES of one row, never parts of one sum, so every
 *    lane performs the scalar loop's operations in the scalar loop's order.
 *  - int8 inner product: the sum is exact in int32, so its order is free; the
 *    lanes split the dimensions.
 *
 * Results are the k smallest by (distance, row), ascending, like oracle.c.
 * The AVX-512 kernels are selected at run time; hosts without AVX-512 fall
 * back to oracle.c's scalar loops (same results, slower).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <immintrin.h>

enum { F_COSINE = 0, F_EUCLIDEAN = 1, F_DOT = 2 };

void orc_exact_search(int metric, const float* base, size_t n, size_t d, const float* queries,
                      size_t nq, size_t k, int nthreads, float* out_d, int64_t* out_r);
void orc_exact_search_masked(int metric, const float* base, size_t n, size_t d,
                             const uint32_t* mask, const float* queries, size_t nq, size_t k,
                             int nthreads, float* out_d, int64_t* out_r);
void orc_int8_ip_search(const int8_t* base, size_t n, size_t d, const int8_t* queries, size_t nq,
                        size_t k, int nthreads, float* out_d, int64_t* out_r);

/* ------------------------------------------------------------------------ */
/* bounded max-heap of the k smallest (distance, row)                         */
/* ------------------------------------------------------------------------ */

typedef struct { float d; int64_t r; } fhit_t;

static int fless(fhit_t a, fhit_t b) { return a.d < b.d || (a.d == b.d && a.r < b.r); }

typedef struct { fhit_t* h; size_t n, cap; } fheap_t;

/* Pushes x; returns the current bound (the heap's largest) once full, else +inf. */
static float fheap_push(fheap_t* hp, fhit_t x) {
    if (hp->n < hp->cap) {
        size_t i = hp->n++;
        hp->h[i] = x;
        while (i > 0) {
            size_t p = (i - 1) / 2;
            if (!fless(hp->h[p], hp->h[i])) break;
            fhit_t t = hp->h[p]; hp->h[p] = hp->h[i]; hp->h[i] = t;
            i = p;
        }
    } else if (fless(x, hp->h[0])) {
        hp->h[0] = x;
        size_t i = 0;
        for (;;) {
            size_t l = 2 * i + 1, r = l + 1, m = i;
            if (l < hp->n && fless(hp->h[m], hp->h[l])) m = l;
            if (r < hp->n && fless(hp->h[m], hp->h[r])) m = r;
            if (m == i) break;
            fhit_t t = hp->h[m]; hp->h[m] = hp->h[i]; hp->h[i] = t;
            i = m;
        }
    }
    return hp->n == hp->cap ? hp->h[0].d : INFINITY;
}

static int fhit_cmp(const void* a, const void* b) {
    const fhit_t x = *(const fhit_t*)a, y = *(const fhit_t*)b;
    if (fless(x, y)) return -1;
    if (fless(y, x)) return 1;
    return 0;
}

/* ------------------------------------------------------------------------ */
/* shared driver: threads pull row chunks; each thread keeps a heap per      */
/* query; the heaps of all threads are merged per query at the end           */
/* ------------------------------------------------------------------------ */

typedef struct job job_t;
typedef void (*chunk_fn)(const job_t* j, size_t r0, size_t r1, fheap_t* heaps, float* bound, void* tls);

struct job {
    int metric;
    const void* base;     /* float [n][d] or int8 [n][d] */
    size_t n, d, nq, k;
    const void* qprep;    /* query operands in the kernel's layout */
    const uint32_t* rows; /* selected rows (mask), or NULL for 0..n-1 */
    size_t nrows;
    size_t chunk;
    size_t tls_bytes;
    chunk_fn fn;
    size_t next;          /* next chunk index (atomic) */
    int nthreads;
    fhit_t* all;          /* [nthreads][nq][k] */
    size_t* counts;       /* [nthreads][nq] */
};

typedef struct { job_t* j; int t; } targ_t;

static void* fast_worker(void* arg) {
    targ_t* a = (targ_t*)arg;
    job_t* j = a->j;
    fheap_t* heaps = (fheap_t*)malloc(sizeof(fheap_t) * (j->nq ? j->nq : 1));
    float* bound = (float*)aligned_alloc(64, ((j->nq + 15) / 16 * 16) * sizeof(float));
    void* tls = j->tls_bytes ? aligned_alloc(64, (j->tls_bytes + 63) / 64 * 64) : NULL;
    for (size_t q = 0; q < j->nq; ++q) {
        heaps[q].h = j->all + ((size_t)a->t * j->nq + q) * j->k;
        heaps[q].n = 0;
        heaps[q].cap = j->k;
    }
    for (size_t q = 0; q < (j->nq + 15) / 16 * 16; ++q) bound[q] = INFINITY;
    const size_t total = j->rows ? j->nrows : j->n;
    for (;;) {
        const size_t c = __atomic_fetch_add(&j->next, 1, __ATOMIC_RELAXED);
        const size_t r0 = c * j->chunk;
        if (r0 >= total) break;
        const size_t r1 = r0 + j->chunk < total ? r0 + j->chunk : total;
        j->fn(j, r0, r1, heaps, bound, tls);
    }
    for (size_t q = 0; q < j->nq; ++q) j->counts[(size_t)a->t * j->nq + q] = heaps[q].n;
    free(heaps);
    free(bound);
    free(tls);
    return NULL;
}

static void run_job(job_t* j, float* out_d, int64_t* out_r) {
    int nt = j->nthreads < 1 ? 1 : j->nthreads;
    j->nthreads = nt;
    j->next = 0;
    j->all = (fhit_t*)malloc(sizeof(fhit_t) * (size_t)nt * j->nq * j->k + sizeof(fhit_t));
    j->counts = (size_t*)calloc((size_t)nt * j->nq + 1, sizeof(size_t));
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nt);
    targ_t* ta = (targ_t*)malloc(sizeof(targ_t) * nt);
    for (int t = 0; t < nt; ++t) {
        ta[t].j = j;
        ta[t].t = t;
        if (nt == 1) fast_worker(&ta[t]);
        else pthread_create(&th[t], NULL, fast_worker, &ta[t]);
    }
    if (nt > 1) for (int t = 0; t < nt; ++t) pthread_join(th[t], NULL);
    fhit_t* merged = (fhit_t*)malloc(sizeof(fhit_t) * ((size_t)nt * j->k + 1));
    for (size_t q = 0; q < j->nq; ++q) {
        size_t m = 0;
        for (int t = 0; t < nt; ++t) {
            const size_t c = j->counts[(size_t)t * j->nq + q];
            memcpy(merged + m, j->all + ((size_t)t * j->nq + q) * j->k, c * sizeof(fhit_t));
            m += c;
        }
        qsort(merged, m, sizeof(fhit_t), fhit_cmp);
        for (size_t i = 0; i < j->k; ++i) {
            if (i < m) { out_d[q * j->k + i] = merged[i].d; out_r[q * j->k + i] = merged[i].r; }
            else { out_d[q * j->k + i] = 0.0f; out_r[q * j->k + i] = -1; }
        }
    }
    free(merged);
    free(th);
    free(ta);
    free(j->all);
    free(j->counts);
}

/* ------------------------------------------------------------------------ */
/* fp32 metrics: 16 queries per vector, 8 rows per group                      */
/* ------------------------------------------------------------------------ */

/* Queries transposed into blocks of 16: qt[block][dim][16]; lanes past nq are 0. */
static float* transpose_queries(const float* q, size_t nq, size_t d) {
    const size_t nb = (nq + 15) / 16;
    float* qt = (float*)aligned_alloc(64, nb * d * 16 * sizeof(float) + 64);
    memset(qt, 0, nb * d * 16 * sizeof(float));
    for (size_t i = 0; i < nq; ++i)
        for (size_t c = 0; c < d; ++c) qt[((i / 16) * d + c) * 16 + (i % 16)] = q[i * d + c];
    return qt;
}

__attribute__((target("avx512f")))
static void f32_chunk_avx512(const job_t* j, size_t r0, size_t r1, fheap_t* heaps, float* bound, void* tls) {
    (void)tls;
    const float* base = (const float*)j->base;
    const float* qt = (const float*)j->qprep;
    const size_t d = j->d, nb = (j->nq + 15) / 16;
    const __m512 one = _mm512_set1_ps(1.0f);
    const __m512 negz = _mm512_set1_ps(-0.0f);
    for (size_t b = 0; b < nb; ++b) {
        const float* qb = qt + b * d * 16;
        const size_t lanes = j->nq - b * 16 < 16 ? j->nq - b * 16 : 16;
        const __mmask16 live = (__mmask16)((1u << lanes) - 1u);
        for (size_t g = r0; g < r1; g += 8) {
            const size_t cnt = r1 - g < 8 ? r1 - g : 8;
            int64_t row[8];
            const float* x[8];
            for (size_t t = 0; t < 8; ++t) {
                const size_t idx = g + (t < cnt ? t : 0);
                row[t] = j->rows ? (int64_t)j->rows[idx] : (int64_t)idx;
                x[t] = base + (size_t)row[t] * d;
            }
            __m512 acc[8];
            for (int t = 0; t < 8; ++t) acc[t] = _mm512_setzero_ps();
            if (j->metric == F_EUCLIDEAN) {
                for (size_t c = 0; c < d; ++c) {
                    const __m512 qv = _mm512_load_ps(qb + c * 16);
                    for (int t = 0; t < 8; ++t) {
                        const __m512 df = _mm512_sub_ps(qv, _mm512_set1_ps(x[t][c]));
                        acc[t] = _mm512_add_ps(acc[t], _mm512_mul_ps(df, df));
                    }
                }
            } else {
                for (size_t c = 0; c < d; ++c) {
                    const __m512 qv = _mm512_load_ps(qb + c * 16);
                    for (int t = 0; t < 8; ++t)
                        acc[t] = _mm512_add_ps(acc[t], _mm512_mul_ps(qv, _mm512_set1_ps(x[t][c])));
                }
            }
            const __m512 bnd = _mm512_load_ps(bound + b * 16);
            for (size_t t = 0; t < cnt; ++t) {
                __m512 dist;
                if (j->metric == F_COSINE) dist = _mm512_sub_ps(one, acc[t]);
                else if (j->metric == F_DOT)
                    dist = _mm512_castsi512_ps(_mm512_xor_si512(_mm512_castps_si512(acc[t]), _mm512_castps_si512(negz)));
                else dist = _mm512_sqrt_ps(acc[t]);
                __mmask16 hit = _mm512_mask_cmp_ps_mask(live, dist, bnd, _CMP_LE_OQ);
                if (!hit) continue;
                float dv[16];
                _mm512_storeu_ps(dv, dist);
                while (hit) {
                    const int l = __builtin_ctz(hit);
                    hit &= (__mmask16)(hit - 1);
                    const size_t q = b * 16 + (size_t)l;
                    fhit_t h = { dv[l], row[t] };
                    bound[q] = fheap_push(&heaps[q], h);
                }
                /* later rows of this group compare with the looser bound
                   loaded before it; the heap's own test stays exact */
            }
        }
    }
}

static int have_avx512(void) {
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw");
}

static uint32_t* mask_rows(const uint32_t* mask, size_t n, size_t* count) {
    size_t c = 0;
    for (size_t i = 0; i < n; ++i) c += (mask[i >> 5] >> (i & 31)) & 1u;
    uint32_t* rows = (uint32_t*)malloc(sizeof(uint32_t) * (c + 1));
    c = 0;
    for (size_t i = 0; i < n; ++i)
        if ((mask[i >> 5] >> (i & 31)) & 1u) rows[c++] = (uint32_t)i;
    *count = c;
    return rows;
}

/* Same results as orc_exact_search (mask == NULL) or orc_exact_search_masked.
 * Returns 1 when the AVX-512 path ran, 0 when the scalar fallback did. */
int orc_exact_search_fast(int metric, const float* base, size_t n, size_t d, const uint32_t* mask,
                          const float* queries, size_t nq, size_t k, int nthreads, float* out_d,
                          int64_t* out_r) {
    if (nq == 0 || k == 0) return 1;
    if (!have_avx512()) {
        if (mask) orc_exact_search_masked(metric, base, n, d, mask, queries, nq, k, nthreads, out_d, out_r);
        else orc_exact_search(metric, base, n, d, queries, nq, k, nthreads, out_d, out_r);
        return 0;
    }
    job_t j;
    memset(&j, 0, sizeof(j));
    j.metric = metric;
    j.base = base;
    j.n = n;
    j.d = d;
    j.nq = nq;
    j.k = k;
    float* qt = transpose_queries(queries, nq, d);
    j.qprep = qt;
    uint32_t* rows = NULL;
    if (mask) {
        rows = mask_rows(mask, n, &j.nrows);
        j.rows = rows;
    }
    /* ~512 KB of rows per chunk (stays in L2 across the query blocks) */
    size_t chunk = (512u << 10) / (d * sizeof(float));
    chunk = chunk < 8 ? 8 : chunk / 8 * 8;
    j.chunk = chunk;
    j.fn = f32_chunk_avx512;
    j.nthreads = nthreads;
    run_job(&j, out_d, out_r);
    free(qt);
    free(rows);
    return 1;
}

/* ------------------------------------------------------------------------ */
/* int8 inner product: exact int32 sums, lanes across dimensions             */
/* ------------------------------------------------------------------------ */

/* Queries widened to int16, dimension padded to a multiple of 32 with zeros. */
static int16_t* widen_queries(const int8_t* q, size_t nq, size_t d, size_t dp) {
    int16_t* w = (int16_t*)aligned_alloc(64, nq * dp * sizeof(int16_t) + 64);
    memset(w, 0, nq * dp * sizeof(int16_t));
    for (size_t i = 0; i < nq; ++i)
        for (size_t c = 0; c < d; ++c) w[i * dp + c] = q[i * d + c];
    return w;
}

__attribute__((target("avx512f,avx512bw")))
static void i8_chunk_avx512(const job_t* j, size_t r0, size_t r1, fheap_t* heaps, float* bound, void* tls) {
    const int8_t* base = (const int8_t*)j->base;
    const int16_t* qw = (const int16_t*)j->qprep;
    const size_t d = j->d, dp = (d + 31) / 32 * 32, nv = dp / 32;
    int16_t* rw = (int16_t*)tls; /* [chunk][dp] rows widened to int16 */
    const size_t cnt = r1 - r0;
    for (size_t t = 0; t < cnt; ++t) {
        const int8_t* x = base + (r0 + t) * d;
        int16_t* o = rw + t * dp;
        size_t c = 0;
        for (; c + 32 <= d; c += 32)
            _mm512_store_si512((void*)(o + c), _mm512_cvtepi8_epi16(_mm256_loadu_si256((const void*)(x + c))));
        for (; c < dp; ++c) o[c] = c < d ? x[c] : 0;
    }
    /* 16 queries x 4 rows per step: 4 independent accumulators per query */
    for (size_t q0 = 0; q0 < j->nq; q0 += 16) {
        const size_t qn = j->nq - q0 < 16 ? j->nq - q0 : 16;
        for (size_t t = 0; t < cnt; t += 4) {
            const size_t tn = cnt - t < 4 ? cnt - t : 4;
            int32_t sc[4][16];
            for (size_t qi = 0; qi < qn; ++qi) {
                const int16_t* qv = qw + (q0 + qi) * dp;
                __m512i a0 = _mm512_setzero_si512(), a1 = a0, a2 = a0, a3 = a0;
                const int16_t* x0 = rw + (t + 0) * dp;
                const int16_t* x1 = rw + (t + (tn > 1 ? 1 : 0)) * dp;
                const int16_t* x2 = rw + (t + (tn > 2 ? 2 : 0)) * dp;
                const int16_t* x3 = rw + (t + (tn > 3 ? 3 : 0)) * dp;
                for (size_t v = 0; v < nv; ++v) {
                    const __m512i qq = _mm512_load_si512((const void*)(qv + v * 32));
                    a0 = _mm512_add_epi32(a0, _mm512_madd_epi16(qq, _mm512_load_si512((const void*)(x0 + v * 32))));
                    a1 = _mm512_add_epi32(a1, _mm512_madd_epi16(qq, _mm512_load_si512((const void*)(x1 + v * 32))));
                    a2 = _mm512_add_epi32(a2, _mm512_madd_epi16(qq, _mm512_load_si512((const void*)(x2 + v * 32))));
                    a3 = _mm512_add_epi32(a3, _mm512_madd_epi16(qq, _mm512_load_si512((const void*)(x3 + v * 32))));
                }
                sc[0][qi] = _mm512_reduce_add_epi32(a0);
                sc[1][qi] = _mm512_reduce_add_epi32(a1);
                sc[2][qi] = _mm512_reduce_add_epi32(a2);
                sc[3][qi] = _mm512_reduce_add_epi32(a3);
            }
            for (size_t u = 0; u < tn; ++u) {
                const int64_t row = (int64_t)(r0 + t + u);
                for (size_t qi = 0; qi < qn; ++qi) {
                    const float dist = -(float)sc[u][qi];
                    const size_t q = q0 + qi;
                    if (dist <= bound[q]) {
                        fhit_t h = { dist, row };
                        bound[q] = fheap_push(&heaps[q], h);
                    }
                }
            }
        }
    }
}

/* Same results as orc_int8_ip_search. Returns 1 when the AVX-512 path ran. */
int orc_int8_ip_search_fast(const int8_t* base, size_t n, size_t d, const int8_t* queries, size_t nq,
                            size_t k, int nthreads, float* out_d, int64_t* out_r) {
    if (nq == 0 || k == 0) return 1;
    if (!have_avx512()) {
        orc_int8_ip_search(base, n, d, queries, nq, k, nthreads, out_d, out_r);
        return 0;
    }
    const size_t dp = (d + 31) / 32 * 32;
    job_t j;
    memset(&j, 0, sizeof(j));
    j.metric = F_DOT;
    j.base = base;
    j.n = n;
    j.d = d;
    j.nq = nq;
    j.k = k;
    int16_t* qw = widen_queries(queries, nq, d, dp);
    j.qprep = qw;
    size_t chunk = (256u << 10) / (dp * sizeof(int16_t));
    chunk = chunk < 4 ? 4 : chunk / 4 * 4;
    j.chunk = chunk;
    j.tls_bytes = chunk * dp * sizeof(int16_t);
    j.fn = i8_chunk_avx512;
    j.nthreads = nthreads;
    run_job(&j, out_d, out_r);
    free(qw);
    return 1;
}
