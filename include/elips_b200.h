/*
 * elips_b200.h -- C ABI of the B200 k-NN search backend for ELIPS.
 *
 * Plain C types only: no C++ exceptions, no torch types, no CUDA headers.
 * Every function returns an int status (ELIPS_B200_OK = 0). Streams are
 * passed as `void*` holding a cudaStream_t (NULL = the legacy default stream).
 *
 * Each entry point names the reference interface it replaces (paths relative
 * to the axiomchronicles/elips source tree).
 */
#ifndef ELIPS_B200_H
#define ELIPS_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ELIPS_B200_API __attribute__((visibility("default")))
#else
#define ELIPS_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. 1..8 are elips::gpu::GpuError (include/elips/gpu_engine/
 * GpuPort.hpp:15-24) as (int)GpuError + 1, so a CudaBackend maps them 1:1. */
enum {
    ELIPS_B200_OK = 0,
    ELIPS_B200_DEVICE_NOT_FOUND = 1,
    ELIPS_B200_INSUFFICIENT_MEMORY = 2,
    ELIPS_B200_KERNEL_LAUNCH_FAILED = 3,
    ELIPS_B200_TRANSFER_FAILED = 4,
    ELIPS_B200_INDEX_BUILD_FAILED = 5,
    ELIPS_B200_UNSUPPORTED_METRIC = 6,
    ELIPS_B200_INITIALIZATION_FAILED = 7,
    ELIPS_B200_BACKEND_UNAVAILABLE = 8,
    /* IndexPort::search throws DimensionMismatch on a bad query width
     * (src/ExactIndex.cpp:14-20); across a C ABI that becomes this code. */
    ELIPS_B200_DIMENSION_MISMATCH = 9,
    ELIPS_B200_INVALID_ARGUMENT = 10,
    /* A bounded device-side wait expired; the kernel returned early. */
    ELIPS_B200_DEVICE_TIMEOUT = 11
};

/* elips::Metric (include/elips/Config.hpp:27). Distances are the reference's
 * ordering-normalised ones (src/Metrics.cpp:104-115): cosine = 1 - dot,
 * euclidean = sqrt(sum (a-b)^2), dot_product = -dot; smaller is closer. */
enum {
    ELIPS_B200_METRIC_COSINE = 0,
    ELIPS_B200_METRIC_EUCLIDEAN = 1,
    ELIPS_B200_METRIC_DOT_PRODUCT = 2
};

/* elips::gpu::GpuPrecision (include/elips/gpu_engine/GpuConfig.hpp:34) with
 * BF16 appended. FP32 runs as 3xTF32 on the tensor cores; INT8 is the
 * symmetric int8 codec (rows and queries are int8, score = -sum q_i*x_i in
 * exact int32, dot_product metric only). */
enum {
    ELIPS_B200_PRECISION_FP32 = 0,
    ELIPS_B200_PRECISION_FP16 = 1,
    ELIPS_B200_PRECISION_INT8 = 2,
    ELIPS_B200_PRECISION_AUTO = 3,
    ELIPS_B200_PRECISION_BF16 = 4
};

/* ------------------------------------------------------------- utilities */

/* Human-readable name of a status code (static storage). */
ELIPS_B200_API const char* elips_b200_status_string(int status);

/* Number of CUDA devices visible (GpuDeviceManager::probe_all_devices,
 * src/gpu_engine/GpuDeviceManager.cpp:68-132). */
ELIPS_B200_API int elips_b200_device_count(int* count_out);

/* Reads and clears the device-side error word of `device` that bounded waits
 * write on timeout (0 = none). Synchronises the device. */
ELIPS_B200_API int elips_b200_device_error(int device, int* code_out);

/* Self-test of the bounded device waits; no counterpart in the reference.
 * One thread waits on an mbarrier that nothing arrives on, for `cycles`
 * clock cycles (1 .. 2^31); the wait expires, records the device error word
 * and raises its abort flag, as any pipeline wait does when a producer or
 * consumer is lost. Returns ELIPS_B200_DEVICE_TIMEOUT when the expiry was
 * reported (the expected outcome; the error word is cleared again and the
 * context stays usable), ELIPS_B200_OK if the wait completed. */
ELIPS_B200_API int elips_b200_wait_selftest(int device, uint64_t cycles);

/* ------------------------------------------------ exact brute-force index */
/* Replaces ExactIndex (include/elips/index_engine/ExactIndex.hpp:26-66) and
 * GpuBruteForceIndex (src/gpu_engine/GpuBruteForceIndex.cpp:77-170): a
 * device-resident base set searched by the fused tensor-core kernel. */

typedef struct elips_b200_exact elips_b200_exact;

/* GpuBruteForceIndex(backend, metric, dimension, config) with
 * config.search_precision = precision. */
ELIPS_B200_API int elips_b200_exact_create(int device, int metric, int precision, uint32_t dimension,
                            elips_b200_exact** out);

/* IndexPort::insert for n rows at once (ExactIndex.cpp:24-35; row i of the
 * call gets the next slot). rows: HOST memory, n x dimension, fp32 (int8 for
 * PRECISION_INT8). */
ELIPS_B200_API int elips_b200_exact_add(elips_b200_exact* index, const void* rows, size_t n);

/* Same as elips_b200_exact_add with rows in DEVICE memory; returns after the
 * rows are converted (work queued on `stream` completes first). */
ELIPS_B200_API int elips_b200_exact_add_device(elips_b200_exact* index, const void* rows, size_t n,
                                               void* stream);

/* IndexPort::size. */
ELIPS_B200_API int elips_b200_exact_size(const elips_b200_exact* index, size_t* n_out);

/* Rows not removed (elips_b200_exact_size counts every row ever added: the
 * row-number space results are reported in). */
ELIPS_B200_API int elips_b200_exact_live(const elips_b200_exact* index, size_t* n_out);

/* GpuIndexPort::device_bytes_used (GpuIndexPort.hpp:42): device memory the
 * index holds (operand rows at capacity, norms, removal bits). */
ELIPS_B200_API int elips_b200_exact_device_bytes(const elips_b200_exact* index, size_t* bytes_out);

/* Incremental removal on the device, in place of GpuBruteForceIndex::remove's
 * full re-upload (src/gpu_engine/GpuBruteForceIndex.cpp:84-99): the row keeps
 * its number but no search returns it again (a removal bit folded into the
 * eligibility mask); the other rows keep their numbers and relative order, so
 * equal distances still rank as the reference's erase-based order ranks them.
 * removed_out (may be NULL) is 0 when the row was already removed. Not
 * concurrent with searches (the reference removes under Vault's unique lock). */
ELIPS_B200_API int elips_b200_exact_remove(elips_b200_exact* index, size_t row, int* removed_out);

/* Drops the removed rows on the device, keeping the order of the others.
 * new_to_old (may be NULL; `capacity` entries, at least the live count)
 * receives each kept row's former number, so the caller can renumber its ids. */
ELIPS_B200_API int elips_b200_exact_compact(elips_b200_exact* index, uint32_t* new_to_old, size_t capacity);

/* Device snapshot (IndexSnapshot, include/elips/index_engine/IndexSnapshot.hpp:
 * 26-56, without the ids the caller keeps): the stored operand rows, norms and
 * removal bits as one host blob, reloaded into an empty index of the same
 * metric, precision and dimension without converting the rows again. */
ELIPS_B200_API int elips_b200_exact_snapshot_bytes(const elips_b200_exact* index, size_t* bytes_out);
ELIPS_B200_API int elips_b200_exact_export(const elips_b200_exact* index, void* out, size_t bytes);
ELIPS_B200_API int elips_b200_exact_import(elips_b200_exact* index, const void* blob, size_t bytes);

ELIPS_B200_API int elips_b200_exact_destroy(elips_b200_exact* index);

/* GpuIndexPort::search_batch (GpuIndexPort.hpp:120-124) / ExactIndex::search
 * (ExactIndex.cpp:55-87) for nq queries. HOST pointers; synchronous.
 * queries: nq x dimension fp32 (int8 for PRECISION_INT8). mask: optional
 * eligibility bitmask over slots (bit i&31 of word i>>5), the dense form of
 * MetadataIndex::exact_candidates (src/MetadataIndex.cpp:66-99), or NULL.
 * Output nq x k, ascending by (distance, slot); slots past the number of
 * eligible rows hold distance +inf and slot -1. */
ELIPS_B200_API int elips_b200_exact_search(const elips_b200_exact* index, const void* queries, size_t nq,
                            size_t k, const uint32_t* mask, float* out_dist, int64_t* out_rows);

/* Same search with DEVICE pointers, asynchronous on `stream`. */
ELIPS_B200_API int elips_b200_exact_search_device(const elips_b200_exact* index, const void* queries,
                                   size_t nq, size_t k, const uint32_t* mask, float* out_dist,
                                   int64_t* out_rows, void* stream);

/* Exact search that allocates no device memory. It has no counterpart in
 * the reference: it exists for callers that cannot call cudaMalloc at search
 * time -- a process whose device memory is already fully reserved by another
 * allocator, or a latency-critical path where an allocation may synchronise
 * the device. Same arguments and results as elips_b200_exact_search_device
 * (DEVICE pointers, asynchronous on `stream`, no row offset). Scratch comes
 * from one fixed 64 MiB device array inside this library, which every GPU that
 * loads the library holds until the process exits; a call needing more (large
 * query batches) fails with ELIPS_B200_INVALID_ARGUMENT, and at most 32 SMs
 * are used. The first call on a device looks up the array's address; under
 * CUDA's default lazy module loading that lookup is also what loads this
 * library's module on the device and so reserves the 64 MiB (a call with
 * nq = 0 does only this). Make that first call at set-up, while device memory
 * is still free and before any stream capture, or run the process with
 * CUDA_MODULE_LOADING=EAGER so the array is reserved when the library loads.
 * All calls
 * share the array and it keeps the last call's contents: calls that overlap
 * on the GPU (different streams, or unordered host threads) race, so the
 * caller must serialise them. */
ELIPS_B200_API int elips_b200_exact_search_noalloc(const elips_b200_exact* index, const void* queries,
                                                   size_t nq, size_t k, const uint32_t* mask,
                                                   float* out_dist, int64_t* out_rows, void* stream);

/* Shard-level search for row-sharded multi-GPU search
 * (GpuDistributedIndex::search_batch, src/gpu_engine/GpuDistributedIndex.cpp:
 * 155-207): DEVICE pointers; writes nq x k candidates as pairs of uint32
 * {ordering key bits, row_offset + slot} to out_cand (2*nq*k words), unsorted,
 * padded with {+inf, 0xFFFFFFFF}. The key is the distance before the final
 * square root for euclidean. */
ELIPS_B200_API int elips_b200_exact_search_candidates_device(const elips_b200_exact* index,
                                              const void* queries, size_t nq, size_t k,
                                              const uint32_t* mask, uint32_t row_offset,
                                              uint32_t* out_cand, void* stream);

/* The shard-level search above with the per-query admission bounds shared
 * by every shard searching the same queries: shared_bound (DEVICE, nq
 * uint32 ordered keys, may be another GPU's memory mapped with
 * elips_b200_peer_open) is read and tightened (atomicMin) by the kernel while
 * it runs, so each shard admits only candidates that can still reach the
 * global top-k. The caller sets it to all ones (0xFF bytes) before the
 * shards' searches and not again until all of them have finished. The merged
 * result over all shards equals the one with private bounds. */
ELIPS_B200_API int elips_b200_exact_search_candidates_shared_device(const elips_b200_exact* index,
                                                                    const void* queries, size_t nq, size_t k,
                                                                    const uint32_t* mask, uint32_t row_offset,
                                                                    uint32_t* out_cand, uint32_t* shared_bound,
                                                                    void* stream);

/* Device buffers shared between the processes of one node (one per GPU) for
 * the shard exchange: elips_b200_peer_alloc allocates `bytes` on `device` and
 * writes its 64-byte interprocess handle; another process maps it into its
 * own device's address space with elips_b200_peer_open (reads, writes and
 * atomics then travel over NVLink) and unmaps it with elips_b200_peer_close;
 * the owner frees it with elips_b200_peer_free. */
ELIPS_B200_API int elips_b200_peer_alloc(int device, size_t bytes, void** ptr_out, void* ipc_handle_out);
ELIPS_B200_API int elips_b200_peer_open(int device, const void* ipc_handle, void** ptr_out);
ELIPS_B200_API int elips_b200_peer_close(int device, void* ptr);
ELIPS_B200_API int elips_b200_peer_free(int device, void* ptr);
/* Stream-ordered copy between device buffers (this GPU's or a mapped peer's)
 * and byte fill of a device buffer. */
ELIPS_B200_API int elips_b200_copy_device(int device, void* dst, const void* src, size_t bytes, void* stream);
ELIPS_B200_API int elips_b200_fill_device(int device, void* dst, int byte_value, size_t bytes, void* stream);

/* Final top-k over candidate lists (GpuDistributedIndex::merge_hits,
 * src/gpu_engine/GpuDistributedIndex.cpp:68-83): cand holds `lists` blocks of
 * nq x k pairs as written above, block-major (block l = one shard's output for
 * every query, e.g. an all-gather over `lists` ranks); 2*lists*nq*k words,
 * DEVICE. Writes the k best per query ascending by (distance, row), applying
 * the metric's final transform (square root for euclidean). */
ELIPS_B200_API int elips_b200_merge_candidates_device(int device, const uint32_t* cand, size_t nq,
                                       size_t lists, size_t k, int metric, float* out_dist,
                                       int64_t* out_rows, void* stream);

/* ------------------------------------------------- GpuPort primitives */
/* GpuPort::compute_distances_batch (include/elips/gpu_engine/GpuPort.hpp:
 * 65-73): distances_out[q * nb + i] = elips::distance(metric, queries[q],
 * database[i]) with the reference's arithmetic bit for bit (sequential fp32,
 * no fused multiply-add, src/Metrics.cpp:20-37,104-115). Row-major fp32
 * inputs. pointers_on_device = 0: HOST pointers, synchronous (copies in and
 * out, as a GpuPort must accept host spans); 1: DEVICE pointers, asynchronous
 * on `stream`. */
ELIPS_B200_API int elips_b200_compute_distances_batch(int device, const float* queries,
                                                      const float* database, float* distances_out,
                                                      size_t nq, size_t nb, size_t dim, int metric,
                                                      int pointers_on_device, void* stream);

/* CudaBackend::gemm_fp32 (src/gpu_engine/backends/cuda/CudaBackend.hpp:42):
 * row-major C[m][n] = op(A) op(B), op(A) m x k_inner (A stored k_inner x m
 * when trans_a), op(B) k_inner x n (B stored n x k_inner when trans_b), fp32
 * with fused multiply-add. Not on the search path (no reference class calls
 * it); a plain SIMT kernel. Pointers as elips_b200_compute_distances_batch. */
ELIPS_B200_API int elips_b200_gemm_fp32(int device, const float* a, const float* b, float* c, size_t m, size_t n,
                                        size_t k_inner, int trans_a, int trans_b, int pointers_on_device,
                                        void* stream);

/* GpuPort::top_k (GpuPort.hpp:75-82): per row of an nq x nb distance matrix,
 * the k smallest values ascending with their column indexes (ties by index);
 * slots past nb hold index 0xFFFFFFFF and +inf. Pointer modes as above. */
ELIPS_B200_API int elips_b200_top_k(int device, const float* distances, uint32_t* indices_out,
                                    float* values_out, size_t nq, size_t nb, size_t k,
                                    int pointers_on_device, void* stream);

/* Vector::normalized (include/elips/domain/Vector.hpp:25-44) of n rows of
 * width d, as Vault::prepare applies it to cosine vaults on insert and query
 * (src/Database.cpp:823-832): magnitude = sqrt(sequential sum of v*v), every
 * value divided by it, zero rows unchanged; bit-identical. in == out is
 * allowed. HOST pointers (synchronous) or DEVICE pointers on `stream`. */
ELIPS_B200_API int elips_b200_normalize_rows(int device, const float* in, float* out, size_t n, size_t d,
                                             int pointers_on_device, void* stream);

/* ---------------------------------------------- quantized exhaustive index */
/* ExactIndex with a trained Quantizer attached (include/elips/index_engine/
 * ExactIndex.hpp:26-66, search at src/ExactIndex.cpp:62-71): codes resident
 * on the device, each query's lookup table built with make_lut and every row
 * scored with lut_distance, bit for bit (ProductQuantizer.cpp:118-183,
 * ScalarQuantizer.cpp:83-128). Codec ids are quant::CodecId
 * (include/elips/quant_engine/QuantParams.hpp:19-26). */
enum {
    ELIPS_B200_CODEC_PQ = 1,
    ELIPS_B200_CODEC_OPQ = 2,
    ELIPS_B200_CODEC_SQ8 = 3
};

typedef struct elips_b200_quant elips_b200_quant;

/* params: PQ/OPQ codebook [pq_dim][2^pq_bits][dimension/pq_dim] (subspace-
 * major, ProductQuantizer.hpp:102-104); SQ8 mins[dimension] followed by
 * scales[dimension]. rotation: OPQ only, dimension x dimension row-major
 * (NULL for PQ and SQ8). HOST pointers, copied. */
ELIPS_B200_API int elips_b200_quant_create(int device, int codec, int metric, uint32_t dimension,
                                           uint32_t pq_dim, uint32_t pq_bits, const float* params,
                                           const float* rotation, elips_b200_quant** out);

/* IndexPort::insert for n fp32 rows (HOST), encoded on the device exactly as
 * Quantizer::encode does (ScalarQuantizer.cpp:52-68; ProductQuantizer.cpp:
 * 71-86 with KMeans.cpp:166-180). */
ELIPS_B200_API int elips_b200_quant_add(elips_b200_quant* index, const float* rows, size_t n);

/* Appends n rows given as codes (HOST, n x code_bytes). */
ELIPS_B200_API int elips_b200_quant_add_codes(elips_b200_quant* index, const uint8_t* codes, size_t n);

ELIPS_B200_API int elips_b200_quant_size(const elips_b200_quant* index, size_t* n_out);

/* ExactIndex::search over the codes: HOST pointers, synchronous; results as
 * elips_b200_exact_search (ascending by (distance, slot)). */
ELIPS_B200_API int elips_b200_quant_search(const elips_b200_quant* index, const float* queries,
                                           size_t nq, size_t k, float* out_dist, int64_t* out_rows);

/* Same with DEVICE pointers, asynchronous on `stream`. */
ELIPS_B200_API int elips_b200_quant_search_device(const elips_b200_quant* index, const float* queries,
                                                  size_t nq, size_t k, float* out_dist,
                                                  int64_t* out_rows, void* stream);

ELIPS_B200_API int elips_b200_quant_destroy(elips_b200_quant* index);

/* ---------------------------------------------------------------- IVF-PQ */
/* GpuIVFPQIndex (src/gpu_engine/GpuIVFPQIndex.cpp): residual product
 * quantization over an inverted-file coarse quantizer. Search = probe the
 * nprobe nearest lists with exact distances (IvfIndexState.cpp:395-423),
 * score their members approximately from the residual codes, rerank the best
 * R = max(4k, k) with exact distances on the raw vectors (GpuIVFPQIndex.cpp:
 * 161-237). The model is imported as GpuIVFPQIndex::import_snapshot does
 * (:327-348): centroids [n_lists][dimension] and the residual codebook
 * [pq_dim][2^pq_bits][dimension/pq_dim] (HOST, copied); nprobe plays
 * GpuConfig::default_ef_search_gpu (IvfIndexState.cpp:45). */
typedef struct elips_b200_ivfpq elips_b200_ivfpq;

ELIPS_B200_API int elips_b200_ivfpq_create(int device, int metric, uint32_t dimension,
                                           uint32_t n_lists, uint32_t nprobe, uint32_t pq_dim,
                                           uint32_t pq_bits, const float* centroids,
                                           const float* codebook, elips_b200_ivfpq** out);

/* Appends n rows: raw vectors (n x dimension fp32, kept for the exact
 * rerank), their list assignments (IvfSnapshot::assignments) and optionally
 * their residual codes (n x pq_dim, IndexSnapshot::pq->codes); with codes =
 * NULL the residuals x - centroid are encoded on the device exactly as
 * GpuIVFPQIndex::rebuild_codes does (:88-130). HOST pointers. */
ELIPS_B200_API int elips_b200_ivfpq_add(elips_b200_ivfpq* index, const float* vectors,
                                        const uint32_t* assignments, const uint8_t* codes, size_t n);

/* Same with DEVICE pointers, ordered on `stream`. */
ELIPS_B200_API int elips_b200_ivfpq_add_device(elips_b200_ivfpq* index, const float* vectors,
                                               const uint32_t* assignments, const uint8_t* codes,
                                               size_t n, void* stream);

ELIPS_B200_API int elips_b200_ivfpq_size(const elips_b200_ivfpq* index, size_t* n_out);

/* Number of lists probed per query (GpuConfig::default_ef_search_gpu). */
ELIPS_B200_API int elips_b200_ivfpq_set_nprobe(elips_b200_ivfpq* index, uint32_t nprobe);

/* GpuIndexPort::search_batch: HOST pointers, synchronous; k <= 256. Results
 * ascending by (exact distance, slot), padded with (+inf, -1). */
ELIPS_B200_API int elips_b200_ivfpq_search(elips_b200_ivfpq* index, const float* queries, size_t nq,
                                           size_t k, float* out_dist, int64_t* out_rows);

/* Same with DEVICE pointers, asynchronous on `stream`. */
ELIPS_B200_API int elips_b200_ivfpq_search_device(elips_b200_ivfpq* index, const float* queries,
                                                  size_t nq, size_t k, float* out_dist,
                                                  int64_t* out_rows, void* stream);

/* Copies the residual codes of every row, slot order (n x pq_dim), to DEVICE
 * memory: the `pq.codes` of GpuIVFPQIndex::export_snapshot (:312-325). */
ELIPS_B200_API int elips_b200_ivfpq_codes_device(const elips_b200_ivfpq* index, uint8_t* codes_out,
                                                 void* stream);

/* List-sharded IVF-PQ over several GPUs (GpuDistributedIndex's shard mode,
 * src/gpu_engine/GpuDistributedIndex.cpp:12-34, applied to IVF lists): this
 * index owns lists [list_lo, list_hi) only; rows may only name them, and a
 * search scans only them. Set before adding rows. */
ELIPS_B200_API int elips_b200_ivfpq_set_list_range(elips_b200_ivfpq* index, uint32_t list_lo,
                                                   uint32_t list_hi);

/* The same with any set of lists: bit (l & 31) of mask_words[l >> 5] set =
 * list l owned; n_words = ceil(n_lists / 32), HOST, copied. */
ELIPS_B200_API int elips_b200_ivfpq_set_owned_lists(elips_b200_ivfpq* index, const uint32_t* mask_words,
                                                    size_t n_words);

/* The approximate stage of search (probe, scan, merge): the R = 4k best
 * {approximate distance bits, slot} per query over the owned probed lists,
 * ascending by (distance, slot), padded with {+inf, 0xFFFFFFFF}; out_cand is
 * nq x R pairs of uint32 (2*nq*R words). DEVICE pointers on `stream`. */
ELIPS_B200_API int elips_b200_ivfpq_search_candidates_device(elips_b200_ivfpq* index,
                                                             const float* queries, size_t nq,
                                                             size_t k, uint32_t* out_cand,
                                                             void* stream);

/* The probe alone (IvfIndexState::probe_lists, IvfIndexState.cpp:395-464):
 * the min(nprobe, n_lists) nearest lists of each query, ascending, ties by
 * list id; probes_out [nq][nprobe] DEVICE. With
 * elips_b200_ivfpq_search_candidates_probed_device the probe of a large batch
 * can be split across GPUs that hold the same centroids: each probes a slice,
 * the slices are exchanged, every GPU scans its own lists with the full
 * probe table (results equal elips_b200_ivfpq_search_candidates_device). */
ELIPS_B200_API int elips_b200_ivfpq_probe_device(const elips_b200_ivfpq* index, const float* queries,
                                                 size_t nq, uint32_t* probes_out, void* stream);
ELIPS_B200_API int elips_b200_ivfpq_search_candidates_probed_device(elips_b200_ivfpq* index,
                                                                    const float* queries, size_t nq,
                                                                    size_t k, const uint32_t* probes,
                                                                    uint32_t* out_cand, void* stream);

/* elips_b200_ivfpq_search_candidates_probed_device (probes may be NULL: this
 * index probes) with the per-query admission bounds in `shared_bound`
 * ([nq] uint32 ordered keys, all 0xFF before the first shard of a batch
 * starts; DEVICE memory of this GPU or of a peer GPU mapped here) instead of
 * the search's own: shards of one list-sharded index searching the same
 * batch at the same time tighten each other's bounds with atomicMin. A bound
 * any shard publishes is the R-th key of R of its candidates, so it is at or
 * above the R-th key of the whole index and admission keeps keys equal to
 * it: every shard's candidates among the index's R best are kept, and the
 * merged result is the one an unshared search gives. The buffer is not
 * reset here. */
ELIPS_B200_API int elips_b200_ivfpq_search_candidates_shared_device(elips_b200_ivfpq* index,
                                                                     const float* queries, size_t nq,
                                                                     size_t k, const uint32_t* probes,
                                                                     uint32_t* out_cand,
                                                                     uint32_t* shared_bound, void* stream);

/* The exact stage (exact_rank, GpuIVFPQIndex.cpp:37-71): for nq x R pairs
 * {any, slot} (slot 0xFFFFFFFF or past size = none), exact distances on this
 * index's raw rows, the k best ascending by (distance, slot). DEVICE. */
ELIPS_B200_API int elips_b200_ivfpq_rerank_device(elips_b200_ivfpq* index, const float* queries,
                                                  size_t nq, size_t k, const uint32_t* cand,
                                                  float* out_dist, int64_t* out_rows, void* stream);

/* Snapshot readback (IndexSnapshot, IndexSnapshot.hpp:26-56): centroids
 * [n_lists][dim], assignments [n], vectors [n][dim], codebook
 * [pq_dim][ksub][dim/pq_dim] and codes [n][pq_dim], all in slot order into host
 * memory (any output may be NULL). elips_b200_ivfpq_create + _add with these
 * rebuilds the same index (GpuIVFPQIndex::import_snapshot, GpuIVFPQIndex.cpp:
 * 327-348, takes the codes as given). */
ELIPS_B200_API int elips_b200_ivfpq_export(const elips_b200_ivfpq* index, float* centroids_out,
                                           uint32_t* assignments_out, float* vectors_out,
                                           float* codebook_out, uint8_t* codes_out);

/* IvfIndexState::remove (src/gpu_engine/detail/IvfIndexState.cpp:262-326) on
 * the device: the slot leaves its list and, unless it is the last slot, the
 * last slot's row moves into it (keeping its place in its list); no
 * re-upload. The reference then runs rebuild_codes
 * (GpuIVFPQIndex.cpp:156-159): call elips_b200_ivfpq_rebuild_codes, which
 * retrains the codebook on every residual (10 rounds) and re-encodes every
 * row, bit-identical to the CPU code (also after an insert: assign with
 * elips_b200_ivf_assign, add, rebuild). Not concurrent with searches. */
ELIPS_B200_API int elips_b200_ivfpq_remove(elips_b200_ivfpq* index, size_t slot);
ELIPS_B200_API int elips_b200_ivfpq_rebuild_codes(elips_b200_ivfpq* index);

ELIPS_B200_API int elips_b200_ivfpq_destroy(elips_b200_ivfpq* index);

/* -------------------------------------------------------------- IVF-Flat */
/* GpuIVFFlatIndex (src/gpu_engine/GpuIVFFlatIndex.cpp): the same inverted
 * file, candidates ranked exactly. search / search_batch (:84-103,
 * :123-164) = probe the nprobe nearest lists (IvfIndexState.cpp:395-423),
 * gather their members in probe order then member order (:466-504), exact
 * elips::distance to each and the k best, ties by gather position
 * (rank_candidates, GpuIVFFlatIndex.cpp:44-82). Centroids
 * [n_lists][dimension] HOST, copied (import_snapshot, :202-205). */
typedef struct elips_b200_ivfflat elips_b200_ivfflat;

ELIPS_B200_API int elips_b200_ivfflat_create(int device, int metric, uint32_t dimension,
                                             uint32_t n_lists, uint32_t nprobe,
                                             const float* centroids, elips_b200_ivfflat** out);

/* Appends n rows with their list ids (HOST pointers, synchronous). Slots are
 * assigned in call order; an id >= n_lists is INVALID_ARGUMENT and nothing is
 * added. */
ELIPS_B200_API int elips_b200_ivfflat_add(elips_b200_ivfflat* index, const float* vectors,
                                          const uint32_t* assignments, size_t n);

/* Same with DEVICE pointers on `stream`. */
ELIPS_B200_API int elips_b200_ivfflat_add_device(elips_b200_ivfflat* index, const float* vectors,
                                                 const uint32_t* assignments, size_t n,
                                                 void* stream);

ELIPS_B200_API int elips_b200_ivfflat_size(const elips_b200_ivfflat* index, size_t* n_out);

ELIPS_B200_API int elips_b200_ivfflat_set_nprobe(elips_b200_ivfflat* index, uint32_t nprobe);

/* k <= 1024. HOST pointers, synchronous: out_dist[nq][k], out_rows[nq][k]
 * ascending by (distance, gather position); rows past the candidate count are
 * -1 (distance +inf). */
ELIPS_B200_API int elips_b200_ivfflat_search(elips_b200_ivfflat* index, const float* queries,
                                             size_t nq, size_t k, float* out_dist,
                                             int64_t* out_rows);

/* Same with DEVICE pointers, asynchronous on `stream`. */
ELIPS_B200_API int elips_b200_ivfflat_search_device(elips_b200_ivfflat* index, const float* queries,
                                                    size_t nq, size_t k, float* out_dist,
                                                    int64_t* out_rows, void* stream);

/* Snapshot readback: centroids, assignments and vectors in slot order (any may be NULL). */
ELIPS_B200_API int elips_b200_ivfflat_export(const elips_b200_ivfflat* index, float* centroids_out,
                                             uint32_t* assignments_out, float* vectors_out);

/* IvfIndexState::remove, as elips_b200_ivfpq_remove (IVF-Flat has no codes). */
ELIPS_B200_API int elips_b200_ivfflat_remove(elips_b200_ivfflat* index, size_t slot);

ELIPS_B200_API int elips_b200_ivfflat_destroy(elips_b200_ivfflat* index);

/* ------------------------------------------------------ dynamic batching */
/* elips::gpu::DynamicBatcher (src/gpu_engine/DynamicBatcher.cpp:1-124) over a
 * device exact index: concurrent single-query callers are coalesced (up to
 * max_batch queries, waiting at most window_us after the first) into one fused
 * search launch. elips_b200_batcher_search blocks until the caller's batch has
 * run and fills its k results exactly as elips_b200_exact_search would. Each
 * caller keeps its own k (the reference uses the first query's k for the
 * whole batch). The index must outlive the batcher and not change while it
 * runs; destroying the batcher serves the queries still pending. */
typedef struct elips_b200_batcher elips_b200_batcher;

ELIPS_B200_API int elips_b200_batcher_create(const elips_b200_exact* index, size_t window_us,
                                             size_t max_batch, elips_b200_batcher** out);
ELIPS_B200_API int elips_b200_batcher_search(elips_b200_batcher* batcher, const void* query, size_t k,
                                             float* out_dist, int64_t* out_rows);
/* Launches and queries so far (BatchStats::kernel_launches / queries_coalesced). */
ELIPS_B200_API int elips_b200_batcher_stats(const elips_b200_batcher* batcher, uint64_t* launches,
                                            uint64_t* queries);
/* DynamicBatcher::flush (DynamicBatcher.cpp:36-65): the queries pending now
 * are dispatched without waiting for the window; returns once every query
 * pending at the call has been served. Queries that arrive after the call
 * do not extend the wait. */
ELIPS_B200_API int elips_b200_batcher_flush(elips_b200_batcher* batcher);
/* Queries waiting for a batch (queued, not yet taken by the worker). The
 * reference's BatchStats (include/elips/gpu_engine/DynamicBatcher.hpp:32-37)
 * has no queue depth; this lets a caller see that its queries are queued. */
ELIPS_B200_API int elips_b200_batcher_pending(const elips_b200_batcher* batcher, uint64_t* pending);
ELIPS_B200_API int elips_b200_batcher_destroy(elips_b200_batcher* batcher);

/* ----------------------------------------------------------- index build */
/* Trainers, bit-identical to the reference's CPU loops (sequential fp32 sums,
 * strict '<' argmin with the lowest index kept). Host pointers unless
 * pointers_on_device is nonzero (then device pointers on `stream`). */

/* quant::detail::kmeans (src/quant_engine/KMeans.cpp:182-247): `k` centroids
 * [k][dim] of `rows` [n][dim], seeded from rows min(n-1, c*max(1,n/k)),
 * squared-L2 Lloyd rounds, at most `iters`, stopping once none moved. */
ELIPS_B200_API int elips_b200_kmeans(int device, const float* rows, size_t n, size_t dim, size_t k,
                                     size_t iters, float* centroids_out, int pointers_on_device,
                                     void* stream);

/* quant::detail::train_pq_codebook (KMeans.cpp:249-268), as called by
 * GpuQuantizationPipeline::train_pq_codebook (GpuQuantizationPipeline.cpp:
 * 17-33, iters = 10): one kmeans per subspace; codebook [pq_dim][ksub][dim/pq_dim]. */
ELIPS_B200_API int elips_b200_train_pq_codebook(int device, const float* rows, size_t n, size_t dim,
                                                size_t pq_dim, size_t ksub, size_t iters,
                                                float* codebook_out, int pointers_on_device,
                                                void* stream);

/* IvfIndexState::assign_vectors_to_centroids (src/gpu_engine/detail/
 * IvfIndexState.cpp:167-191): nearest list of every row by elips::distance,
 * and (distances_out, may be NULL) that distance, FLT_MAX where no distance
 * was below FLT_MAX (the reference's best_distance). */
ELIPS_B200_API int elips_b200_ivf_assign(int device, int metric, const float* rows, size_t n,
                                         size_t dim, const float* centroids, size_t n_lists,
                                         uint32_t* assignments_out, float* distances_out,
                                         int pointers_on_device, void* stream);

/* IvfIndexState::train_centroids + the final assignment (IvfIndexState.cpp:
 * 118-165, 193-208): max(1, iters) rounds; cosine centroids normalised.
 * n_lists in [1, n] (rebuild_from_current_data passes max(1, min(requested, n)));
 * assignments_out may be NULL. */
ELIPS_B200_API int elips_b200_ivf_train(int device, int metric, const float* rows, size_t n, size_t dim,
                                        size_t n_lists, size_t iters, float* centroids_out,
                                        uint32_t* assignments_out, int pointers_on_device,
                                        void* stream);

/* GpuIVFPQIndex's model build: ivf_train, residuals v - centroid, the PQ
 * codebook of the residuals (10 rounds, ksub = 1 << pq_bits) and the residual
 * codes [n][pq_dim] (GpuIVFPQIndex.cpp:88-131). codes_out may be NULL. */
ELIPS_B200_API int elips_b200_ivfpq_train(int device, int metric, const float* rows, size_t n,
                                          size_t dim, size_t n_lists, size_t iters, size_t pq_dim,
                                          uint32_t pq_bits, float* centroids_out,
                                          uint32_t* assignments_out, float* codebook_out,
                                          uint8_t* codes_out, int pointers_on_device, void* stream);

/* ------------------------------------------------------------ profiling */
/* Device-side counterpart of GpuProfiler (src/gpu_engine/GpuProfiler.cpp:
 * 5-23) and GpuConfig::enable_profiling (GpuConfig.hpp:83): while enabled,
 * every kernel this library launches is bracketed by CUDA events on its
 * launching stream. */
ELIPS_B200_API int elips_b200_profiler_enable(int enabled);

/* Totals since the last reset for one kernel ("exact_topk", "merge_topk",
 * "prep_rows", ...; NULL = all): timed launches, summed milliseconds, summed
 * work items. Waits for the pending events. Any output pointer may be NULL. */
ELIPS_B200_API int elips_b200_profiler_stats(const char* kernel, uint64_t* launches,
                                             double* total_ms, uint64_t* items);

ELIPS_B200_API int elips_b200_profiler_reset(void);

/* Kernels launched by this library since it was loaded (always counted,
 * GpuProfiler::total_launches). */
ELIPS_B200_API int elips_b200_launch_count(uint64_t* launches);

#ifdef __cplusplus
}
#endif

#endif /* ELIPS_B200_H */
