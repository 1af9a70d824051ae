/*
 * zcgvs_sm100.h - C ABI of the B200 (sm_100a) search hot path.
 *
 * This library replaces the reference engine's src/cuda/ directory (the brute-force scan,
 * multi-pass top-k, gather-rescore, BM25 and converter launchers) with fused sm_100a kernels
 * behind a plain C interface: pointers, sizes and an opaque stream handle, no C++ or torch
 * types. The C++ declarations of the reference (include/zcgvs/cuda/*.cuh, Searcher) are
 * re-implemented on top of this ABI in include/zcgvs/.
 *
 * Conventions shared by every entry point:
 *   - All device memory is owned by the caller. Entry points never allocate, never
 *     synchronise the stream and can be captured into a CUDA graph. Scratch is passed in as
 *     an explicit workspace whose size comes from the matching *_workspace_bytes() query.
 *   - A workspace must be zero-filled once before its first use (zcgvs_workspace_init or a
 *     cudaMemset); every call leaves its counters at zero again, so it can be reused by the
 *     next call on the same stream without re-initialisation.
 *   - `stream` is a cudaStream_t passed as void*; NULL is the legacy default stream.
 *   - Zero-sized problems (doc_count, batch or dim <= 0) are silent no-ops returning
 *     ZCGVS_OK, as in the reference launchers (src/cuda/similarity.cu:356-358).
 *   - Errors are reported as zcgvs_status codes; zcgvs_last_error_message() returns a
 *     thread-local description of the last failure on the calling thread.
 *   - Top-k order is the total order (score descending, document id ascending), identical to
 *     the reference CPU oracle's std::stable_sort (tests/cpp/cpu_reference.hpp:26-34). Padding
 *     slots hold id -1 and score -FLT_MAX. Masked documents score exactly -FLT_MAX
 *     (src/cuda/similarity.cu:109-113) and therefore rank after every unmasked document.
 */
#ifndef ZCGVS_SM100_H
#define ZCGVS_SM100_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. ZCGVS_ERR_INVALID_ARG mirrors the reference's std::invalid_argument
 * (src/cuda/topk.cu:146-153, src/cuda/similarity.cu:326-329), ZCGVS_ERR_CUDA its CudaError
 * (include/zcgvs/core/cuda_check.hpp:10-37). ZCGVS_ERR_DEVICE_STATUS means a kernel gave up a
 * bounded wait and recorded it in the workspace status word. */
typedef enum zcgvs_status {
    ZCGVS_OK = 0,
    ZCGVS_ERR_INVALID_ARG = 1,
    ZCGVS_ERR_CUDA = 2,
    ZCGVS_ERR_UNSUPPORTED = 3,
    ZCGVS_ERR_DEVICE_STATUS = 4,
    ZCGVS_ERR_COMM = 5 /* an NCCL call of the sharded search failed, or NCCL is unavailable */
} zcgvs_status;

/* Storage precision of a corpus. Codes 0-3 equal the reference ScalarType
 * (include/zcgvs/core/scalar_type.hpp:12-17) and the ZCVE dtype field
 * (include/zcgvs/data/binary_format.hpp:59-62). ZCGVS_DTYPE_I8_ROW is an extension: int8 rows
 * with one fp32 scale per row, scored as an exact int32 dot of the int8 query and row times
 * the two scales. */
typedef enum zcgvs_dtype {
    ZCGVS_DTYPE_F32 = 0,
    ZCGVS_DTYPE_F16 = 1,
    ZCGVS_DTYPE_I8 = 2,
    ZCGVS_DTYPE_BINARY = 3,
    ZCGVS_DTYPE_I8_ROW = 4
} zcgvs_dtype;

/* Similarity metric; codes equal the reference Metric (include/zcgvs/core/metric.hpp:8-12).
 * Cosine is the dot product of pre-normalised rows (include/zcgvs/cuda/decode.cuh:30-42). */
typedef enum zcgvs_metric {
    ZCGVS_METRIC_COSINE = 0,
    ZCGVS_METRIC_DOT = 1,
    ZCGVS_METRIC_L2 = 2
} zcgvs_metric;

/* Largest k / candidate count any selection supports; equals topKMaxK() of the reference
 * (src/cuda/topk.cu:117). */
#define ZCGVS_MAX_K 1024

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int zcgvs_version(void);

/* Thread-local description of the last error returned on this thread ("" if none). */
const char* zcgvs_last_error_message(void);

/* The cudaError_t value behind the last ZCGVS_ERR_CUDA returned on this thread (0 if none). */
int zcgvs_last_cuda_error(void);

/* Zero-fills `bytes` of a workspace on `stream` (a cudaMemsetAsync). */
int zcgvs_workspace_init(void* workspace, size_t bytes, void* stream);

/* Bits of the device status word that kernels set in the first 4 bytes of a workspace
 * (sticky: they stay set until the caller clears them, e.g. with zcgvs_workspace_init).
 * A non-zero word means the results of the calls since it was last cleared may be incomplete. */
#define ZCGVS_DEVICE_TILE_WAIT_TIMEOUT 0x1u  /* a bounded wait for a corpus tile ran out */
#define ZCGVS_DEVICE_DRAIN_TIMEOUT 0x2u      /* a bounded wait for in-flight copies ran out */
#define ZCGVS_DEVICE_TMEM_WAIT_TIMEOUT 0x4u  /* a tensor-memory accumulator hand-off ran out */
#define ZCGVS_DEVICE_CANDIDATE_OVERFLOW 0x8u /* a query of the tensor-core path kept more
                                                candidates than its buffer holds after every
                                                retry; its top-k is incomplete */

/* Copies the device status word of a workspace to *status and synchronises `stream`.
 * 0 means every bounded wait of every call that used the workspace completed and no
 * candidate buffer overflowed (ZCGVS_DEVICE_* bits above otherwise). */
int zcgvs_workspace_status(const void* workspace, size_t bytes, uint32_t* status, void* stream);

/* Test hook (no reference counterpart): caps the per-query candidate buffer of the tensor-core
 * path (zcgvs_gemm_topk, and zcgvs_scan_topk where it dispatches there) at `cap` entries instead
 * of 16384, so tests can drive a query past its buffer and check that the overflow reaches the
 * caller. 0 restores the default; 1..16384 are accepted. Process-wide; not for production use. */
int zcgvs_test_set_candidate_cap(int cap);

/* Diagnostic (no reference counterpart): launches one warp that waits on a shared-memory
 * barrier nothing ever completes, through the same bounded wait every kernel of this library
 * uses. The wait gives up after its 2 s budget, sets ZCGVS_DEVICE_TILE_WAIT_TIMEOUT in the
 * workspace status word and the kernel returns normally: the failure path a caller sees when a
 * real wait runs out, exercised without faulting or hanging the GPU. */
int zcgvs_check_bounded_wait(void* workspace, size_t bytes, void* stream);

/* Diagnostics (no reference counterpart): CUDA-event timing of the library's main kernel
 * launches, off by default. zcgvs_kernel_timing(1) clears earlier records and starts recording
 * an event pair around every tagged launch on its own stream; zcgvs_kernel_timing(0) stops.
 * zcgvs_kernel_timing_read synchronises the recorded events of `tag` and returns their summed
 * duration and count. Tags: "scan" (streaming scan), "gemm_sample", "gemm_threshold",
 * "gemm_filter", "gemm_bucket", "gemm_select", "gemm_retry", "gemm_emit", "rescore", "lexical",
 * "merge". */
int zcgvs_kernel_timing(int enable);
int zcgvs_kernel_timing_read(const char* tag, double* total_ms, int* launches);

/* ---------------------------------------------------------------------------------------
 * Fused scan + top-k. Replaces the launchSimilarity -> launchTopK chain of
 * Searcher::recordPipeline (src/search/searcher.cpp:230-232, :281-284): scores are kept on
 * chip and only the final [batch, k] selection is written.
 *
 *   corpus      : [doc_count, row] in `dtype` storage, row-major, rows of rowBytes(dtype, dim)
 *                 bytes (binary rows are ceil(dim/32) uint32 words).
 *   scale       : per-matrix dequantisation scale for ZCGVS_DTYPE_I8 (ignored otherwise).
 *   row_scales  : [doc_count] fp32 per-row scales for ZCGVS_DTYPE_I8_ROW (NULL otherwise).
 *   queries     : [batch, dim] fp32 on the device. The kernel widens (fp16/int8 paths, which
 *                 score against the fp32 query exactly as src/cuda/similarity.cu:83-164 does),
 *                 quantises per row (I8_ROW: s = max|x|/127, q = clamp(rint(x/s), +-127)) or
 *                 packs sign bits (BINARY, bit b of word w = dim 32w+b, set when x >= 0).
 *   mask        : optional [doc_count] uint8 allow-mask; 0 = excluded (scores -FLT_MAX).
 *   metric      : ZCGVS_METRIC_*; L2 scores -sum((q-x)^2). Ignored for BINARY, whose score is
 *                 (dim - 2*hamming)/dim (include/zcgvs/cuda/decode.cuh:45-47). L2 is
 *                 unsupported for I8_ROW.
 *   k           : 1..min(ZCGVS_MAX_K, doc_count).
 *   id_base     : added to every row index (global ids of a row shard); 0 for a whole corpus.
 *   out_indices : [batch, k] int32 document ids, descending by score.
 *   out_scores  : [batch, k] fp32 scores.
 *   Outputs may be device memory or pinned host memory (cudaHostAlloc / cudaMallocHost, which
 *   kernels can address under unified addressing): the last kernel then writes the result
 *   across the bus itself and no device-to-host copy is needed (worth it for small results;
 *   the same holds for zcgvs_hybrid_topk and zcgvs_rescore_topk). Inputs and the workspace
 *   stay in device memory.
 * --------------------------------------------------------------------------------------- */
size_t zcgvs_scan_topk_workspace_bytes(int dtype, int64_t doc_count, int dim, int batch, int k);

int zcgvs_scan_topk(const void* corpus, int dtype, float scale, const float* row_scales,
                    int64_t doc_count, int dim, const float* queries, int batch,
                    const uint8_t* mask, int metric, int k, int id_base, int* out_indices,
                    float* out_scores, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------
 * Fused scan + top-k without a workspace, for callers that cannot allocate device memory
 * (hosts that own every byte of GPU memory and forbid plug-ins from calling cudaMalloc, or
 * paths where an allocation's implicit device synchronisation is not allowed). No
 * counterpart in the reference: it has no entry point that runs without caller scratch.
 *
 * Same arguments, results and errors as zcgvs_scan_topk, minus the workspace. Scratch is a
 * fixed 32 MiB __device__ array inside this library, reserved on every GPU that loads it until
 * the process exits; searches needing more (zcgvs_scan_topk_workspace_bytes() > 32 MiB, e.g. a
 * single query over more than ~4M rows) return ZCGVS_ERR_INVALID_ARG. The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress) and should come before any
 * stream capture. All calls on a device share the array: each clears its header on `stream`,
 * and calls whose kernels overlap on the GPU race, so callers must serialise them. Allocates
 * nothing (no cudaMalloc / cudaFree).
 * --------------------------------------------------------------------------------------- */
int zcgvs_scan_topk_noalloc(const void* corpus, int dtype, float scale, const float* row_scales,
                            int64_t doc_count, int dim, const float* queries, int batch,
                            const uint8_t* mask, int metric, int k, int id_base, int* out_indices,
                            float* out_scores, void* stream);

/* ---------------------------------------------------------------------------------------
 * Score matrix. Same contract as the reference launchSimilarity
 * (include/zcgvs/cuda/similarity.cuh:20-30): writes [batch, doc_count] fp32 scores. Float
 * storage takes fp32 queries; binary storage takes packed query words [batch, ceil(dim/32)]
 * (as produced by zcgvs_pack_binary), like the reference.
 * --------------------------------------------------------------------------------------- */
int zcgvs_similarity(const void* corpus, int dtype, float scale, const float* row_scales,
                     int64_t doc_count, int dim, const void* queries, int batch,
                     const uint8_t* mask, int metric, float* scores, void* stream);

/* ---------------------------------------------------------------------------------------
 * Fused candidate rescoring. Replaces the rescore chain of Searcher::recordPipeline
 * (src/search/searcher.cpp:266-279): launchGatherRescore (src/cuda/rescore.cu:87-130), the
 * second launchTopK over its [batch, candidate_count] values and launchRemapIndices
 * (:132-146), as one kernel that gathers every candidate row, scores it exactly against the
 * fp32 query and writes the final top-k with corpus ids.
 *
 *   store           : the rescore corpus (F32, F16, I8 with `scale`, or I8_ROW with
 *                     `row_scales`); BINARY returns ZCGVS_ERR_INVALID_ARG, as in the reference.
 *   candidates      : [batch, candidate_count] corpus ids (e.g. a coarse zcgvs_scan_topk
 *                     result); ids outside [0, doc_count), such as -1 padding, are skipped.
 *   candidate_count : 1..8192.
 *   k               : 1..min(ZCGVS_MAX_K, candidate_count).
 *   out_indices / out_scores : [batch, k], (score desc, id asc), padded with (-1, -FLT_MAX)
 *                     when fewer than k candidates are valid.
 * --------------------------------------------------------------------------------------- */
int zcgvs_rescore_topk(const void* store, int dtype, float scale, const float* row_scales,
                       int64_t doc_count, int dim, const float* queries, int batch,
                       const int* candidates, int candidate_count, int metric, int k,
                       int* out_indices, float* out_scores, void* stream);

/* Score matrix of a candidate set: the reference launchGatherRescore contract
 * (include/zcgvs/cuda/rescore.cuh:20-32). values[q, j] = exact score of candidates[q, j], or
 * -FLT_MAX when that id is outside [0, doc_count). */
int zcgvs_gather_rescore(const void* store, int dtype, float scale, const float* row_scales,
                         int64_t doc_count, int dim, const float* queries, int batch,
                         const int* candidates, int candidate_count, int metric, float* values,
                         void* stream);

/* ---------------------------------------------------------------------------------------
 * Tensor-core batched search (tcgen05 MMA, TMEM accumulators, TMA). For large query batches
 * the scan is a dense contraction; the reference has no tensor-core path (it runs its CUDA-core
 * similarity kernel per 8 queries, src/cuda/similarity.cu:83-164, and writes the [batch, N]
 * score matrix). Corpora: ZCGVS_DTYPE_F16 (queries rounded to fp16, fp32 accumulation),
 * ZCGVS_DTYPE_I8_ROW (queries quantised per row as in zcgvs_scan_topk, exact int32 dot, so the
 * result equals zcgvs_scan_topk bit for bit) and ZCGVS_DTYPE_BINARY (sign bits expanded to int8
 * on chip, the exact Hamming score (dim - 2 h) / dim, equal to zcgvs_scan_topk bit for bit).
 * Rows must be multiples of 128 bytes of operand (dim % 64 == 0 for F16, dim % 128 == 0 for
 * I8_ROW and BINARY); metric dot or cosine (BINARY: any metric, the score is Hamming's).
 * zcgvs_scan_topk routes I8_ROW batches >= 64 and BINARY batches >= 16 over >= 65536 rows here.
 *
 * zcgvs_gemm_topk: a threshold pre-pass over a sample of document tiles (per query, the k-th
 * largest tile maximum, a lower bound of the k-th best score), a filtered pass over the whole
 * corpus that keeps only documents at or above it, and an exact selection of those candidates.
 * Arguments and result as zcgvs_scan_topk. A query still holding more than 16384 candidates
 * at its threshold after both retries sets ZCGVS_DEVICE_CANDIDATE_OVERFLOW (value 8, bit 3) in
 * the workspace status word (zcgvs_workspace_status); its result is then incomplete. The
 * workspace must be 256-byte aligned; apart from its status word (the first 4 bytes: zero
 * them once, and again after reading a non-zero value, since the bits are sticky) it needs no
 * zero-fill.
 *
 * zcgvs_gemm_similarity: the [batch, doc_count] score matrix (masked documents -FLT_MAX).
 * --------------------------------------------------------------------------------------- */
size_t zcgvs_gemm_topk_workspace_bytes(int dtype, int64_t doc_count, int dim, int batch, int k);

int zcgvs_gemm_topk(const void* corpus, int dtype, const float* row_scales, int64_t doc_count,
                    int dim, const float* queries, int batch, const uint8_t* mask, int metric,
                    int k, int id_base, int* out_indices, float* out_scores, void* workspace,
                    size_t workspace_bytes, void* stream);

size_t zcgvs_gemm_similarity_workspace_bytes(int dtype, int64_t doc_count, int dim, int batch);

int zcgvs_gemm_similarity(const void* corpus, int dtype, const float* row_scales,
                          int64_t doc_count, int dim, const float* queries, int batch,
                          const uint8_t* mask, int metric, float* scores, void* workspace,
                          size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------
 * Merge of per-shard top-k lists (row-sharded multi-GPU search). No reference counterpart:
 * the reference runs on one GPU; its single-GPU merge is mergeTopKKernel
 * (src/cuda/topk.cu:76-115).
 *
 *   list_indices / list_scores : [lists, batch, k_in] (the layout an all-gather of every
 *                     shard's [batch, k_in] result produces); ids are global (each shard
 *                     searched with id_base = its first row); ids < 0 are padding.
 *   lists * k_in    : at most 16384.
 *   out_indices / out_scores   : [batch, k], (score desc, id asc), padded with (-1, -FLT_MAX).
 * --------------------------------------------------------------------------------------- */
int zcgvs_merge_topk(const int* list_indices, const float* list_scores, int lists, int batch,
                     int k_in, int k, int* out_indices, float* out_scores, void* stream);

/* The general form of zcgvs_merge_topk, which reads an all-gather's output in place and folds
 * in the steps around the merge of a sharded search:
 *   list p's entries are list_indices[p * list_stride + q * k_in + i] and the same offsets of
 *   list_scores (an all-gather of packed [2, batch, k_in] int32 blocks, ids then score bits, is
 *   read with list_stride = 2 * batch * k_in and list_scores = list_indices + batch * k_in);
 *   list_id_offsets (optional, [lists] int32 on the device) is added to the ids of list p
 *   (shard-local ids become global ids);
 *   out_indices / out_scores (optional together) receive the merged [batch, k];
 *   out_owned (optional) receives, per merged entry, id - own_begin when the id lies in
 *   [own_begin, own_end) and -1 otherwise: the shard-local candidate list a rank rescores.
 * At least one output must be given. */
int zcgvs_merge_topk_lists(const int* list_indices, const float* list_scores, int64_t list_stride,
                           int lists, int batch, int k_in, const int* list_id_offsets, int k,
                           int* out_indices, float* out_scores, int own_begin, int own_end,
                           int* out_owned, void* stream);

/* ---------------------------------------------------------------------------------------
 * Row-sharded search across the GPUs of one node, one process per GPU, over NCCL. No reference
 * counterpart (the reference runs on one GPU). The corpus' rows are split evenly into `world`
 * contiguous shards (zcgvs_shard_bounds); rank r holds rows [begin, end) of every store on its
 * GPU. A search runs the local fused search with global ids, an NCCL all-gather of every
 * rank's packed [batch, k] (id, score) list and zcgvs_merge_topk_lists on the device, so every
 * rank ends with the global top-k, identical to a one-GPU search over the whole corpus (the
 * union of the per-shard top-k lists contains the global top-k and the order is total). The
 * rescore search follows the reference's pipeline semantics: global coarse top-M (exchange and
 * merge), each rank rescoring the candidates it owns, exchange and merge of the top-k.
 *
 * NCCL is loaded at run time (libnccl.so.2; in a process that already loaded NCCL, such as one
 * running torch.distributed, the loaded copy). A handle owns its communicator, its exchange
 * buffers and workspace (allocated, and zero-filled, by the first search of a larger shape) and
 * one CUDA graph: with ZCGVS_SHARDED_GRAPH the first search of a shape runs directly and is then
 * captured, and later searches with the same arguments replay the whole step (local search,
 * all-gathers, merges, rescoring) as one graph launch. Every rank must make the same calls in
 * the same order. Not thread-safe: one handle per process and stream.
 * --------------------------------------------------------------------------------------- */
typedef struct zcgvs_sharded zcgvs_sharded;

#define ZCGVS_SHARDED_GRAPH 0x1u       /* capture each search shape once, replay it after */
#define ZCGVS_SHARDED_F16_TENSOR 0x2u  /* fp16 shards: local search on the tensor cores
                                          (zcgvs_gemm_topk, fp16 queries) */

/* Rows [*begin, *end) of shard `rank` when total_rows rows are split over `world` shards as
 * evenly as possible (the first total_rows % world shards hold one row more). */
int zcgvs_shard_bounds(int64_t total_rows, int world, int rank, int64_t* begin, int64_t* end);

/* Bytes of an NCCL unique id (128). Rank 0 makes one with zcgvs_nccl_unique_id and sends it to
 * the other ranks by any channel (a file, a TCP store, MPI). */
size_t zcgvs_nccl_id_bytes(void);
int zcgvs_nccl_unique_id(void* id);

/* Creates the handle of rank `rank` of `world` on the current device (a collective: every rank
 * must call it with the same id, world and total_rows). */
int zcgvs_sharded_create(const void* nccl_id, int world, int rank, int64_t total_rows,
                         zcgvs_sharded** out);
int zcgvs_sharded_destroy(zcgvs_sharded* handle);

/* Dense search: `shard` holds this rank's shard_rows rows (the arguments of zcgvs_scan_topk
 * otherwise; ids in the result are global). k <= shard_rows. Writes [batch, k] on every rank. */
int zcgvs_sharded_search(zcgvs_sharded* handle, const void* shard, int dtype, float scale,
                         const float* row_scales, int64_t shard_rows, int dim, const float* queries,
                         int batch, const uint8_t* mask, int metric, int k, unsigned flags,
                         int* out_indices, float* out_scores, void* stream);

/* Coarse search over this rank's codes (any dtype zcgvs_scan_topk takes, e.g. 1-bit), the
 * global top-`candidates`, exact rescoring of the owned candidates against this rank's rows of
 * `store` (as zcgvs_rescore_topk), and the global top-k. k <= candidates <= shard_rows. */
int zcgvs_sharded_rescore_search(zcgvs_sharded* handle, const void* codes, int code_dtype,
                                 float code_scale, const float* code_row_scales, const void* store,
                                 int store_dtype, float store_scale, const float* store_row_scales,
                                 int64_t shard_rows, int dim, const float* queries, int batch,
                                 int metric, int candidates, int k, unsigned flags,
                                 int* out_indices, float* out_scores, void* stream);

/* The device status word of the handle's local-search workspace (ZCGVS_DEVICE_* bits; sticky)
 * and the communicator's asynchronous NCCL error, after synchronising `stream`. A non-zero
 * status or comm_error means the searches since the last clear may be incomplete. */
int zcgvs_sharded_status(zcgvs_sharded* handle, uint32_t* status, int* comm_error, void* stream);
int zcgvs_sharded_clear_status(zcgvs_sharded* handle, void* stream);

/* ---------------------------------------------------------------------------------------
 * Hybrid lexical + dense search. Replaces the hybrid stages of Searcher::recordPipeline
 * (src/search/searcher.cpp:236-263: per query launchBm25, launchMaxPositive and
 * launchFuseScores over [batch, N] score matrices, then launchTopK) with two kernels, blending
 * score = w * dense + ((1 - w) * lex) * (1 / max(lex)) (0 when the max is not positive;
 * src/cuda/lexical.cu:66-72) before the top-k. One query (batch 1, k <= 192, a dense dtype and
 * dimension of the single-query scan, 16-byte aligned posting arrays): a scan whose CTAs also
 * accumulate the BM25 scores of their own documents, writing both score vectors to the
 * workspace, then a blend + top-k kernel launched as its programmatic dependent. Otherwise: a
 * BM25 kernel that writes each query's lexical scores and partial maxima, then the scan that
 * blends before its top-k. Both give the same results, bit for bit.
 *
 *   offsets / posting_docs / posting_weights : the CSR index of the reference LexicalIndex
 *                     (include/zcgvs/data/lexical_index.hpp:14-46): offsets [vocab_size + 1]
 *                     int64, per-term posting documents int32 and BM25 weights fp32. Posting
 *                     lists must be sorted by document id within each term (the reference
 *                     builder writes them so, python/zcgvs_tools/build_lexical.py:143-162).
 *   query_terms     : [batch, term_stride] term ids; ids outside [0, vocab_size), such as the
 *                     -1 padding, are ignored. Duplicate ids count once per occurrence, as in
 *                     the reference (the engine de-duplicates before searching).
 *   dense_weight    : w above; the dense score is the corpus scan's (masked documents
 *                     -FLT_MAX before blending, as in the reference).
 * Lexical scores are sums in (term slot, posting) order, identical to the sequential CPU sum;
 * term_stride <= 0 or query_terms == NULL runs the dense search alone. The remaining arguments
 * and the result are those of zcgvs_scan_topk (id_base is 0).
 * --------------------------------------------------------------------------------------- */
size_t zcgvs_hybrid_topk_workspace_bytes(int dtype, int64_t doc_count, int dim, int batch, int k);

int zcgvs_hybrid_topk(const void* corpus, int dtype, float scale, const float* row_scales,
                      int64_t doc_count, int dim, const float* queries, int batch,
                      const uint8_t* mask, int metric, const int64_t* offsets,
                      const int* posting_docs, const float* posting_weights, int vocab_size,
                      const int* query_terms, int term_stride, float dense_weight, int k,
                      int* out_indices, float* out_scores, void* workspace,
                      size_t workspace_bytes, void* stream);

/* The reference lexical launchers (include/zcgvs/cuda/lexical.cuh:20-40), same contracts:
 *   zcgvs_bm25         : scores[d] += weights of d's postings under the valid terms of one
 *                        query, summed in (slot, posting) order (deterministic), for postings
 *                        in any order; every document range reads the query's whole lists, so
 *                        zcgvs_hybrid_topk (sorted lists, each range reads its slice) is the fast
 *                        path. Term ids are trusted to be < the index's vocabulary, as in the
 *                        reference.
 *   zcgvs_max_positive : *out_max = max(*out_max, max(0, max_i values[i])) (zero it first).
 *   zcgvs_fuse_scores  : dense[i] = w * dense[i] + ((1 - w) * lexical[i]) * inv, inv =
 *                        1 / *lexical_max when positive, else 0. */
int zcgvs_bm25(const int64_t* offsets, const int* posting_docs, const float* posting_weights,
               const int* query_terms, int term_count, int doc_count, float* scores, void* stream);
int zcgvs_max_positive(const float* values, int count, float* out_max, void* stream);
int zcgvs_fuse_scores(float* dense, const float* lexical, const float* lexical_max, float weight,
                      int count, void* stream);

/* ---------------------------------------------------------------------------------------
 * The remaining reference launchers, same contracts (for callers that still build a score
 * matrix or convert host matrices into stores):
 *   zcgvs_topk          : launchTopK (include/zcgvs/cuda/topk.cuh:8-43): the top-k of every
 *                         row of scores [batch, doc_count] into [batch, k], (score desc, id asc);
 *                         1 <= k <= min(ZCGVS_MAX_K, doc_count); needs no scratch.
 *   zcgvs_convert_f16   : launchConvertF32ToF16 (include/zcgvs/cuda/convert.cuh:10-20).
 *   zcgvs_convert_i8    : launchConvertF32ToI8: clamp(rint(x * (1 / scale)), +-127) with the
 *                         reciprocal taken on the host (0 when scale <= 0).
 *   zcgvs_convert_i8_rows : the per-row extension of launchConvertF32ToI8 that builds
 *                         ZCGVS_DTYPE_I8_ROW stores: per row, scale = max|x| / 127 (1 for an
 *                         all-zero row) into row_scales[rows], then clamp(rint(x * (1 / scale)),
 *                         +-127) into dst_int8 [rows, dim].
 *   zcgvs_pack_binary   : launchPackBinary: bit b of word w = dim 32w+b, set when x >= 0.
 *   zcgvs_remap_indices : launchRemapIndices (include/zcgvs/cuda/rescore.cuh:34-45).
 * --------------------------------------------------------------------------------------- */
int zcgvs_topk(const float* scores, int64_t doc_count, int k, int batch, int* out_indices,
               float* out_scores, void* stream);
int zcgvs_convert_f16(const float* src, void* dst_half, size_t count, void* stream);
int zcgvs_convert_i8(const float* src, void* dst_int8, size_t count, float scale, void* stream);
int zcgvs_convert_i8_rows(const float* src, void* dst_int8, float* row_scales, int64_t rows, int dim,
                          void* stream);
int zcgvs_pack_binary(const float* src, void* dst_words, int64_t rows, int dim, void* stream);
int zcgvs_remap_indices(const int* candidates, const int* local_indices, int candidate_count,
                        int k, int batch, int* out_indices, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* ZCGVS_SM100_H */
