// Host side of the streaming scan: launch planning (tile size, stage depth, query pass width,
// grid), workspace layout, argument validation and the C-ABI entry points zcgvs_scan_topk and
// zcgvs_similarity.
#include <algorithm>
#include <climits>
#include <string>

#include "host_common.h"
#include "lexical.h"
#include "scan_fast.cuh"
#include "scan_instances.h"
#include "zcgvs_sm100.h"

namespace zc {

namespace {

constexpr int kTileTargetBytes = 48 * 1024;
constexpr int kMaxStages = 8;
constexpr int kMaxTileRows = 512;
constexpr size_t kWorkspaceAlign = 256;

struct ScanPlan {
    int mode = 0;
    int k = 1;
    int qb = 1;
    int jc = 0;
    bool l2 = false;
    bool emit = false;
    int row_bytes = 0;
    int stride = 0;
    int nch = 0;
    int elems_per_row = 0;
    bool use_tma = false;
    int rows_per_tile = 0;
    long long ntiles = 0;
    int grid_rows = 0;  // CTAs along the corpus (gridDim.y)
    int passes = 0;     // query passes (gridDim.x)
    int cap = 0;
    int stages = 1;
    int query_bytes = 0;
    bool side_scales = false;
    bool side_mask = false;
    int stage_bytes = 0;
    int side_off_scales = 0;
    int side_off_mask = 0;
    int smem_query_off = 0;
    int smem_topk_off = 0;
    int smem_bar_off = 0;
    int smem_total = 0;
    size_t ws_header = 0;
    size_t ws_lists = 0;
    size_t ws_total = 0;
    // Warp-specialised single-query variant (scan_fast.cuh), same tiles, grid and workspace.
    bool fast = false;
    int fast_stages = 0;
    int fast_ccap = 0;
    int fast_scap = 0;
    int fast_cap_final = 0;
    int cap_final = 0;
    long long fast_spill_stride = 0;
    int fast_query_off = 0;
    int fast_topk_off = 0;
    int fast_bar_off = 0;
    int fast_smem = 0;
};

int mode_of(int dtype) {
    switch (dtype) {
        case ZCGVS_DTYPE_F32: return kModeF32;
        case ZCGVS_DTYPE_F16: return kModeF16;
        case ZCGVS_DTYPE_I8: return kModeI8M;
        case ZCGVS_DTYPE_BINARY: return kModeBin;
        case ZCGVS_DTYPE_I8_ROW: return kModeI8R;
        default: return -1;
    }
}

int query_bytes_of(int mode, int stride) {
    switch (mode) {
        case kModeF32: return stride;       // 4 fp32 per 16-byte chunk
        case kModeF16: return 2 * stride;   // 8 fp32 per chunk
        case kModeI8M: return 4 * stride;   // 16 fp32 per chunk
        default: return stride;             // int8 values / packed words, like the rows
    }
}

// Fills the shared-memory layout for a given pass width / tile size; false if it cannot fit.
bool layout(ScanPlan& plan, int budget) {
    const int R = plan.rows_per_tile;
    plan.side_off_scales = R * plan.stride;
    plan.side_off_mask = plan.side_off_scales + (plan.side_scales ? static_cast<int>(round_up(4 * R, 16)) : 0);
    const int tile_bytes = static_cast<int>(
        round_up(plan.side_off_mask + (plan.side_mask ? static_cast<int>(round_up(R, 16)) : 0), 128));
    plan.stage_bytes = tile_bytes;
    const int query = plan.qb * plan.query_bytes;
    const int topk = plan.emit ? 0 : plan.qb * (plan.cap * 8 + 16);
    const int fixed = static_cast<int>(round_up(query, 128)) + static_cast<int>(round_up(topk, 128)) +
                      kMaxStages * 8 + 128;
    int stages = 1;
    if (plan.use_tma) {
        stages = std::min(kMaxStages, (budget - fixed) / std::max(tile_bytes, 1));
        if (stages < 2) return false;
    } else if (fixed + tile_bytes > budget) {
        return false;
    }
    plan.stages = stages;
    // After the scan the ring hosts the cross-CTA merge buffer: at least k + kScanThreads keys.
    size_t ring = static_cast<size_t>(stages) * tile_bytes;
    if (!plan.emit) {
        ring = std::max(ring, 8 * static_cast<size_t>(next_pow2(plan.k + kScanThreads)));
        size_t cap = 1;
        while (cap * 2 * 8 <= ring) cap *= 2;
        plan.cap_final = static_cast<int>(cap);
    }
    plan.smem_query_off = static_cast<int>(round_up(ring, 128));
    plan.smem_topk_off = plan.smem_query_off + static_cast<int>(round_up(query, 128));
    plan.smem_bar_off = plan.smem_topk_off + static_cast<int>(round_up(topk, 128));
    plan.smem_total = plan.smem_bar_off + kMaxStages * 8;
    return plan.smem_total <= budget;
}

// Builds the launch plan. Returns ZCGVS_OK or an error status (message recorded).
int make_plan(int dtype, long long n, int dim, int batch, int k, int metric, bool emit,
              bool aligned, bool has_mask, ScanPlan& plan) {
    plan.mode = mode_of(dtype);
    if (plan.mode < 0) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs: unknown storage dtype " + std::to_string(dtype));
    if (metric < ZCGVS_METRIC_COSINE || metric > ZCGVS_METRIC_L2) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs: unknown metric " + std::to_string(metric));
    }
    plan.l2 = (metric == ZCGVS_METRIC_L2) && plan.mode != kModeBin;
    if (plan.l2 && plan.mode == kModeI8R) {
        return fail(ZCGVS_ERR_UNSUPPORTED, "zcgvs: the per-row int8 store scores dot/cosine only");
    }
    plan.emit = emit;
    plan.k = k;
    plan.side_scales = (plan.mode == kModeI8R);
    plan.side_mask = has_mask;
    const long long rb = row_bytes_of(dtype, dim);
    plan.row_bytes = static_cast<int>(rb);
    plan.stride = static_cast<int>(round_up(static_cast<size_t>(rb), 16));
    plan.nch = plan.stride / 16;
    plan.elems_per_row = (plan.mode == kModeBin) ? (dim + 31) / 32 : dim;
    plan.use_tma = aligned && (rb % 16 == 0);
    plan.query_bytes = query_bytes_of(plan.mode, plan.stride);

    const int budget = device_max_smem() - 2048;
    // Fast path: a single query held in registers, 16 lanes per row, two rows per lane group,
    // planned when the row is exactly 2/3/4/6/8 sweeps of 16 lanes x 16 bytes.
    const int fast_jc = (plan.nch % 16 == 0) ? plan.nch / 16 : 0;
    const bool fast_ok = !emit && !plan.l2 && plan.mode != kModeBin &&
                         (fast_jc == 2 || fast_jc == 3 || fast_jc == 4 || fast_jc == 6 || fast_jc == 8);
    // Rows per tile: about kTileTargetBytes, rounded to whole CTA steps so no warp idles at the
    // tile barrier (64 rows for the fast path, 16 for warp-per-row, 32 for thread-per-row).
    auto rows_for = [&](int qb) {
        const int step = (qb == 1 && fast_ok) ? 64 : (plan.mode == kModeBin ? 32 : 16);
        int r = std::max(1, kTileTargetBytes / plan.stride);
        if (r >= step) {
            r = r / step * step;
        } else if (step * plan.stride <= 2 * kTileTargetBytes) {
            r = step;
        } else if (r >= 16) {
            r &= ~15;
        }
        return std::min(r, kMaxTileRows);
    };
    int qb = emit ? 8 : (batch <= 1 ? 1 : std::min(8, next_pow2(batch)));
    int rows = rows_for(qb);
    const int sms = device_sm_count();

    for (;;) {
        plan.qb = qb;
        plan.rows_per_tile = rows;
        plan.ntiles = (n + rows - 1) / rows;
        plan.grid_rows = static_cast<int>(std::min<long long>(plan.ntiles, sms));
        plan.cap = emit ? 0 : next_pow2(k + std::max(rows, plan.grid_rows));
        if (layout(plan, budget)) break;
        if (rows > 1) {
            rows = std::max(1, rows / 2);
            continue;
        }
        if (qb > 1) {
            qb /= 2;
            rows = rows_for(qb);
            continue;
        }
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs similarity: embedding dim " + std::to_string(dim) +
                                               " needs more shared memory than a block can stage");
    }
    plan.passes = (batch + plan.qb - 1) / plan.qb;
    plan.jc = (plan.qb == 1 && fast_ok) ? fast_jc : 0;

    // The warp-specialised kernel needs the bulk-copy ring and k <= 192. Its shared memory
    // holds the stage ring, the query, the CTA candidate buffer and the selector's buffer; the
    // ring must also fit the final merge buffer once the scan is over.
    if (plan.jc > 0 && plan.use_tma && k <= kSelCap - 64 && !(plan.mode == kModeI8M && plan.jc > 4)) {
        plan.fast_ccap = kCandCap;
        plan.fast_scap = kSelCap;
        plan.fast_cap_final = next_pow2(k + 8 * kFastThreads);
        const int query = static_cast<int>(round_up(plan.query_bytes, 128));
        const int bufs = 8 * (plan.fast_ccap + plan.fast_scap);
        const int fixed = query + bufs + 2 * kMaxStages * 8 + 128;
        const int stages = std::min(kMaxStages, (budget - fixed) / plan.stage_bytes);
        const long long ring = static_cast<long long>(stages) * plan.stage_bytes;
        if (stages >= 2 && ring >= 8LL * plan.fast_cap_final) {
            plan.fast = true;
            plan.fast_stages = stages;
            plan.fast_query_off = static_cast<int>(round_up(static_cast<size_t>(ring), 128));
            plan.fast_topk_off = plan.fast_query_off + query;
            plan.fast_bar_off = plan.fast_topk_off + bufs;
            plan.fast_smem = plan.fast_bar_off + 2 * kMaxStages * 8;
            // Per consumer warp: a slot for every row it can score (whole 64-row CTA steps).
            const long long steps = (plan.rows_per_tile + 63) / 64;
            plan.fast_spill_stride = (plan.ntiles + plan.grid_rows - 1) / plan.grid_rows * steps * 64;
        }
    }
    plan.ws_header = round_up(16 + 4 * static_cast<size_t>(plan.passes), kWorkspaceAlign);
    plan.ws_lists = static_cast<size_t>(batch) * plan.grid_rows * static_cast<size_t>(k) * 8;
    plan.ws_total = emit ? 0 : plan.ws_header + plan.ws_lists;
    if (plan.fast) {
        plan.ws_total += static_cast<size_t>(plan.passes) * plan.grid_rows *
                         static_cast<size_t>(plan.fast_spill_stride) * 8;
    }
    return ZCGVS_OK;
}

ScanKernelFn lookup(const ScanPlan& plan) {
    switch (plan.mode) {
        case kModeF32: return scan_lookup_f32(plan.qb, plan.jc, plan.l2, plan.emit);
        case kModeF16: return scan_lookup_f16(plan.qb, plan.jc, plan.l2, plan.emit);
        case kModeI8M:
        case kModeI8R: return scan_lookup_i8(plan.mode, plan.qb, plan.jc, plan.l2, plan.emit);
        case kModeBin: return scan_lookup_bin(plan.qb, plan.emit);
        default: return nullptr;
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool aligned_to(const void* p, uintptr_t bytes) {
    return (reinterpret_cast<uintptr_t>(p) & (bytes - 1u)) == 0;
}

// Every device pointer must be aligned to its element type (the plain-copy staging path reads
// whole elements); fp32 / int32 buffers to 4 bytes, fp16 rows to 2.
int check_alignment(int dtype, const void* corpus, const void* row_scales, const void* queries,
                    const void* out_a, const void* out_b) {
    const uintptr_t elem = (dtype == ZCGVS_DTYPE_F32 || dtype == ZCGVS_DTYPE_BINARY) ? 4u
                           : (dtype == ZCGVS_DTYPE_F16)                               ? 2u
                                                                                      : 1u;
    if (!aligned_to(corpus, elem) || !aligned_to(row_scales, 4) || !aligned_to(queries, 4) ||
        !aligned_to(out_a, 4) || !aligned_to(out_b, 4)) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs: a device pointer is not aligned to its element size");
    }
    return ZCGVS_OK;
}

// The plan's tile, stage and shared-memory layout fields of the kernel arguments.
void fill_params(const ScanPlan& plan, ScanParams& params) {
    params.rows_per_tile = plan.rows_per_tile;
    params.ntiles = plan.ntiles;
    params.use_tma = plan.use_tma ? 1 : 0;
    params.stages = plan.fast ? plan.fast_stages : plan.stages;
    params.cap = plan.fast ? plan.fast_ccap : plan.cap;
    params.merge_cap = plan.fast_scap;
    params.cap_final = plan.fast ? plan.fast_cap_final : plan.cap_final;
    params.spill_stride = plan.fast_spill_stride;
    params.row_bytes = plan.row_bytes;
    params.stride = plan.stride;
    params.nch = plan.nch;
    params.elems_per_row = plan.elems_per_row;
    params.query_bytes = plan.query_bytes;
    params.stage_bytes = plan.stage_bytes;
    params.side_scales = plan.side_scales ? 1 : 0;
    params.side_off_scales = plan.side_off_scales;
    params.side_off_mask = plan.side_off_mask;
    params.side_tma = (plan.use_tma && plan.rows_per_tile % 16 == 0 &&
                       (!plan.side_scales || aligned16(params.row_scales)) &&
                       (params.mask == nullptr || aligned16(params.mask)))
                          ? 1
                          : 0;
    params.smem_query_off = plan.fast ? plan.fast_query_off : plan.smem_query_off;
    params.smem_topk_off = plan.fast ? plan.fast_topk_off : plan.smem_topk_off;
    params.smem_bar_off = plan.fast ? plan.fast_bar_off : plan.smem_bar_off;
}

int launch(const ScanPlan& plan, ScanParams& params, cudaStream_t stream) {
    const ScanKernelFn kernel = plan.fast ? scan_lookup_fast(plan.mode, plan.jc) : lookup(plan);
    if (kernel == nullptr) {
        return fail(ZCGVS_ERR_UNSUPPORTED, "zcgvs: no scan kernel variant for this configuration");
    }
    cudaError_t status = ensure_smem_optin(reinterpret_cast<const void*>(kernel));
    if (status != cudaSuccess) return fail_cuda(status, "cudaFuncSetAttribute(scan_kernel)");
    fill_params(plan, params);
    const dim3 grid(static_cast<unsigned>(plan.passes), static_cast<unsigned>(plan.grid_rows));
    const int threads = plan.fast ? kFastThreads : kScanThreads;
    const int smem = plan.fast ? plan.fast_smem : plan.smem_total;
    {
        KernelTimer timer("scan", stream);
        kernel<<<grid, threads, smem, stream>>>(params);
    }
    status = cudaGetLastError();
    if (status != cudaSuccess) return fail_cuda(status, "scan_kernel launch");
    return ok();
}

}  // namespace

}  // namespace zc

namespace zc {
namespace {

// Large batches over per-row int8 and 1-bit corpora run on the tensor cores (zcgvs_gemm_topk):
// the same exact integer dot products, so the same results bit for bit. Smaller problems stay on
// the streaming scan, whose single pass has no fixed cost. A 1-bit row costs the streaming scan
// 32 popcounts per 1,024 dimensions and query, so the tensor cores take over at smaller batches.
constexpr int kGemmMinBatch = 64;
constexpr int kGemmMinBatchBinary = 16;
constexpr long long kGemmMinDocs = 65536;

bool gemm_eligible(int dtype, long long n, int dim, int batch, int metric) {
    if (n < kGemmMinDocs || dim % 128 != 0) return false;
    if (dtype == ZCGVS_DTYPE_BINARY) return batch >= kGemmMinBatchBinary;  // every metric scores Hamming
    return dtype == ZCGVS_DTYPE_I8_ROW && batch >= kGemmMinBatch &&
           (metric == ZCGVS_METRIC_DOT || metric == ZCGVS_METRIC_COSINE);
}

}  // namespace
}  // namespace zc

extern "C" {

size_t zcgvs_scan_topk_workspace_bytes(int dtype, int64_t doc_count, int dim, int batch, int k) {
    if (doc_count <= 0 || dim <= 0 || batch <= 0 || k <= 0) return 0;
    if (zc::gemm_eligible(dtype, doc_count, dim, batch, ZCGVS_METRIC_DOT)) {
        const size_t gemm = zcgvs_gemm_topk_workspace_bytes(dtype, doc_count, dim, batch, k);
        zc::ok();
        // Either path may run (the tensor-core one needs a 256-byte aligned workspace).
        size_t generic = 0;
        const int metrics[2] = {ZCGVS_METRIC_DOT, ZCGVS_METRIC_L2};
        for (const int metric : metrics) {
            for (const bool aligned : {true, false}) {
                for (const bool has_mask : {true, false}) {
                    zc::ScanPlan plan;
                    if (zc::make_plan(dtype, doc_count, dim, batch, std::min(k, ZCGVS_MAX_K), metric, false, aligned,
                                      has_mask, plan) == ZCGVS_OK) {
                        generic = std::max(generic, plan.ws_total);
                    }
                }
            }
        }
        zc::ok();
        return std::max(generic, gemm);
    }
    // The plan may differ with the corpus alignment (bulk-copy vs plain staging) and the
    // metric, so report the largest workspace any of them needs.
    size_t bytes = 0;
    const int metrics[2] = {ZCGVS_METRIC_DOT, ZCGVS_METRIC_L2};
    for (const int metric : metrics) {
        for (const bool aligned : {true, false}) {
            for (const bool has_mask : {true, false}) {
                zc::ScanPlan plan;
                if (zc::make_plan(dtype, doc_count, dim, batch, std::min(k, ZCGVS_MAX_K), metric,
                                  false, aligned, has_mask, plan) == ZCGVS_OK) {
                    bytes = std::max(bytes, plan.ws_total);
                }
            }
        }
    }
    zc::ok();
    return bytes;
}

}  // extern "C"

namespace zc {
namespace {

// Lexical inputs of a hybrid search (nullptr = dense only).
struct HybridArgs {
    const float* lex = nullptr;
    const float* lex_part = nullptr;
    int lex_parts = 0;
    float dense_weight = 1.0f;
};

// Validation shared by the dense and hybrid entry points; fills the plan.
int validate_scan(const void* corpus, int dtype, const float* row_scales, int64_t doc_count, int dim,
                  const float* queries, int batch, const uint8_t* mask, int metric, int k, int id_base,
                  int* out_indices, float* out_scores, ScanPlan& plan) {
    if (k <= 0) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs: k must be positive");
    if (k > ZCGVS_MAX_K) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs: k=" + std::to_string(k) + " exceeds kernel capacity " +
                                               std::to_string(ZCGVS_MAX_K));
    }
    if (doc_count > INT_MAX) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs: corpus exceeds the supported document count");
    }
    if (k > doc_count) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs: k=" + std::to_string(k) + " exceeds corpus size " +
                                               std::to_string(doc_count));
    }
    if (id_base < 0 || static_cast<long long>(id_base) + doc_count - 1 > INT_MAX) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs: id_base + doc_count exceeds the int32 id range");
    }
    if (corpus == nullptr || queries == nullptr || out_indices == nullptr || out_scores == nullptr) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs: null corpus, query or output pointer");
    }
    if (dtype == ZCGVS_DTYPE_I8_ROW && row_scales == nullptr) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs: the per-row int8 store needs row_scales");
    }
    int status = check_alignment(dtype, corpus, row_scales, queries, out_indices, out_scores);
    if (status != ZCGVS_OK) return status;
    return make_plan(dtype, doc_count, dim, batch, k, metric, false, aligned16(corpus), mask != nullptr, plan);
}

int run_scan_topk(const ScanPlan& plan, const void* corpus, float scale, const float* row_scales,
                  int64_t doc_count, int dim, const float* queries, int batch, const uint8_t* mask, int k,
                  int id_base, int* out_indices, float* out_scores, uint8_t* ws, const HybridArgs& hy,
                  cudaStream_t stream) {
    ScanParams params{};
    params.corpus = static_cast<const uint8_t*>(corpus);
    params.row_scales = row_scales;
    params.scale = scale;
    params.n = doc_count;
    params.dim = dim;
    params.queries = queries;
    params.query_packed = 0;
    params.batch = batch;
    params.mask = mask;
    params.k = k;
    params.id_base = static_cast<unsigned int>(id_base);
    params.status = reinterpret_cast<unsigned int*>(ws);
    params.counters = reinterpret_cast<unsigned int*>(ws + 16);
    params.lists = reinterpret_cast<unsigned long long*>(ws + plan.ws_header);
    params.spill = reinterpret_cast<unsigned long long*>(ws + plan.ws_header + plan.ws_lists);
    params.out_idx = out_indices;
    params.out_scores = out_scores;
    params.out_matrix = nullptr;
    params.lex = hy.lex;
    params.lex_part = hy.lex_part;
    params.lex_parts = hy.lex_parts;
    params.dense_weight = hy.dense_weight;
    return launch(plan, params, stream);
}

// Hybrid workspace: the scan's, then lexical scores [batch][n], then the lexical kernel's
// partial maxima, then for one query the dense scores [n] of the hybrid scan, the select
// kernel's global candidates (k per CTA, one CTA per SM) and its cross-CTA state.
struct HybridLayout {
    size_t scan = 0, lex = 0, part = 0, dense = 0, select = 0, state = 0, total = 0;
    int parts = 0;
    int select_ctas = 0;
};

HybridLayout hybrid_layout(size_t scan_ws, long long n, int batch, int k) {
    HybridLayout h;
    h.parts = lexical_parts(n);
    const int sms = device_sm_count();
    h.scan = round_up(scan_ws, kWorkspaceAlign);
    h.lex = round_up(static_cast<size_t>(batch) * static_cast<size_t>(n) * 4, kWorkspaceAlign);
    h.part = round_up(static_cast<size_t>(batch) * h.parts * 4, kWorkspaceAlign);
    if (batch == 1) {
        h.dense = round_up(static_cast<size_t>(n) * 4, kWorkspaceAlign);
        h.select_ctas = static_cast<int>(std::min<long long>(sms, (n + 3) / 4));
        h.select = round_up(static_cast<size_t>(h.select_ctas) * static_cast<size_t>(k) * 8, kWorkspaceAlign);
        h.state = round_up(sizeof(HybridSelectState), kWorkspaceAlign);
    }
    h.total = h.scan + h.lex + h.part + h.dense + h.select + h.state;
    return h;
}

// Shared-memory layout of the hybrid scan with lexical warps (scan_fast_kernel<MODE, JC, true>):
// the stage ring, the query, the CTA's BM25 accumulator, the ring's barriers.
struct FusedPlan {
    int stages = 0;
    int query_off = 0;
    int lex_off = 0;
    int bar_off = 0;
    int smem = 0;
    int lex_window = 0;
};

// The hybrid scan runs one query on the single-query fast-path tiles (bulk copies), with an
// index whose postings are sorted and 16-byte aligned. Its BM25 accumulator covers the CTA's
// documents in as few windows as keep the stage ring as deep as it would be without it (at most
// four stages: a shallower ring costs the dense stream more than a second window of posting
// searches costs the lexical warps). Otherwise the lexical kernel and the blending scan run one
// after the other.
bool plan_fused(const ScanPlan& plan, long long n, int batch, int k, const LexIndex& lexi, FusedPlan& f) {
    if (batch != 1 || plan.jc == 0 || !plan.use_tma || !lexi.vec || k > kSelCap - 64) return false;
    if (scan_lookup_fused(plan.mode, plan.jc) == nullptr) return false;
    const long long per_cta = (plan.ntiles + plan.grid_rows - 1) / plan.grid_rows * plan.rows_per_tile;
    const long long span = std::min(per_cta, n);
    const long long query = static_cast<long long>(round_up(static_cast<size_t>(plan.query_bytes), 128));
    // The kernel's static shared memory (slot bounds, reductions) stays under 4 KB.
    const long long budget = device_max_smem() - 4096;
    const long long base = query + 2 * kMaxStages * 8 + 128;
    auto stages_with = [&](long long lex_bytes) {
        return base + lex_bytes >= budget ? 0LL
                                          : std::min<long long>(kMaxStages, (budget - base - lex_bytes) / plan.stage_bytes);
    };
    const long long wanted = std::min<long long>(4, stages_with(0));
    long long window = 0, lex_bytes = 0, stages = 0;
    for (int windows = 1; windows <= 8; ++windows) {
        window = (span + windows - 1) / windows;
        lex_bytes = static_cast<long long>(round_up(static_cast<size_t>(window) * 4, 128));
        stages = stages_with(lex_bytes);
        if (stages >= wanted) break;
    }
    if (stages < 2) return false;
    f.stages = static_cast<int>(stages);
    f.lex_window = static_cast<int>(window);
    f.query_off = static_cast<int>(round_up(static_cast<size_t>(stages * plan.stage_bytes), 128));
    f.lex_off = f.query_off + static_cast<int>(query);
    f.bar_off = f.lex_off + static_cast<int>(lex_bytes);
    f.smem = f.bar_off + 2 * kMaxStages * 8;
    return f.smem <= budget;
}

// One query: the hybrid scan writes the dense scores, the lexical scores and one lexical
// maximum per CTA; the select kernel (a programmatic dependent launch) blends and selects.
int run_hybrid_fused(const ScanPlan& plan, const FusedPlan& f, const HybridLayout& h, const LexIndex& lexi,
                     const void* corpus, float scale, const float* row_scales, int64_t doc_count, int dim,
                     const float* queries, const uint8_t* mask, const int* query_terms, int term_stride,
                     float dense_weight, int k, int* out_indices, float* out_scores, uint8_t* ws,
                     cudaStream_t stream) {
    const ScanKernelFn kernel = scan_lookup_fused(plan.mode, plan.jc);
    cudaError_t status = ensure_smem_optin(reinterpret_cast<const void*>(kernel));
    if (status != cudaSuccess) return fail_cuda(status, "cudaFuncSetAttribute(scan_fast_kernel<lexical>)");
    float* lex = reinterpret_cast<float*>(ws + h.scan);
    float* dense = reinterpret_cast<float*>(ws + h.scan + h.lex + h.part);
    unsigned long long* select_cand = reinterpret_cast<unsigned long long*>(ws + h.scan + h.lex + h.part + h.dense);
    HybridSelectState* state =
        reinterpret_cast<HybridSelectState*>(ws + h.scan + h.lex + h.part + h.dense + h.select);
    unsigned int* counters = reinterpret_cast<unsigned int*>(ws + 16);
    unsigned long long* lists = reinterpret_cast<unsigned long long*>(ws + plan.ws_header);
    ScanParams params{};
    params.corpus = static_cast<const uint8_t*>(corpus);
    params.row_scales = row_scales;
    params.scale = scale;
    params.n = doc_count;
    params.dim = dim;
    params.queries = queries;
    params.batch = 1;
    params.mask = mask;
    params.k = k;
    params.status = reinterpret_cast<unsigned int*>(ws);
    params.counters = counters;
    params.lists = lists;
    params.out_idx = out_indices;
    params.out_scores = out_scores;
    params.out_matrix = dense;
    params.lexi = lexi;
    params.lex_terms = query_terms;
    params.lex_stride = term_stride;
    params.lex_out = lex;
    params.lex_peak = &state->peak;
    fill_params(plan, params);
    params.stages = f.stages;
    params.spill_stride = 0;
    params.smem_query_off = f.query_off;
    params.smem_topk_off = 0;
    params.smem_bar_off = f.bar_off;
    params.smem_lex_off = f.lex_off;
    params.lex_window = f.lex_window;
    const dim3 grid(1u, static_cast<unsigned>(plan.grid_rows));
    {
        KernelTimer timer("scan", stream);
        kernel<<<grid, kFusedThreads, f.smem, stream>>>(params);
    }
    status = cudaGetLastError();
    if (status != cudaSuccess) return fail_cuda(status, "scan_fast_kernel<lexical> launch");
    return launch_hybrid_select(dense, lex, state, dense_weight, doc_count, k, 0u, select_cand, out_indices,
                                out_scores, h.select_ctas, stream);
}

}  // namespace
}  // namespace zc

extern "C" {

int zcgvs_scan_topk(const void* corpus, int dtype, float scale, const float* row_scales,
                    int64_t doc_count, int dim, const float* queries, int batch,
                    const uint8_t* mask, int metric, int k, int id_base, int* out_indices,
                    float* out_scores, void* workspace, size_t workspace_bytes, void* stream) {
    using namespace zc;
    if (doc_count <= 0 || batch <= 0 || dim <= 0) return ok();
    ScanPlan plan;
    int status = validate_scan(corpus, dtype, row_scales, doc_count, dim, queries, batch, mask, metric, k, id_base,
                               out_indices, out_scores, plan);
    if (status != ZCGVS_OK) return status;
    if (workspace == nullptr || workspace_bytes < plan.ws_total) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs: workspace smaller than zcgvs_scan_topk_workspace_bytes()");
    }
    if (!aligned16(workspace)) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs: workspace must be 16-byte aligned");
    if (gemm_eligible(dtype, doc_count, dim, batch, metric) && (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0 &&
        (reinterpret_cast<uintptr_t>(corpus) & 15u) == 0 &&
        workspace_bytes >= zcgvs_gemm_topk_workspace_bytes(dtype, doc_count, dim, batch, k)) {
        return zcgvs_gemm_topk(corpus, dtype, row_scales, doc_count, dim, queries, batch, mask, metric, k, id_base,
                               out_indices, out_scores, workspace, workspace_bytes, stream);
    }
    return run_scan_topk(plan, corpus, scale, row_scales, doc_count, dim, queries, batch, mask, k, id_base,
                         out_indices, out_scores, static_cast<uint8_t*>(workspace), HybridArgs{},
                         static_cast<cudaStream_t>(stream));
}

size_t zcgvs_hybrid_topk_workspace_bytes(int dtype, int64_t doc_count, int dim, int batch, int k) {
    if (doc_count <= 0 || dim <= 0 || batch <= 0 || k <= 0) return 0;
    const size_t scan = zcgvs_scan_topk_workspace_bytes(dtype, doc_count, dim, batch, k);
    return zc::hybrid_layout(scan, doc_count, batch, k).total;
}

int zcgvs_hybrid_topk(const void* corpus, int dtype, float scale, const float* row_scales, int64_t doc_count,
                      int dim, const float* queries, int batch, const uint8_t* mask, int metric,
                      const int64_t* offsets, const int* posting_docs, const float* posting_weights, int vocab_size,
                      const int* query_terms, int term_stride, float dense_weight, int k, int* out_indices,
                      float* out_scores, void* workspace, size_t workspace_bytes, void* stream) {
    using namespace zc;
    if (doc_count <= 0 || batch <= 0 || dim <= 0) return ok();
    ScanPlan plan;
    int status = validate_scan(corpus, dtype, row_scales, doc_count, dim, queries, batch, mask, metric, k, 0,
                               out_indices, out_scores, plan);
    if (status != ZCGVS_OK) return status;
    const bool lexical = term_stride > 0 && query_terms != nullptr;
    if (lexical && (offsets == nullptr || posting_docs == nullptr || posting_weights == nullptr || vocab_size <= 0)) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_hybrid_topk: null or empty lexical index");
    }
    const HybridLayout h = hybrid_layout(zcgvs_scan_topk_workspace_bytes(dtype, doc_count, dim, batch, k),
                                         doc_count, batch, k);
    if (workspace == nullptr || workspace_bytes < h.total) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs: workspace smaller than zcgvs_hybrid_topk_workspace_bytes()");
    }
    if (!aligned16(workspace)) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs: workspace must be 16-byte aligned");
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (lexical) {
        const LexIndex lexi = lex_index(reinterpret_cast<const long long*>(offsets), posting_docs, posting_weights,
                                        vocab_size, doc_count, true);
        FusedPlan f;
        if (plan_fused(plan, doc_count, batch, k, lexi, f)) {
            return run_hybrid_fused(plan, f, h, lexi, corpus, scale, row_scales, doc_count, dim, queries, mask,
                                    query_terms, term_stride, dense_weight, k, out_indices, out_scores, ws, st);
        }
    }
    HybridArgs hy;
    if (lexical) {
        hy.lex = reinterpret_cast<float*>(ws + h.scan);
        hy.lex_part = reinterpret_cast<float*>(ws + h.scan + h.lex);
        hy.lex_parts = h.parts;
        hy.dense_weight = dense_weight;
        status = launch_lexical(reinterpret_cast<const long long*>(offsets), posting_docs, posting_weights, vocab_size,
                                query_terms, term_stride, doc_count, batch, nullptr, reinterpret_cast<float*>(ws + h.scan),
                                reinterpret_cast<float*>(ws + h.scan + h.lex), true, st);
        if (status != ZCGVS_OK) return status;
    }
    return run_scan_topk(plan, corpus, scale, row_scales, doc_count, dim, queries, batch, mask, k, 0, out_indices,
                         out_scores, ws, hy, st);
}

int zcgvs_similarity(const void* corpus, int dtype, float scale, const float* row_scales,
                     int64_t doc_count, int dim, const void* queries, int batch,
                     const uint8_t* mask, int metric, float* scores, void* stream) {
    using namespace zc;
    if (doc_count <= 0 || batch <= 0 || dim <= 0) return ok();
    if (doc_count > INT_MAX) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs: corpus exceeds the supported document count");
    }
    if (corpus == nullptr || queries == nullptr || scores == nullptr) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs: null corpus, query or score pointer");
    }
    if (dtype == ZCGVS_DTYPE_I8_ROW && row_scales == nullptr) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs: the per-row int8 store needs row_scales");
    }
    int status = check_alignment(dtype, corpus, row_scales, queries, scores, nullptr);
    if (status != ZCGVS_OK) return status;
    ScanPlan plan;
    status = make_plan(dtype, doc_count, dim, batch, 1, metric, true, aligned16(corpus),
                       mask != nullptr, plan);
    if (status != ZCGVS_OK) return status;
    ScanParams params{};
    params.corpus = static_cast<const uint8_t*>(corpus);
    params.row_scales = row_scales;
    params.scale = scale;
    params.n = doc_count;
    params.dim = dim;
    params.queries = queries;
    params.query_packed = (dtype == ZCGVS_DTYPE_BINARY) ? 1 : 0;
    params.batch = batch;
    params.mask = mask;
    params.k = 1;
    params.out_matrix = scores;
    return launch(plan, params, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
