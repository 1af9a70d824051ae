// Row-sharded search across the GPUs of one node over NCCL (zcgvs_sharded_* in zcgvs_sm100.h).
//
// One process per GPU. Rank r holds rows [begin, end) of the corpus (the even split of
// zcgvs_shard_bounds) and runs, per search, on its own stream:
//
//   dense   : local fused search with id_base = begin        -> send  [2, B, k] (ids, score bits)
//             ncclAllGather(send -> recv [P, 2, B, k])
//             zcgvs_merge_topk_lists(recv)                     -> out [B, k] (global top-k)
//   rescore : local coarse search with id_base = begin       -> send  [2, B, M]
//             ncclAllGather(send -> recv [P, 2, B, M])
//             zcgvs_merge_topk_lists(recv, owned rows)         -> owned [B, M] (shard-local ids, -1
//                                                                 for candidates of other shards)
//             zcgvs_rescore_topk(store shard, owned)           -> send2 [2, B, K] (shard-local ids)
//             ncclAllGather(send2 -> recv2 [P, 2, B, K])
//             zcgvs_merge_topk_lists(recv2, + shard begins)    -> out [B, K] (global ids)
//
// Each step equals the one-GPU pipeline: the union of per-shard top lists contains the global
// ones and (score desc, id asc) is a total order. The exchanges are a few hundred KB at most, so
// one library all-gather each is the right tool (there is no compute step to fuse with).
//
// NCCL is resolved at run time (dlopen of libnccl.so.2), so the library loads and its other
// entry points work where NCCL is absent. With ZCGVS_SHARDED_GRAPH a search whose arguments
// match the cached graph's replays it; otherwise it runs its launches directly (establishing
// NCCL's connections on first use) and then captures the same launches into a graph for next
// time. The graph key is the list of every argument the launches take, buffers included.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <climits>
#include <cstring>
#include <string>
#include <vector>

#include "host_common.h"
#include "zcgvs_sm100.h"

namespace zc {
namespace {

// The NCCL entry points this file calls, resolved once.
struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclCommAbort) comm_abort = nullptr;
    decltype(&ncclCommGetAsyncError) async_error = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    std::string missing;  // why NCCL could not be used ("" when it can)
};

template <typename Fn>
void resolve(void* handle, const char* name, Fn& fn, std::string& missing) {
    fn = reinterpret_cast<Fn>(dlsym(handle, name));
    if (fn == nullptr && missing.empty()) missing = std::string("libnccl.so.2 lacks ") + name;
}

const NcclApi& nccl() {
    static const NcclApi api = [] {
        NcclApi a;
        void* handle = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (handle == nullptr) {
            const char* why = dlerror();
            a.missing = std::string("cannot load libnccl.so.2: ") + (why != nullptr ? why : "unknown error");
            return a;
        }
        resolve(handle, "ncclGetUniqueId", a.get_unique_id, a.missing);
        resolve(handle, "ncclCommInitRank", a.comm_init_rank, a.missing);
        resolve(handle, "ncclCommDestroy", a.comm_destroy, a.missing);
        resolve(handle, "ncclCommAbort", a.comm_abort, a.missing);
        resolve(handle, "ncclCommGetAsyncError", a.async_error, a.missing);
        resolve(handle, "ncclAllGather", a.all_gather, a.missing);
        resolve(handle, "ncclGetErrorString", a.error_string, a.missing);
        return a;
    }();
    return api;
}

int fail_nccl(ncclResult_t result, const char* what) {
    const char* text = nccl().error_string != nullptr ? nccl().error_string(result) : "unknown";
    return fail(ZCGVS_ERR_COMM, std::string(what) + " failed: " + text + " (" + std::to_string(static_cast<int>(result)) + ")");
}

int need_nccl() {
    return nccl().missing.empty() ? ZCGVS_OK : fail(ZCGVS_ERR_COMM, "zcgvs sharded search: " + nccl().missing);
}

void split(long long total, int world, int rank, long long* begin, long long* end) {
    const long long base = total / world, extra = total % world;
    *begin = rank * base + std::min<long long>(rank, extra);
    *end = *begin + base + (rank < extra ? 1 : 0);
}

// A device allocation that only grows. grow() returns true when it reallocated.
struct DeviceBytes {
    void* ptr = nullptr;
    size_t bytes = 0;
    ~DeviceBytes() {
        if (ptr != nullptr) cudaFree(ptr);
    }
    int grow(size_t need, bool* grown) {
        *grown = false;
        if (need <= bytes) return ZCGVS_OK;
        if (ptr != nullptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
        const cudaError_t e = cudaMalloc(&ptr, need);
        if (e != cudaSuccess) return fail_cuda(e, "zcgvs sharded search: cudaMalloc");
        bytes = need;
        *grown = true;
        return ZCGVS_OK;
    }
    int* i32() const { return static_cast<int*>(ptr); }
};

}  // namespace
}  // namespace zc

struct zcgvs_sharded {
    int world = 0;
    int rank = 0;
    int device = 0;
    long long total = 0, begin = 0, end = 0;
    ncclComm_t comm = nullptr;
    zc::DeviceBytes shard_begins;  // [world] int32: every shard's first row (global id offsets)
    zc::DeviceBytes workspace;     // the local search's workspace (its first 4 bytes: status word)
    zc::DeviceBytes send, recv, owned, send2, recv2;
    unsigned long long generation = 0;  // bumped whenever a buffer is reallocated
    cudaStream_t capture_stream = nullptr;  // graphs are captured here (the caller's stream may be
                                            // the legacy default stream, which cannot capture)
    cudaGraphExec_t graph = nullptr;
    std::vector<long long> graph_key;
};

namespace zc {
namespace {

// Everything one search's launches take: the graph key, and the recording of the step.
struct Step {
    bool rescore = false;
    bool f16_tensor = false;
    const void* corpus = nullptr;  // dense corpus or coarse codes
    int dtype = 0;
    float scale = 1.0f;
    const float* row_scales = nullptr;
    const void* store = nullptr;  // rescore store
    int store_dtype = 0;
    float store_scale = 1.0f;
    const float* store_row_scales = nullptr;
    long long rows = 0;
    int dim = 0;
    const float* queries = nullptr;
    int batch = 0;
    const uint8_t* mask = nullptr;
    int metric = 0;
    int width = 0;  // k of the local search (M for the rescore search)
    int k = 0;
    int* out_indices = nullptr;
    float* out_scores = nullptr;

    std::vector<long long> key(const zcgvs_sharded& s) const {
        auto ptr = [](const void* p) { return static_cast<long long>(reinterpret_cast<uintptr_t>(p)); };
        long long scale_bits = 0, store_scale_bits = 0;
        std::memcpy(&scale_bits, &scale, sizeof(float));
        std::memcpy(&store_scale_bits, &store_scale, sizeof(float));
        return {rescore,    f16_tensor, ptr(corpus),           dtype,       scale_bits,       ptr(row_scales),
                ptr(store), store_dtype, store_scale_bits,     ptr(store_row_scales), rows, dim,
                ptr(queries), batch,     ptr(mask),            metric,      width,            k,
                ptr(out_indices), ptr(out_scores), static_cast<long long>(s.generation)};
    }
};

int all_gather(const zcgvs_sharded& s, const void* send, void* recv, size_t count, cudaStream_t st) {
    KernelTimer timer("allgather", st);
    const ncclResult_t r = nccl().all_gather(send, recv, count, ncclInt32, s.comm, st);
    return r == ncclSuccess ? ZCGVS_OK : fail_nccl(r, "ncclAllGather");
}

// The launches of one search on `st` (direct, or under stream capture).
int record(zcgvs_sharded& s, const Step& p, cudaStream_t st) {
    const size_t block = static_cast<size_t>(p.batch) * p.width;  // one [B, width] list
    int* send = s.send.i32();
    int* recv = s.recv.i32();
    int status;
    if (p.f16_tensor) {
        status = zcgvs_gemm_topk(p.corpus, p.dtype, p.row_scales, p.rows, p.dim, p.queries, p.batch, p.mask, p.metric,
                                 p.width, static_cast<int>(s.begin), send, reinterpret_cast<float*>(send + block),
                                 s.workspace.ptr, s.workspace.bytes, st);
    } else {
        status = zcgvs_scan_topk(p.corpus, p.dtype, p.scale, p.row_scales, p.rows, p.dim, p.queries, p.batch, p.mask,
                                 p.metric, p.width, static_cast<int>(s.begin), send,
                                 reinterpret_cast<float*>(send + block), s.workspace.ptr, s.workspace.bytes, st);
    }
    if (status != ZCGVS_OK) return status;
    status = all_gather(s, send, recv, 2 * block, st);
    if (status != ZCGVS_OK) return status;
    if (!p.rescore) {
        return zcgvs_merge_topk_lists(recv, reinterpret_cast<const float*>(recv + block), static_cast<int64_t>(2 * block),
                                      s.world, p.batch, p.width, nullptr, p.k, p.out_indices, p.out_scores, 0, 0,
                                      nullptr, st);
    }
    int* owned = s.owned.i32();
    status = zcgvs_merge_topk_lists(recv, reinterpret_cast<const float*>(recv + block), static_cast<int64_t>(2 * block),
                                    s.world, p.batch, p.width, nullptr, p.width, nullptr, nullptr,
                                    static_cast<int>(s.begin), static_cast<int>(s.end), owned, st);
    if (status != ZCGVS_OK) return status;
    const size_t block2 = static_cast<size_t>(p.batch) * p.k;
    int* send2 = s.send2.i32();
    int* recv2 = s.recv2.i32();
    status = zcgvs_rescore_topk(p.store, p.store_dtype, p.store_scale, p.store_row_scales, p.rows, p.dim, p.queries,
                                p.batch, owned, p.width, p.metric, p.k, send2, reinterpret_cast<float*>(send2 + block2),
                                st);
    if (status != ZCGVS_OK) return status;
    status = all_gather(s, send2, recv2, 2 * block2, st);
    if (status != ZCGVS_OK) return status;
    return zcgvs_merge_topk_lists(recv2, reinterpret_cast<const float*>(recv2 + block2), static_cast<int64_t>(2 * block2),
                                  s.world, p.batch, p.k, s.shard_begins.i32(), p.k, p.out_indices, p.out_scores, 0, 0,
                                  nullptr, st);
}

// Sizes the buffers for `p` (reallocating, and zero-filling the workspace, when they grow).
int prepare(zcgvs_sharded& s, const Step& p) {
    size_t ws = p.f16_tensor ? zcgvs_gemm_topk_workspace_bytes(p.dtype, p.rows, p.dim, p.batch, p.width)
                             : zcgvs_scan_topk_workspace_bytes(p.dtype, p.rows, p.dim, p.batch, p.width);
    if (ws == 0) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs sharded search: no workspace size for these arguments");
    ws = round_up(std::max<size_t>(ws, 256), 256);
    const size_t block = static_cast<size_t>(p.batch) * p.width * 4;
    const size_t block2 = static_cast<size_t>(p.batch) * p.k * 4;
    bool grown = false, any = false;
    struct Need {
        DeviceBytes* buf;
        size_t bytes;
    } needs[] = {{&s.workspace, ws},
                 {&s.send, 2 * block},
                 {&s.recv, 2 * block * s.world},
                 {&s.owned, p.rescore ? block : 0},
                 {&s.send2, p.rescore ? 2 * block2 : 0},
                 {&s.recv2, p.rescore ? 2 * block2 * s.world : 0}};
    for (const Need& n : needs) {
        if (n.bytes == 0) continue;
        const int status = n.buf->grow(n.bytes, &grown);
        if (status != ZCGVS_OK) return status;
        if (grown && n.buf == &s.workspace) {
            const cudaError_t e = cudaMemset(s.workspace.ptr, 0, s.workspace.bytes);  // counters start at zero once
            if (e != cudaSuccess) return fail_cuda(e, "zcgvs sharded search: zero-filling the workspace");
        }
        any |= grown;
    }
    if (any) ++s.generation;
    return ZCGVS_OK;
}

void drop_graph(zcgvs_sharded& s) {
    if (s.graph != nullptr) cudaGraphExecDestroy(s.graph);
    s.graph = nullptr;
    s.graph_key.clear();
}

int run(zcgvs_sharded& s, const Step& p, unsigned flags, cudaStream_t st) {
    int status = prepare(s, p);
    if (status != ZCGVS_OK) return status;
    if ((flags & ZCGVS_SHARDED_GRAPH) == 0u) return record(s, p, st);
    std::vector<long long> key = p.key(s);
    if (s.graph != nullptr && key == s.graph_key) {
        const cudaError_t e = cudaGraphLaunch(s.graph, st);
        return e == cudaSuccess ? ok() : fail_cuda(e, "zcgvs sharded search: cudaGraphLaunch");
    }
    // First search of this shape: run it on the caller's stream, then capture the same launches
    // on the handle's own stream (capturing executes nothing) for the next ones, which launch the
    // graph on the caller's stream.
    status = record(s, p, st);
    if (status != ZCGVS_OK) return status;
    drop_graph(s);
    cudaError_t e = cudaStreamBeginCapture(s.capture_stream, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return fail_cuda(e, "zcgvs sharded search: cudaStreamBeginCapture");
    status = record(s, p, s.capture_stream);
    cudaGraph_t graph = nullptr;
    e = cudaStreamEndCapture(s.capture_stream, &graph);
    if (status != ZCGVS_OK) {
        if (graph != nullptr) cudaGraphDestroy(graph);
        return status;
    }
    if (e != cudaSuccess) return fail_cuda(e, "zcgvs sharded search: cudaStreamEndCapture");
    e = cudaGraphInstantiateWithFlags(&s.graph, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) {
        s.graph = nullptr;
        return fail_cuda(e, "zcgvs sharded search: cudaGraphInstantiate");
    }
    s.graph_key = std::move(key);
    return ok();
}

int check_handle(const zcgvs_sharded* s, long long rows, int dim, const float* queries, int batch) {
    if (s == nullptr) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs sharded search: null handle");
    if (rows != s->end - s->begin) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs sharded search: shard_rows " + std::to_string(rows) +
                                               " differs from this rank's shard [" + std::to_string(s->begin) + ", " +
                                               std::to_string(s->end) + ")");
    }
    if (dim <= 0 || batch <= 0 || queries == nullptr) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs sharded search: needs queries, dim > 0 and batch > 0");
    }
    int device = 0;
    if (cudaGetDevice(&device) == cudaSuccess && device != s->device) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs sharded search: the current device is not the handle's");
    }
    return ZCGVS_OK;
}

}  // namespace
}  // namespace zc

extern "C" {

int zcgvs_shard_bounds(int64_t total_rows, int world, int rank, int64_t* begin, int64_t* end) {
    if (total_rows < 0 || world <= 0 || rank < 0 || rank >= world || begin == nullptr || end == nullptr) {
        return zc::fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_shard_bounds: needs total_rows >= 0 and 0 <= rank < world");
    }
    long long b = 0, e = 0;
    zc::split(total_rows, world, rank, &b, &e);
    *begin = b;
    *end = e;
    return zc::ok();
}

size_t zcgvs_nccl_id_bytes(void) { return sizeof(ncclUniqueId); }

int zcgvs_nccl_unique_id(void* id) {
    if (id == nullptr) return zc::fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_nccl_unique_id: null id buffer");
    int status = zc::need_nccl();
    if (status != ZCGVS_OK) return status;
    const ncclResult_t r = zc::nccl().get_unique_id(static_cast<ncclUniqueId*>(id));
    return r == ncclSuccess ? zc::ok() : zc::fail_nccl(r, "ncclGetUniqueId");
}

int zcgvs_sharded_create(const void* nccl_id, int world, int rank, int64_t total_rows, zcgvs_sharded** out) {
    if (nccl_id == nullptr || out == nullptr || world <= 0 || rank < 0 || rank >= world || total_rows < world ||
        total_rows > INT_MAX) {
        return zc::fail(ZCGVS_ERR_INVALID_ARG,
                        "zcgvs_sharded_create: needs an id, 0 <= rank < world and world <= total_rows <= INT_MAX");
    }
    *out = nullptr;
    int status = zc::need_nccl();
    if (status != ZCGVS_OK) return status;
    auto* s = new zcgvs_sharded();
    s->world = world;
    s->rank = rank;
    s->total = total_rows;
    zc::split(total_rows, world, rank, &s->begin, &s->end);
    cudaError_t e = cudaGetDevice(&s->device);
    if (e != cudaSuccess) {
        delete s;
        return zc::fail_cuda(e, "zcgvs_sharded_create: cudaGetDevice");
    }
    e = cudaStreamCreateWithFlags(&s->capture_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete s;
        return zc::fail_cuda(e, "zcgvs_sharded_create: cudaStreamCreateWithFlags");
    }
    ncclUniqueId id;
    std::memcpy(&id, nccl_id, sizeof(id));
    const ncclResult_t r = zc::nccl().comm_init_rank(&s->comm, world, id, rank);
    if (r != ncclSuccess) {
        s->comm = nullptr;
        zcgvs_sharded_destroy(s);
        return zc::fail_nccl(r, "ncclCommInitRank");
    }
    std::vector<int> begins(static_cast<size_t>(world));
    for (int p = 0; p < world; ++p) {
        long long b = 0, end = 0;
        zc::split(total_rows, world, p, &b, &end);
        begins[static_cast<size_t>(p)] = static_cast<int>(b);
    }
    bool grown = false;
    status = s->shard_begins.grow(begins.size() * sizeof(int), &grown);
    if (status == ZCGVS_OK) {
        e = cudaMemcpy(s->shard_begins.ptr, begins.data(), begins.size() * sizeof(int), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) status = zc::fail_cuda(e, "zcgvs_sharded_create: copying the shard offsets");
    }
    if (status != ZCGVS_OK) {
        zcgvs_sharded_destroy(s);
        return status;
    }
    *out = s;
    return zc::ok();
}

int zcgvs_sharded_destroy(zcgvs_sharded* s) {
    if (s == nullptr) return zc::ok();
    zc::drop_graph(*s);  // before the communicator its collectives use
    if (s->comm != nullptr) {
        ncclResult_t async = ncclSuccess;
        zc::nccl().async_error(s->comm, &async);
        if (async != ncclSuccess) {
            zc::nccl().comm_abort(s->comm);
        } else {
            zc::nccl().comm_destroy(s->comm);
        }
    }
    if (s->capture_stream != nullptr) cudaStreamDestroy(s->capture_stream);
    delete s;
    return zc::ok();
}

int zcgvs_sharded_search(zcgvs_sharded* s, const void* shard, int dtype, float scale, const float* row_scales,
                         int64_t shard_rows, int dim, const float* queries, int batch, const uint8_t* mask, int metric,
                         int k, unsigned flags, int* out_indices, float* out_scores, void* stream) {
    int status = zc::check_handle(s, shard_rows, dim, queries, batch);
    if (status != ZCGVS_OK) return status;
    if (k <= 0 || k > ZCGVS_MAX_K || k > shard_rows) {
        return zc::fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_sharded_search: k must be in [1, min(" +
                                                   std::to_string(ZCGVS_MAX_K) + ", rows per shard = " +
                                                   std::to_string(shard_rows) + ")]");
    }
    if (static_cast<long long>(k) * s->world > 16384) {
        return zc::fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_sharded_search: k * world exceeds the merge's 16384 entries");
    }
    if (shard == nullptr || out_indices == nullptr || out_scores == nullptr) {
        return zc::fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_sharded_search: null shard or output");
    }
    const bool tensor = (flags & ZCGVS_SHARDED_F16_TENSOR) != 0u;
    if (tensor && dtype != ZCGVS_DTYPE_F16) {
        return zc::fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_sharded_search: ZCGVS_SHARDED_F16_TENSOR needs an fp16 shard");
    }
    zc::Step p;
    p.f16_tensor = tensor;
    p.corpus = shard;
    p.dtype = dtype;
    p.scale = scale;
    p.row_scales = row_scales;
    p.rows = shard_rows;
    p.dim = dim;
    p.queries = queries;
    p.batch = batch;
    p.mask = mask;
    p.metric = metric;
    p.width = k;
    p.k = k;
    p.out_indices = out_indices;
    p.out_scores = out_scores;
    return zc::run(*s, p, flags, static_cast<cudaStream_t>(stream));
}

int zcgvs_sharded_rescore_search(zcgvs_sharded* s, const void* codes, int code_dtype, float code_scale,
                                 const float* code_row_scales, const void* store, int store_dtype, float store_scale,
                                 const float* store_row_scales, int64_t shard_rows, int dim, const float* queries,
                                 int batch, int metric, int candidates, int k, unsigned flags, int* out_indices,
                                 float* out_scores, void* stream) {
    int status = zc::check_handle(s, shard_rows, dim, queries, batch);
    if (status != ZCGVS_OK) return status;
    if (k <= 0 || candidates < k || candidates > ZCGVS_MAX_K || candidates > shard_rows) {
        return zc::fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_sharded_rescore_search: needs 0 < k <= candidates <= min(" +
                                                   std::to_string(ZCGVS_MAX_K) + ", rows per shard = " +
                                                   std::to_string(shard_rows) + ")");
    }
    if (static_cast<long long>(candidates) * s->world > 16384) {
        return zc::fail(ZCGVS_ERR_INVALID_ARG,
                        "zcgvs_sharded_rescore_search: candidates * world exceeds the merge's 16384 entries");
    }
    if (codes == nullptr || store == nullptr || out_indices == nullptr || out_scores == nullptr) {
        return zc::fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_sharded_rescore_search: null codes, store or output");
    }
    if (store_dtype == ZCGVS_DTYPE_BINARY) {
        return zc::fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_sharded_rescore_search: the rescore store must not be binary");
    }
    if ((flags & ZCGVS_SHARDED_F16_TENSOR) != 0u) {
        return zc::fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_sharded_rescore_search: ZCGVS_SHARDED_F16_TENSOR is for dense searches");
    }
    zc::Step p;
    p.rescore = true;
    p.corpus = codes;
    p.dtype = code_dtype;
    p.scale = code_scale;
    p.row_scales = code_row_scales;
    p.store = store;
    p.store_dtype = store_dtype;
    p.store_scale = store_scale;
    p.store_row_scales = store_row_scales;
    p.rows = shard_rows;
    p.dim = dim;
    p.queries = queries;
    p.batch = batch;
    p.metric = metric;
    p.width = candidates;
    p.k = k;
    p.out_indices = out_indices;
    p.out_scores = out_scores;
    return zc::run(*s, p, flags, static_cast<cudaStream_t>(stream));
}

int zcgvs_sharded_status(zcgvs_sharded* s, uint32_t* status, int* comm_error, void* stream) {
    if (s == nullptr || status == nullptr || comm_error == nullptr) {
        return zc::fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_sharded_status: null argument");
    }
    *status = 0u;
    *comm_error = 0;
    if (s->workspace.ptr != nullptr) {
        const int rc = zcgvs_workspace_status(s->workspace.ptr, s->workspace.bytes, status, stream);
        if (rc != ZCGVS_OK) return rc;
    } else {
        const cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) return zc::fail_cuda(e, "zcgvs_sharded_status");
    }
    ncclResult_t async = ncclSuccess;
    const ncclResult_t r = zc::nccl().async_error(s->comm, &async);
    if (r != ncclSuccess) return zc::fail_nccl(r, "ncclCommGetAsyncError");
    *comm_error = static_cast<int>(async);
    return zc::ok();
}

int zcgvs_sharded_clear_status(zcgvs_sharded* s, void* stream) {
    if (s == nullptr) return zc::fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_sharded_clear_status: null handle");
    if (s->workspace.ptr == nullptr) return zc::ok();
    return zcgvs_workspace_init(s->workspace.ptr, sizeof(uint32_t), stream);
}

}  // extern "C"
