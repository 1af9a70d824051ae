// Device-side building blocks shared by every sm_100a kernel of the search path:
// selection keys, mbarrier / bulk-copy (TMA) wrappers with bounded waits, and warp reductions.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>

namespace zc {

// Storage modes of the scan kernels; the codes equal the ABI dtype codes.
enum ScanMode : int { kModeF32 = 0, kModeF16 = 1, kModeI8M = 2, kModeBin = 3, kModeI8R = 4 };

using u64 = unsigned long long;

// ---------------------------------------------------------------------------------------
// Selection keys.
//
// A candidate (score, id) is packed into one 64-bit key whose unsigned order is the search
// order: score descending, then document id ascending. The high word is the score's bits
// mapped to an order-preserving unsigned integer; the low word is the bitwise complement of
// the id, so a smaller id gives a larger key. Key 0 is reserved for "empty slot" (it would
// need a NaN score), which decodes to (-FLT_MAX, -1), the reference's padding pair
// (src/cuda/topk.cu:36-52).
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t orderable_bits(float score) {
    uint32_t u = __float_as_uint(score);
    if (u == 0x80000000u) u = 0u;  // -0.0 and +0.0 compare equal in the reference's sort
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float score_from_bits(uint32_t o) {
    const uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
    return __uint_as_float(u);
}

__device__ __forceinline__ u64 make_key(float score, uint32_t id) {
    return (static_cast<u64>(orderable_bits(score)) << 32) | static_cast<uint32_t>(~id);
}

__device__ __forceinline__ int key_id(u64 key) {
    return key == 0ull ? -1 : static_cast<int>(~static_cast<uint32_t>(key));
}

__device__ __forceinline__ float key_score(u64 key) {
    return key == 0ull ? -FLT_MAX : score_from_bits(static_cast<uint32_t>(key >> 32));
}

// ---------------------------------------------------------------------------------------
// Device status word bits (workspace header). A kernel that gives up a bounded wait records
// why here instead of hanging; the host reads it with zcgvs_workspace_status.
// ---------------------------------------------------------------------------------------
enum : uint32_t {
    kStatusTileWaitTimeout = 1u << 0,
    kStatusDrainTimeout = 1u << 1,
};

// Wall-clock budget of any single bounded wait, in nanoseconds of %globaltimer.
constexpr u64 kWaitBudgetNs = 2000000000ull;

__device__ __forceinline__ u64 global_timer_ns() {
    u64 t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------
// mbarrier + bulk async copy (the TMA engine's 1-D form). A tile of whole corpus rows is one
// contiguous byte range, so the un-tiled cp.async.bulk moves it global -> shared in a single
// instruction issued by one thread, and completion is tracked by an mbarrier transaction
// count. Every copy lands in the issuing CTA's own shared memory only.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(u64* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(u64* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_cta(u64* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar_addr), "r"(parity)
        : "memory");
    return done != 0u;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete sleeps until it
// completes or `hint_ns` passes, instead of re-issuing the test (the issue slots go to the
// other warps of its scheduler).
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar_addr, uint32_t parity, uint32_t hint_ns) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar_addr), "r"(parity), "r"(hint_ns)
        : "memory");
    return done != 0u;
}

// mbar_wait_bounded with sleeping tests (mbar_try_wait_sleep), the same budget.
__device__ __forceinline__ bool mbar_wait_sleep_bounded(u64* bar, uint32_t parity, uint32_t* status, uint32_t flag) {
    const uint32_t addr = smem_u32(bar);
    if (mbar_try_wait(addr, parity)) return true;
    const u64 start = global_timer_ns();
    for (uint32_t spin = 0; spin < (1u << 28); ++spin) {
        if (mbar_try_wait_sleep(addr, parity, 20000u)) return true;
        if ((spin & 15u) == 0u && global_timer_ns() - start > kWaitBudgetNs) break;
    }
    if (status != nullptr) atomicOr(status, flag);
    return false;
}

// Waits for phase `parity` of an mbarrier, giving up after kWaitBudgetNs. Returns false (and
// sets `flag` in the device status word) when the wait ran out.
__device__ __forceinline__ bool mbar_wait_bounded(u64* bar, uint32_t parity,
                                                  uint32_t* status, uint32_t flag) {
    const uint32_t addr = smem_u32(bar);
    if (mbar_try_wait(addr, parity)) return true;
    const u64 start = global_timer_ns();
    for (uint32_t spin = 0; spin < (1u << 28); ++spin) {
        if (mbar_try_wait(addr, parity)) return true;
        if ((spin & 255u) == 0u && global_timer_ns() - start > kWaitBudgetNs) break;
    }
    if (status != nullptr) atomicOr(status, flag);
    return false;
}

// Global -> shared bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned),
// completing on `bar` with a transaction count.
__device__ __forceinline__ void bulk_copy_g2s(void* dst_smem, const void* src_gmem,
                                              uint32_t bytes, u64* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
        "[%3];" ::"r"(smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// L2 policy for data read exactly once (the corpus stream): its lines are the first to be
// evicted, so the small data the kernel reuses (candidate lists, counters) is not pushed out
// of L2 by the hundreds of MB streaming through it. (On the 1M x 768 batch-1 scan the
// measured time is the same with and without it.)
__device__ __forceinline__ u64 l2_policy_evict_first() {
    u64 policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

__device__ __forceinline__ u64 l2_policy_evict_last() {
    u64 policy;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

// A 4-byte global store with an L2 cache policy (data the next kernel reads back soon).
__device__ __forceinline__ void st_global_hint(float* ptr, float value, u64 policy) {
    asm volatile("st.global.L2::cache_hint.f32 [%0], %1, %2;" ::"l"(ptr), "f"(value), "l"(policy) : "memory");
}

// bulk_copy_g2s with an L2 cache policy from createpolicy.
__device__ __forceinline__ void bulk_copy_g2s_hint(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                                   u64* bar, u64 policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, "
        "[%3], %4;" ::"r"(smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// ---------------------------------------------------------------------------------------
// Warp reductions.
// ---------------------------------------------------------------------------------------

// Transposing reduction of V per-lane partial sums across each aligned segment of W lanes
// (V <= W, both powers of two). Each exchange halves the values a lane holds, so reducing V
// sums costs (V - 1) + (log2 W - log2 V) shuffles instead of V log2 W. On return v[0] of lane
// l holds the full segment sum of value index (l % W) >> (log2 W - log2 V), replicated across
// W / V lanes.
template <int V, int W, typename T>
__device__ __forceinline__ void transpose_reduce(T (&v)[V], int lane) {
    static_assert(V <= W, "segment narrower than the value count");
#pragma unroll
    for (int nv = V, offset = W / 2; offset >= 1; offset >>= 1) {
        if (nv > 1) {
            const int half = nv >> 1;
            const bool upper = (lane & offset) != 0;
#pragma unroll
            for (int i = 0; i < half; ++i) {
                const T send = upper ? v[i] : v[i + half];
                const T keep = upper ? v[i + half] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, offset);
            }
            nv = half;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], offset);
        }
    }
}

template <int V>
struct Log2 {
    static constexpr int value = (V <= 1) ? 0 : 1 + Log2<V / 2>::value;
};
template <>
struct Log2<1> {
    static constexpr int value = 0;
};

__device__ __forceinline__ u64 warp_max_u64(u64 v) {
#pragma unroll
    for (int offset = 16; offset >= 1; offset >>= 1) {
        const u64 other = __shfl_xor_sync(0xffffffffu, v, offset);
        v = other > v ? other : v;
    }
    return v;
}

__device__ __forceinline__ float warp_max_f32(float v) {
#pragma unroll
    for (int offset = 16; offset >= 1; offset >>= 1) {
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, offset));
    }
    return v;
}

}  // namespace zc
