// Kernel lookup tables of the streaming scan. Each scan_<mode>.cu instantiates the variants
// of one storage mode; the launcher picks one by (query pass width, register chunk count,
// metric, output form).
#pragma once

#include "scan_kernel.cuh"

namespace zc {

using ScanKernelFn = void (*)(const ScanParams);

ScanKernelFn scan_lookup_f32(int qb, int jc, bool l2, bool emit);
ScanKernelFn scan_lookup_f16(int qb, int jc, bool l2, bool emit);
ScanKernelFn scan_lookup_i8(int mode, int qb, int jc, bool l2, bool emit);
ScanKernelFn scan_lookup_bin(int qb, bool emit);
// Warp-specialised single-query kernel (scan_fast.cuh), 16 lanes per row, `jc` sweeps.
ScanKernelFn scan_lookup_fast(int mode, int jc);
// Its hybrid variant with lexical warps (dense scores and BM25 scores out, no selection).
ScanKernelFn scan_lookup_fused(int mode, int jc);

}  // namespace zc

// Instantiation helpers. Generic variants (query read from shared memory, warp per row) for
// query pass widths 1/2/4/8, the register-resident single-query fast path with 16 lanes per
// row and two rows per lane group (four rows per warp iteration) for 2/3/4/6/8 chunks
// per lane, and one score-matrix variant
// (8 queries per pass).
#define ZC_SCAN_TOPK_TABLE(MODE, L2)                                          \
    if (emit) {                                                               \
        if (qb == 8 && jc == 0) return &scan_kernel<MODE, 8, 0, 32, 1, L2, true>;\
        return nullptr;                                                       \
    }                                                                         \
    if (jc == 0) {                                                            \
        switch (qb) {                                                         \
            case 1: return &scan_kernel<MODE, 1, 0, 32, 1, L2, false>;           \
            case 2: return &scan_kernel<MODE, 2, 0, 32, 1, L2, false>;           \
            case 4: return &scan_kernel<MODE, 4, 0, 32, 1, L2, false>;           \
            case 8: return &scan_kernel<MODE, 8, 0, 32, 1, L2, false>;           \
            default: return nullptr;                                          \
        }                                                                     \
    }

#define ZC_SCAN_FAST_TABLE(MODE)                                              \
    if (!emit && qb == 1) {                                                   \
        switch (jc) {                                                         \
            case 2: return &scan_kernel<MODE, 1, 2, 16, 2, false, false>;        \
            case 3: return &scan_kernel<MODE, 1, 3, 16, 2, false, false>;        \
            case 4: return &scan_kernel<MODE, 1, 4, 16, 2, false, false>;        \
            case 6: return &scan_kernel<MODE, 1, 6, 16, 2, false, false>;        \
            case 8: return &scan_kernel<MODE, 1, 8, 16, 2, false, false>;        \
            default: break;                                                   \
        }                                                                     \
    }
