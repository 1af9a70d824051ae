#include "scan_fast.cuh"
#include "scan_instances.h"

namespace zc {

ScanKernelFn scan_lookup_fused(int mode, int jc) {
#define ZC_FUSED_CASES(MODE)                                  \
    switch (jc) {                                             \
        case 2: return &scan_fast_kernel<MODE, 2, true>;      \
        case 3: return &scan_fast_kernel<MODE, 3, true>;      \
        case 4: return &scan_fast_kernel<MODE, 4, true>;      \
        case 6: return &scan_fast_kernel<MODE, 6, true>;      \
        case 8: return &scan_fast_kernel<MODE, 8, true>;      \
        default: return nullptr;                              \
    }
    switch (mode) {
        case kModeF32: ZC_FUSED_CASES(kModeF32)
        case kModeF16: ZC_FUSED_CASES(kModeF16)
        case kModeI8M:
            // fp32 query slices of 6 or 8 int8 sweeps do not fit the register budget.
            if (jc > 4) return nullptr;
            ZC_FUSED_CASES(kModeI8M)
        case kModeI8R: ZC_FUSED_CASES(kModeI8R)
        default: return nullptr;
    }
#undef ZC_FUSED_CASES
}

}  // namespace zc
