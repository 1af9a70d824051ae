#include "scan_fast.cuh"
#include "scan_instances.h"

namespace zc {

ScanKernelFn scan_lookup_fast(int mode, int jc) {
#define ZC_FAST_CASES(MODE)                                   \
    switch (jc) {                                             \
        case 2: return &scan_fast_kernel<MODE, 2>;            \
        case 3: return &scan_fast_kernel<MODE, 3>;            \
        case 4: return &scan_fast_kernel<MODE, 4>;            \
        case 6: return &scan_fast_kernel<MODE, 6>;            \
        case 8: return &scan_fast_kernel<MODE, 8>;            \
        default: return nullptr;                              \
    }
    switch (mode) {
        case kModeF32: ZC_FAST_CASES(kModeF32)
        case kModeF16: ZC_FAST_CASES(kModeF16)
        case kModeI8M:
            // fp32 query slices of 6 or 8 int8 sweeps do not fit the register budget.
            if (jc > 4) return nullptr;
            ZC_FAST_CASES(kModeI8M)
        case kModeI8R: ZC_FAST_CASES(kModeI8R)
        default: return nullptr;
    }
#undef ZC_FAST_CASES
}

}  // namespace zc
