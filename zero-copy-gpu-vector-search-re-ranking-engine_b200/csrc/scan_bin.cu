#include "scan_instances.h"

namespace zc {

ScanKernelFn scan_lookup_bin(int qb, bool emit) {
    if (emit) return qb == 8 ? &scan_kernel<kModeBin, 8, 0, 32, 1, false, true> : nullptr;
    switch (qb) {
        case 1: return &scan_kernel<kModeBin, 1, 0, 32, 1, false, false>;
        case 2: return &scan_kernel<kModeBin, 2, 0, 32, 1, false, false>;
        case 4: return &scan_kernel<kModeBin, 4, 0, 32, 1, false, false>;
        case 8: return &scan_kernel<kModeBin, 8, 0, 32, 1, false, false>;
        default: return nullptr;
    }
}

}  // namespace zc
