#include "scan_instances.h"

namespace zc {

ScanKernelFn scan_lookup_i8(int mode, int qb, int jc, bool l2, bool emit) {
    if (mode == kModeI8R) {
        if (l2) return nullptr;
        ZC_SCAN_FAST_TABLE(kModeI8R)
        ZC_SCAN_TOPK_TABLE(kModeI8R, false)
        return nullptr;
    }
    if (l2) {
        ZC_SCAN_TOPK_TABLE(kModeI8M, true)
        return nullptr;
    }
    ZC_SCAN_FAST_TABLE(kModeI8M)
    ZC_SCAN_TOPK_TABLE(kModeI8M, false)
    return nullptr;
}

}  // namespace zc
