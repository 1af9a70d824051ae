#include "scan_instances.h"

namespace zc {

ScanKernelFn scan_lookup_f32(int qb, int jc, bool l2, bool emit) {
    if (l2) {
        ZC_SCAN_TOPK_TABLE(kModeF32, true)
        return nullptr;
    }
    ZC_SCAN_FAST_TABLE(kModeF32)
    ZC_SCAN_TOPK_TABLE(kModeF32, false)
    return nullptr;
}

}  // namespace zc
