#include "scan_instances.h"

namespace zc {

ScanKernelFn scan_lookup_f16(int qb, int jc, bool l2, bool emit) {
    if (l2) {
        ZC_SCAN_TOPK_TABLE(kModeF16, true)
        return nullptr;
    }
    ZC_SCAN_FAST_TABLE(kModeF16)
    ZC_SCAN_TOPK_TABLE(kModeF16, false)
    return nullptr;
}

}  // namespace zc
