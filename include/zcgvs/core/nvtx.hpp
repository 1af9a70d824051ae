// Profiler range annotations with the reference's interface (include/zcgvs/core/nvtx.hpp:12-37):
// NvtxRange pushes a named range for its lifetime and ZCGVS_NVTX_RANGE(name) declares one in the
// current scope. Without ZCGVS_WITH_NVTX both compile to nothing, so the default build needs no
// profiler headers; defining it uses the header-only NVTX v3 API from the CUDA toolkit.
#pragma once

#ifdef ZCGVS_WITH_NVTX
#include <nvtx3/nvToolsExt.h>
#endif

namespace zcgvs {

class NvtxRange {
public:
    explicit NvtxRange(const char* name) {
#ifdef ZCGVS_WITH_NVTX
        nvtxRangePushA(name);
#else
        static_cast<void>(name);
#endif
    }
    ~NvtxRange() {
#ifdef ZCGVS_WITH_NVTX
        nvtxRangePop();
#endif
    }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

}  // namespace zcgvs

#define ZCGVS_NVTX_JOIN_(a, b) a##b
#define ZCGVS_NVTX_JOIN(a, b) ZCGVS_NVTX_JOIN_(a, b)
#define ZCGVS_NVTX_RANGE(name) ::zcgvs::NvtxRange ZCGVS_NVTX_JOIN(zcgvs_nvtx_range_, __LINE__)(name)
