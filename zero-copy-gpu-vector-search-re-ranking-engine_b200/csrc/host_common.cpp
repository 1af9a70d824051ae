#include "host_common.h"

#include <mutex>
#include <set>
#include <utility>

namespace zc {

namespace {

thread_local std::string g_last_error;
thread_local int g_last_cuda_error = 0;

constexpr int kMaxDevices = 64;

struct DeviceCache {
    int sm_count = 0;
    int max_smem = 0;
};

DeviceCache g_devices[kMaxDevices];
std::mutex g_mutex;
std::set<std::pair<int, const void*>> g_optin;

int current_device() {
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return 0;
    return device;
}

DeviceCache& cache_for(int device) {
    static DeviceCache fallback;
    if (device < 0 || device >= kMaxDevices) return fallback;
    DeviceCache& entry = g_devices[device];
    if (entry.sm_count == 0) {
        int sms = 0;
        int smem = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
        std::lock_guard<std::mutex> lock(g_mutex);
        entry.max_smem = smem > 0 ? smem : 48 * 1024;
        entry.sm_count = sms > 0 ? sms : 148;
    }
    return entry;
}

}  // namespace

int fail(int status, const std::string& message) {
    g_last_error = message;
    return status;
}

int fail_cuda(cudaError_t error, const char* what) {
    g_last_cuda_error = static_cast<int>(error);
    g_last_error = std::string("zcgvs: CUDA error '") + cudaGetErrorName(error) + "' (" +
                   cudaGetErrorString(error) + ") in " + what;
    return ZCGVS_ERR_CUDA;
}

int ok() {
    g_last_error.clear();
    g_last_cuda_error = 0;
    return ZCGVS_OK;
}

const char* last_error_cstr() { return g_last_error.c_str(); }

int device_sm_count() { return cache_for(current_device()).sm_count; }

int device_max_smem() { return cache_for(current_device()).max_smem; }

cudaError_t ensure_smem_optin(const void* kernel) {
    const int device = current_device();
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        if (g_optin.count({device, kernel}) != 0) return cudaSuccess;
    }
    // The opt-in limit covers static and dynamic shared memory together.
    cudaFuncAttributes attr{};
    cudaError_t status = cudaFuncGetAttributes(&attr, kernel);
    if (status != cudaSuccess) return status;
    status = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  device_max_smem() - static_cast<int>(attr.sharedSizeBytes));
    if (status == cudaSuccess) {
        std::lock_guard<std::mutex> lock(g_mutex);
        g_optin.insert({device, kernel});
    }
    return status;
}

}  // namespace zc

extern "C" {

int zcgvs_version(void) { return 100; }

const char* zcgvs_last_error_message(void) { return zc::last_error_cstr(); }

int zcgvs_last_cuda_error(void) { return zc::g_last_cuda_error; }

int zcgvs_workspace_init(void* workspace, size_t bytes, void* stream) {
    if (bytes == 0) return zc::ok();
    if (workspace == nullptr) return zc::fail(ZCGVS_ERR_INVALID_ARG, "zcgvs: null workspace");
    const cudaError_t status =
        cudaMemsetAsync(workspace, 0, bytes, static_cast<cudaStream_t>(stream));
    if (status != cudaSuccess) return zc::fail_cuda(status, "zcgvs_workspace_init");
    return zc::ok();
}

int zcgvs_workspace_status(const void* workspace, size_t bytes, uint32_t* status, void* stream) {
    if (workspace == nullptr || status == nullptr || bytes < sizeof(uint32_t)) {
        return zc::fail(ZCGVS_ERR_INVALID_ARG, "zcgvs: workspace_status needs a workspace");
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(status, workspace, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return zc::fail_cuda(e, "zcgvs_workspace_status");
    return zc::ok();
}

}  // extern "C"
