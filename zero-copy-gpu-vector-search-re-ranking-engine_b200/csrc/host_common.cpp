#include "host_common.h"

#include <atomic>
#include <cstring>
#include <mutex>
#include <set>
#include <string>
#include <utility>
#include <vector>

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

struct TimedLaunch {
    std::string tag;
    cudaEvent_t start = nullptr;
    cudaEvent_t stop = nullptr;
};

std::atomic<bool> g_timing{false};
std::mutex g_timing_mutex;
std::vector<TimedLaunch> g_timed;

void clear_timed() {
    for (TimedLaunch& t : g_timed) {
        if (t.start != nullptr) cudaEventDestroy(t.start);
        if (t.stop != nullptr) cudaEventDestroy(t.stop);
    }
    g_timed.clear();
}

}  // namespace

KernelTimer::KernelTimer(const char* tag, cudaStream_t stream) : stream_(stream) {
    if (!g_timing.load(std::memory_order_relaxed)) return;
    TimedLaunch t;
    t.tag = tag;
    if (cudaEventCreate(&t.start) != cudaSuccess || cudaEventCreate(&t.stop) != cudaSuccess ||
        cudaEventRecord(t.start, stream) != cudaSuccess) {
        if (t.start != nullptr) cudaEventDestroy(t.start);
        if (t.stop != nullptr) cudaEventDestroy(t.stop);
        cudaGetLastError();
        return;
    }
    std::lock_guard<std::mutex> lock(g_timing_mutex);
    slot_ = static_cast<int>(g_timed.size());
    g_timed.push_back(t);
}

KernelTimer::~KernelTimer() {
    if (slot_ < 0) return;
    std::lock_guard<std::mutex> lock(g_timing_mutex);
    if (slot_ < static_cast<int>(g_timed.size())) cudaEventRecord(g_timed[slot_].stop, stream_);
}

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

extern "C" {

int zcgvs_kernel_timing(int enable) {
    std::lock_guard<std::mutex> lock(zc::g_timing_mutex);
    if (enable) zc::clear_timed();
    zc::g_timing.store(enable != 0);
    return zc::ok();
}

int zcgvs_kernel_timing_read(const char* tag, double* total_ms, int* launches) {
    if (tag == nullptr || total_ms == nullptr || launches == nullptr) {
        return zc::fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_kernel_timing_read: null argument");
    }
    std::lock_guard<std::mutex> lock(zc::g_timing_mutex);
    double sum = 0.0;
    int count = 0;
    for (const zc::TimedLaunch& t : zc::g_timed) {
        if (t.tag != tag) continue;
        cudaError_t e = cudaEventSynchronize(t.stop);
        float ms = 0.0f;
        if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, t.start, t.stop);
        if (e != cudaSuccess) return zc::fail_cuda(e, "zcgvs_kernel_timing_read");
        sum += ms;
        ++count;
    }
    *total_ms = sum;
    *launches = count;
    return zc::ok();
}

}  // extern "C"
