// Device selection and the device facts the reference's tools print and measure against: the
// reference's cuda_context interface (include/zcgvs/core/cuda_context.hpp:8-32, implemented in
// src/core/cuda_context.cpp:9-45), with the same names, fields and exceptions (CudaError on a
// failed runtime call), so its engine and kernel benchmark compile unchanged against it.
// Implemented in csrc/cxx_api.cpp.
#pragma once

#include <cstddef>
#include <string>

namespace zcgvs {

struct DeviceInfo {
    int device_id = 0;
    std::string name;
    std::size_t total_memory = 0;
    int compute_major = 0;
    int compute_minor = 0;
    int multiprocessor_count = 0;
    int memory_clock_khz = 0;       // DRAM clock (the data rate is twice it)
    int memory_bus_width_bits = 0;

    // Theoretical DRAM bandwidth in GB/s: two transfers per memory clock over the whole bus.
    // A brute-force scan reads the corpus once, so this is the roofline it is measured against
    // (a measured copy bandwidth is the better denominator; see the bench's MEASURED_PEAKS).
    double peakBandwidthGBs() const {
        const double bytes_per_clock = static_cast<double>(memory_bus_width_bits) / 8.0;
        return 2.0 * static_cast<double>(memory_clock_khz) * 1e3 * bytes_per_clock / 1e9;
    }
};

// Makes `device_id` current for the calling thread (cudaSetDevice).
void setDevice(int device_id);

// The calling thread's current device.
int currentDevice();

// Number of visible CUDA devices.
int deviceCount();

// Properties of `device_id` (cudaGetDeviceProperties plus the memory-clock attribute).
DeviceInfo queryDevice(int device_id);

}  // namespace zcgvs
