// Host-side helpers shared by the C-ABI translation units: per-device properties (cached once per
// device), argument checks and launch-error mapping.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "../../include/qmoe_b200.h"

namespace qmoe {

constexpr int MAX_DEVICES = 64;

struct DeviceInfo {
    int sms = 0;
    int cc_major = 0;
    int cc_minor = 0;
    size_t smem_optin = 0;
};

// Lazily filled, one entry per device; the only global state of the library.
inline DeviceInfo &device_info(int dev) {
    static DeviceInfo info[MAX_DEVICES];
    static std::once_flag once[MAX_DEVICES];
    std::call_once(once[dev], [dev] {
        cudaDeviceGetAttribute(&info[dev].sms, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&info[dev].cc_major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&info[dev].cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        info[dev].smem_optin = (size_t)v;
    });
    return info[dev];
}

// Current device, checked to be an sm_100 part. Returns QMOE_OK or QMOE_ERR_DEVICE.
inline int current_device(int *dev_out, DeviceInfo **info_out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return QMOE_ERR_DEVICE;
    DeviceInfo &di = device_info(dev);
    if (di.cc_major != 10) return QMOE_ERR_DEVICE;
    if (dev_out) *dev_out = dev;
    if (info_out) *info_out = &di;
    return QMOE_OK;
}

// Raise a kernel's dynamic shared-memory limit to the device's opt-in maximum, once per device. The
// limit only caps what a launch may request; occupancy follows the bytes each launch asks for.
template <typename K>
inline bool ensure_smem(K kernel, size_t bytes, int dev, std::atomic<uint64_t> &done_mask) {
    const uint64_t bit = 1ull << (dev & 63);
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, kernel) != cudaSuccess) return false;
    const size_t optin = device_info(dev).smem_optin;
    if (fa.sharedSizeBytes > optin) return false;
    const size_t lim = optin - fa.sharedSizeBytes;   // static + dynamic must fit the opt-in maximum
    if (bytes > lim) return false;
    if (done_mask.load(std::memory_order_acquire) & bit) return true;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lim) != cudaSuccess)
        return false;
    done_mask.fetch_or(bit, std::memory_order_acq_rel);
    return true;
}

inline int launch_status() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? QMOE_OK : QMOE_ERR_LAUNCH;
}

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned4(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

inline bool valid_dtype(int dt) { return dt == QMOE_DT_F32 || dt == QMOE_DT_BF16 || dt == QMOE_DT_F16; }

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

} // namespace qmoe
