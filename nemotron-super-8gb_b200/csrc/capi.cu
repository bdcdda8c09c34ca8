// Library-level entry points of libqmoe_b200: version, status names, the workspace status word, and the chained
// copy of small per-call records (qmoe_copy_async).
#include "common.cuh"
#include "host.h"

namespace qmoe {

// A small record moved by a kernel, as a programmatic dependent of the kernel before it on the stream: the CTAs
// wait in griddepcontrol.wait and copy as soon as that kernel is done, and the next kernel (launched the same
// way) waits only for the copy. Either end may be pinned host memory (device-accessible under unified
// addressing), so a per-layer host round trip costs a PCIe read or write inside the kernel chain instead of a
// copy-engine transfer between two kernels. 16-byte words when both ends are 16-byte aligned, bytes otherwise.
__global__ void __launch_bounds__(256) copy_kernel(uint8_t *__restrict__ dst, const uint8_t *__restrict__ src, size_t n) {
    pdl_launch_dependents();
    pdl_wait();
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x, step = (size_t)gridDim.x * blockDim.x;
    size_t done = 0;
    if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15u) == 0) {
        const size_t nw = n / 16;
        for (size_t k = i; k < nw; k += step) reinterpret_cast<uint4 *>(dst)[k] = reinterpret_cast<const uint4 *>(src)[k];
        done = nw * 16;
    }
    for (size_t k = done + i; k < n; k += step) dst[k] = src[k];
}

} // namespace qmoe

extern "C" {

const char *qmoe_version(void) { return "qmoe_b200 0.1.0 (sm_100a)"; }

const char *qmoe_status_string(int status) {
    switch (status) {
    case QMOE_OK: return "ok";
    case QMOE_ERR_SHAPE: return "bad shape or count";
    case QMOE_ERR_ALIGN: return "bad alignment";
    case QMOE_ERR_LAUNCH: return "CUDA launch failed";
    case QMOE_ERR_TIMEOUT: return "device-side wait timed out";
    case QMOE_ERR_NULL: return "null pointer";
    case QMOE_ERR_DTYPE: return "unknown activation dtype";
    case QMOE_ERR_DEVICE: return "current device is not sm_100";
    case QMOE_ERR_WORKSPACE: return "workspace too small";
    case QMOE_ERR_SCRATCH_LIMIT: return "K exceeds the static scratch of the allocation-free entry point";
    default: return "unknown status";
    }
}

int qmoe_workspace_status(void *workspace, int clear, void *stream) {
    if (!workspace) return QMOE_ERR_NULL;
    int v = 0;
    cudaStream_t st = qmoe::as_stream(stream);
    if (cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess) return QMOE_ERR_LAUNCH;
    if (cudaStreamSynchronize(st) != cudaSuccess) return QMOE_ERR_LAUNCH;
    if (clear && v != 0) {
        if (cudaMemsetAsync(workspace, 0, sizeof(int), st) != cudaSuccess) return QMOE_ERR_LAUNCH;
    }
    return v;
}

int qmoe_copy_async(void *dst, const void *src, size_t bytes, void *stream) {
    if (bytes == 0) return QMOE_OK;
    if (!dst || !src) return QMOE_ERR_NULL;
    int dev;
    qmoe::DeviceInfo *di;
    if (int rc = qmoe::current_device(&dev, &di)) return rc;
    const size_t per_cta = 256 * 16;
    size_t blocks = (bytes + per_cta - 1) / per_cta;
    if (blocks > (size_t)4 * di->sms) blocks = (size_t)4 * di->sms;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(256);
    cfg.stream = qmoe::as_stream(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, qmoe::copy_kernel, static_cast<uint8_t *>(dst), static_cast<const uint8_t *>(src), bytes) !=
        cudaSuccess)
        return QMOE_ERR_LAUNCH;
    return qmoe::launch_status();
}

} // extern "C"
