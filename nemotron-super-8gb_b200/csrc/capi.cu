// Library-level entry points of libqmoe_b200: version, status names, and the workspace status word.
#include "common.cuh"
#include "host.h"

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

} // extern "C"
