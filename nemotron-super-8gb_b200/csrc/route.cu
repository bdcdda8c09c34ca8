// Router top-k of a decode step (bs = 1) in one kernel, with the expert-store bookkeeping the routed-expert layer
// needs: the reference's routing (NemotronHTopkRouter + NemotronHMoE.route_tokens_to_experts, tf:697-720, 748-751)
// is a chain of small torch operations (sigmoid, bias, top-k, gather, scaling) and the store lookup adds several
// more (slot ids, block addresses, s2 rows); in a decode step each is a separate launch of a few microseconds.
// Here the router logits still come from the caller's fp32 linear (so they are the reference's own), and this
// kernel does the rest: score = sigmoid(logit) (expf, IEEE division, as torch's fp32 sigmoid), choice = score +
// bias, the top_k choices (ties to the lower expert id), weight = score * scaling, and for each chosen expert its
// store slot, block address and s2 row.
#include <climits>
#include <cmath>

#include "common.cuh"
#include "host.h"

namespace qmoe {

constexpr int RT_MAX_E = 1024;
constexpr int RT_MAX_K = 32;

__global__ void __launch_bounds__(RT_MAX_E) route_decode_kernel(const float *__restrict__ logits,
                                                                 const float *__restrict__ bias, int ne, int topk,
                                                                 float scaling, int slot_base, const uint8_t *blocks,
                                                                 int64_t block_stride, const float *__restrict__ s2,
                                                                 int64_t *ids, int32_t *sidx, int64_t *tab,
                                                                 float *s2_sel, float *coef) {
    __shared__ float score[RT_MAX_E];
    __shared__ float wbest[32];
    __shared__ int wbesti[32];
    __shared__ int sel[RT_MAX_K];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    float c = -INFINITY;
    if (tid < ne) {
        const float s = 1.f / (1.f + expf(-logits[tid]));
        score[tid] = s;
        c = s + bias[tid];
        if (c != c) c = -INFINITY;   // a NaN choice is never taken (torch.topk would rank it first)
    }
    for (int r = 0; r < topk; ++r) {
        // block arg-max of (choice, -id): the largest choice, ties to the lower expert id
        float v = c;
        int i = tid < ne ? tid : INT_MAX;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
            const int i2 = __shfl_xor_sync(0xffffffffu, i, o);
            if (v2 > v || (v2 == v && i2 < i)) v = v2, i = i2;
        }
        if (lane == 0) wbest[warp] = v, wbesti[warp] = i;
        __syncthreads();
        if (warp == 0) {
            v = lane < nw ? wbest[lane] : -INFINITY;
            i = lane < nw ? wbesti[lane] : INT_MAX;
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
                const int i2 = __shfl_xor_sync(0xffffffffu, i, o);
                if (v2 > v || (v2 == v && i2 < i)) v = v2, i = i2;
            }
            if (lane == 0) sel[r] = i;
        }
        __syncthreads();
        if (tid == sel[r]) c = -INFINITY;   // taken
    }
    if (tid < topk) {
        const int e = sel[tid];
        const int slot = slot_base + e;
        ids[tid] = e;
        sidx[tid] = slot;
        tab[tid] = reinterpret_cast<int64_t>(blocks + (int64_t)slot * block_stride);
        s2_sel[2 * tid] = s2[2 * e];
        s2_sel[2 * tid + 1] = s2[2 * e + 1];
        coef[tid] = score[e] * scaling;
    }
}

} // namespace qmoe

using namespace qmoe;

extern "C" {

int qmoe_route_decode(const float *logits, const float *bias, int n_experts, int top_k, float scaling, int slot_base,
                      const uint8_t *blocks, int64_t block_stride, const float *s2, int64_t *ids, int32_t *sidx,
                      int64_t *tab, float *s2_sel, float *coef, void *stream) {
    if (!logits || !bias || !blocks || !s2 || !ids || !sidx || !tab || !s2_sel || !coef) return QMOE_ERR_NULL;
    if (n_experts < 1 || n_experts > RT_MAX_E || top_k < 1 || top_k > RT_MAX_K || top_k > n_experts)
        return QMOE_ERR_SHAPE;
    int dev;
    DeviceInfo *di;
    if (int rc = current_device(&dev, &di)) return rc;
    const int threads = ((n_experts + 31) / 32) * 32;
    route_decode_kernel<<<1, threads, 0, as_stream(stream)>>>(logits, bias, n_experts, top_k, scaling, slot_base, blocks,
                                                               block_stride, s2, ids, sidx, tab, s2_sel, coef);
    return launch_status();
}

} // extern "C"
