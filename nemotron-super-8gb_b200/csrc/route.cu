// Router top-k of a decode step (bs = 1) in one kernel, with the expert-store bookkeeping the routed-expert layer
// needs: the reference's routing (NemotronHTopkRouter + NemotronHMoE.route_tokens_to_experts, tf:697-720, 748-751)
// is a chain of small torch operations (sigmoid, bias, top-k, gather, scaling) and the store lookup adds several
// more (slot ids, block addresses, s2 rows); in a decode step each is a separate launch of a few microseconds.
// Here the router logits still come from the caller's fp32 linear (so they are the reference's own), and this
// kernel does the rest: score = sigmoid(logit) (expf, IEEE division, as torch's fp32 sigmoid), choice = score +
// bias, the top_k choices (ties to the lower expert id; each expert's rank among all choices is counted in
// parallel, so no sequential selection rounds), weight = score * scaling, and for each chosen expert its store slot,
// block address and s2 row.
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
    __shared__ __align__(16) float choice[RT_MAX_E];
    __shared__ int sel[RT_MAX_K];
    const int tid = threadIdx.x;
    float c = -INFINITY;
    if (tid < ne) {
        const float s = 1.f / (1.f + expf(-logits[tid]));
        score[tid] = s;
        c = s + bias[tid];
        if (c != c) c = -INFINITY;   // a NaN choice is never taken (torch.topk would rank it first)
    }
    if (tid < ne) choice[tid] = c;
    __syncthreads();
    // rank of this expert = the experts whose choice beats it (larger, or equal with a lower id): a unique
    // position in the order of decreasing choice, so the top_k need no sequential selection rounds
    if (tid < ne) {
        int rank = 0;
        const int n4 = ne & ~3;
        for (int j = 0; j < n4; j += 4) {
            const float4 v = *reinterpret_cast<const float4 *>(choice + j);
            rank += (v.x > c || (v.x == c && j < tid)) + (v.y > c || (v.y == c && j + 1 < tid)) +
                    (v.z > c || (v.z == c && j + 2 < tid)) + (v.w > c || (v.w == c && j + 3 < tid));
        }
        for (int j = n4; j < ne; ++j) rank += choice[j] > c || (choice[j] == c && j < tid);
        if (rank < topk) sel[rank] = tid;
    }
    __syncthreads();
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
