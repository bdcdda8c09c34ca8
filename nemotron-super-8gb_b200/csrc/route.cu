// Router top-k of a decode step (bs = 1) in one kernel, with the expert-store bookkeeping the routed-expert layer
// needs: the reference's routing (NemotronHTopkRouter + NemotronHMoE.route_tokens_to_experts, tf:697-720, 748-751)
// is a chain of small torch operations (sigmoid, bias, top-k, gather, scaling) and the store lookup adds several
// more (slot ids, block addresses, s2 rows); in a decode step each is a separate launch of a few microseconds.
// Here the router logits still come from the caller's fp32 linear (so they are the reference's own), and this
// kernel does the rest: score = sigmoid(logit) (expf, IEEE division, as torch's fp32 sigmoid), choice = score +
// bias, the top_k choices (ties to the lower expert id; each expert's rank among all choices is counted in
// parallel over several CTAs, so no sequential selection rounds), weight = score * scaling, and for each chosen
// expert its store slot, block address and s2 row.
#include <climits>
#include <cmath>

#include "common.cuh"
#include "host.h"

namespace qmoe {

constexpr int RT_MAX_E = 1024;
constexpr int RT_MAX_K = 32;
constexpr int RT_THREADS = 512;
constexpr int RT_PER_CTA = 64;                       // experts ranked by one CTA
constexpr int RT_SPLIT = RT_THREADS / RT_PER_CTA;     // threads counting one expert's rank

// Grid of ceil(ne / 64) CTAs. Each CTA computes every expert's choice (one sigmoid per thread) into shared memory,
// then ranks its 64 experts, 8 threads each over an eighth of the choices. The rank of an expert is the number of
// experts whose choice beats it (larger, or equal with a lower id): a unique position in the order of decreasing
// choice, so the expert of rank r < top_k writes output r, with no communication between CTAs.
__global__ void __launch_bounds__(RT_THREADS) route_decode_kernel(const float *__restrict__ logits,
                                                                   const float *__restrict__ bias, int ne, int topk,
                                                                   float scaling, int slot_base, const uint8_t *blocks,
                                                                   int64_t block_stride, const float *__restrict__ s2,
                                                                   int64_t *ids, int32_t *sidx, int64_t *tab,
                                                                   float *s2_sel, float *coef) {
    __shared__ float score[RT_MAX_E];
    __shared__ float choice[RT_MAX_E];
    const int tid = threadIdx.x;
    for (int j = tid; j < ne; j += RT_THREADS) {
        const float s = 1.f / (1.f + expf(-logits[j]));
        float c = s + bias[j];
        if (c != c) c = -INFINITY;   // a NaN choice is never taken (torch.topk would rank it first)
        score[j] = s;
        choice[j] = c;
    }
    __syncthreads();
    const int e = blockIdx.x * RT_PER_CTA + tid / RT_SPLIT, part = tid % RT_SPLIT;
    const float c = e < ne ? choice[e] : -INFINITY;
    int rank = 0;
    for (int j = part; j < ne; j += RT_SPLIT) {
        const float v = choice[j];
        rank += v > c || (v == c && j < e);
    }
#pragma unroll
    for (int o = RT_SPLIT / 2; o; o >>= 1) rank += __shfl_xor_sync(0xffffffffu, rank, o);   // the 8 threads of e
    if (part == 0 && e < ne && rank < topk) {
        const int slot = slot_base + e;
        ids[rank] = e;
        sidx[rank] = slot;
        tab[rank] = reinterpret_cast<int64_t>(blocks + (int64_t)slot * block_stride);
        s2_sel[2 * rank] = s2[2 * e];
        s2_sel[2 * rank + 1] = s2[2 * e + 1];
        coef[rank] = score[e] * scaling;
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
    const int grid = (n_experts + RT_PER_CTA - 1) / RT_PER_CTA;
    route_decode_kernel<<<grid, RT_THREADS, 0, as_stream(stream)>>>(logits, bias, n_experts, top_k, scaling, slot_base,
                                                                    blocks, block_stride, s2, ids, sidx, tab, s2_sel,
                                                                    coef);
    return launch_status();
}

} // extern "C"
