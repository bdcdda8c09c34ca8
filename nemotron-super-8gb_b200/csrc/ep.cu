// Expert parallelism: pack a rank's tokens for the dispatch all-to-all and sum the partial outputs that come
// back in the combine all-to-all.
//
// The reference runs every expert on one GPU (nem_super.py:278-348). Here the 512 experts of a layer are
// sharded over `world` ranks, expert e on rank e / (n_experts / world). A layer step is
//   pack (this file) -> all_to_all(x, ids/weights) -> local expert forward (qmoe_prefill_grouped with
//   local ids, -1 = expert on another rank) -> all_to_all(partials) -> combine (this file).
// Every block of the exchange has a fixed upper bound of T rows per (source, destination) so the split sizes
// never travel to the host: with 22 of 512 experts per token a token reaches nearly every rank anyway.
// Determinism: each rank sums its own experts of a token in k order (qmoe_prefill_grouped); the combine sums
// the ranks' partials in rank order.
#include "common.cuh"
#include "host.h"

namespace qmoe {
namespace ep {

constexpr int SCAN_THREADS = 1024;
constexpr int MAX_WORLD = 64;
constexpr int MAX_TOPK = 32;
constexpr int MAX_T = 65536;

// One CTA per destination rank d: row_of[d, t] = row of token t in block d (tokens in order), or -1 when no
// expert of t lives on d; send_cnt[d] = rows used; the unused rows of block d get ids -1 (no expert).
__global__ void __launch_bounds__(SCAN_THREADS) ep_rows_kernel(const int32_t *ids, int T, int topk, int e_local,
                                                                int32_t *row_of, int32_t *send_cnt,
                                                                int32_t *send_meta) {
    __shared__ int warp_sum[32];
    __shared__ int carry;
    const int d = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int t0 = 0; t0 < T; t0 += SCAN_THREADS) {
        const int t = t0 + threadIdx.x;
        int hit = 0;
        if (t < T) {
            for (int k = 0; k < topk; k++) {
                const int e = ids[(int64_t)t * topk + k];
                hit |= (e >= 0 && e / e_local == d);
            }
        }
        int incl = hit;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        if (lane == 31) warp_sum[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            int w = warp_sum[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += y;
            }
            warp_sum[lane] = w;
        }
        __syncthreads();
        const int excl = carry + incl - hit + (warp ? warp_sum[warp - 1] : 0);
        if (t < T) row_of[(int64_t)d * T + t] = hit ? excl : -1;
        __syncthreads();
        if (threadIdx.x == 0) carry += warp_sum[31];
        __syncthreads();
    }
    const int cnt = carry;
    if (threadIdx.x == 0) send_cnt[d] = cnt;
    // rows past the count: no expert (the weights half of the row is left as is)
    for (int64_t i = (int64_t)cnt * topk + threadIdx.x; i < (int64_t)T * topk; i += SCAN_THREADS) {
        const int64_t r = i / topk, k = i % topk;
        send_meta[((int64_t)d * T + r) * 2 * topk + k] = -1;
    }
}

// One warp per (token, destination): copies the token's activation row into its block and writes the
// block-local ids (-1 for experts on other ranks) and the routing weights (as f32 bits) next to them.
__global__ void __launch_bounds__(256) ep_pack_kernel(const uint8_t *x, int row_bytes, const int32_t *ids,
                                                      const float *wts, int T, int topk, int world, int e_local,
                                                      const int32_t *row_of, uint8_t *send_x, int32_t *send_meta) {
    const int lane = threadIdx.x & 31;
    const int64_t w = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (w >= (int64_t)T * world) return;
    const int t = (int)(w / world), d = (int)(w % world);
    const int r = row_of[(int64_t)d * T + t];
    if (r < 0) return;
    const uint4 *src = reinterpret_cast<const uint4 *>(x + (int64_t)t * row_bytes);
    uint4 *dst = reinterpret_cast<uint4 *>(send_x + ((int64_t)d * T + r) * row_bytes);
    for (int i = lane; i < row_bytes / 16; i += 32) dst[i] = src[i];
    int32_t *meta = send_meta + ((int64_t)d * T + r) * 2 * topk;
    if (lane < topk) {
        const int e = ids[(int64_t)t * topk + lane];
        meta[lane] = (e >= 0 && e / e_local == d) ? e - d * e_local : -1;
        meta[topk + lane] = __float_as_int(wts[(int64_t)t * topk + lane]);
    }
}

// out[t] = sum over ranks d = 0..world-1 (in order) of part[d, row_of[d, t]] (rows with row_of = -1 skipped).
__global__ void __launch_bounds__(256) ep_combine_kernel(const float *part, const int32_t *row_of, int T, int world,
                                                         float *out) {
    const int t = blockIdx.x;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int d = 0; d < world; d++) {
        const int r = row_of[(int64_t)d * T + t];
        if (r < 0) continue;
        const float4 v = reinterpret_cast<const float4 *>(part + ((int64_t)d * T + r) * LAT)[threadIdx.x];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    reinterpret_cast<float4 *>(out + (int64_t)t * LAT)[threadIdx.x] = acc;
}

} // namespace ep
} // namespace qmoe

using namespace qmoe;

extern "C" {

int qmoe_ep_dispatch_pack(const void *x, int x_dtype, const int32_t *ids, const float *weights, int T, int topk,
                          int n_experts, int world, void *send_x, int32_t *send_meta, int32_t *row_of,
                          int32_t *send_cnt, void *stream) {
    if (!x || !ids || !weights || !send_x || !send_meta || !row_of || !send_cnt) return QMOE_ERR_NULL;
    if (T < 1 || T > ep::MAX_T || topk < 1 || topk > ep::MAX_TOPK || world < 1 || world > ep::MAX_WORLD ||
        n_experts < world || n_experts % world != 0)
        return QMOE_ERR_SHAPE;
    if (!valid_dtype(x_dtype)) return QMOE_ERR_DTYPE;
    if (!aligned16(x) || !aligned16(send_x) || !aligned4(ids) || !aligned4(weights) || !aligned4(send_meta))
        return QMOE_ERR_ALIGN;
    if (int rc = current_device(nullptr, nullptr)) return rc;
    const int row_bytes = LAT * (x_dtype == QMOE_DT_F32 ? 4 : 2);
    const int e_local = n_experts / world;
    cudaStream_t st = as_stream(stream);
    ep::ep_rows_kernel<<<world, ep::SCAN_THREADS, 0, st>>>(ids, T, topk, e_local, row_of, send_cnt, send_meta);
    const int64_t warps = (int64_t)T * world;
    ep::ep_pack_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(static_cast<const uint8_t *>(x), row_bytes, ids,
                                                                   weights, T, topk, world, e_local, row_of,
                                                                   static_cast<uint8_t *>(send_x), send_meta);
    return launch_status();
}

int qmoe_ep_combine(const float *recv_part, const int32_t *row_of, int T, int world, float *out, void *stream) {
    if (!recv_part || !row_of || !out) return QMOE_ERR_NULL;
    if (T < 1 || T > ep::MAX_T || world < 1 || world > ep::MAX_WORLD) return QMOE_ERR_SHAPE;
    if (!aligned16(recv_part) || !aligned16(out) || !aligned4(row_of)) return QMOE_ERR_ALIGN;
    if (int rc = current_device(nullptr, nullptr)) return rc;
    ep::ep_combine_kernel<<<T, 256, 0, as_stream(stream)>>>(recv_part, row_of, T, world, out);
    return launch_status();
}

} // extern "C"
