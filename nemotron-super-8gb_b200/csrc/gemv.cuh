// Quantized GEMV over "items" for sm_100a: y_item[m, n] = mult_item * sum_k W_item[n, k] * v_item[m, k].
//
// One kernel serves the reference's dense FP8 / NVFP4 GEMVs (dense_q.py:35-136), the orig-layout expert
// down GEMV `_down` (qmoe_ns.py:47-67) and the per-pair prompt kernels `_up_pairs` / `_down_pairs`
// (qmoe_ns.py:79-124). Arithmetic as the reference's: codes and scales decoded exactly, every product exact,
// every sum in fp32 ("x -> fp32, accumulation fp32", qmoe_ns.py:4). Design:
//   - each CTA owns ROWS rows of one item; its vectors are staged once in shared memory, either as f16x2
//     scaled by an exact power of two (bf16 / f16 activations: exact, amax*2^E in [256, 512)) or as fp32
//     (fp32 activations and the down modes' h, which are never rounded);
//   - a warp streams whole rows with 16-byte non-allocating loads, all chunks of two rows in flight per
//     lane; codes are decoded with the hardware e2m1x2 / e4m3x2 -> f16x2 converts and multiplied into fp32
//     accumulators (fma.rn.f32.f16 against the f16 vector, or fp32 FMAs against the fp32 vector); an NVFP4
//     16-element group sum is then scaled by its block scale in fp32;
//   - rows are reduced with warp shuffles; the item epilogue applies the fp32 multiplier (and ReLU^2).
// The shared-memory vector layout is [m][q][chunk] of uint4 so that the 8 lanes of a quarter-warp read
// 8 consecutive uint4 (no bank conflicts).
#pragma once
#include "common.cuh"

namespace qmoe {

enum GemvMode { GM_DENSE = 0, GM_EXPERT_DOWN = 1, GM_PAIR_UP = 2, GM_PAIR_DOWN = 3 };

struct GemvArgs {
    // dense
    const uint8_t *w;    // [N, KB]
    const uint8_t *sc;   // [N, K/16] (NVFP4)
    const float *s;      // [1] device scalar (FP8 s / NVFP4 s2)
    const void *x;       // [M, K] (dense) or [T, K] (pairs up) in x_dtype
    int x_dtype;
    float *y;            // output
    int M, N, K;
    // experts / pairs
    const uint8_t *slots;
    int64_t slot_bytes;
    int64_t nslots;       // slot indices outside [0, nslots) read nothing and yield NaN
    const int32_t *sidx;  // expert down: slot of item j; pairs: pslot
    const int32_t *ptok;  // pairs up: token of item p (tokens outside [0, T) yield NaN)
    int T;
    const float *s2;      // [items, 2]
    const float *coef;    // [items]
    const float *hin;     // down modes: f32 vectors [items, K]
    float *hout;          // pair up: h out [items, N]
    // dense, bf16 output instead of y: 1 = bf16 of relu(bf16(v))^2, 2 = bf16 of bf16(v) + res, 3 = bf16(v)
    // (torch's roundings); 0 = the fp32 y
    int out_op;
    uint16_t *ybf;
    const uint16_t *res;
};

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;

// The vector of a GEMV in shared memory: f16x2 (bf16 / f16 activations, prescaled) or fp32.
__host__ __device__ constexpr int gemv_vec_bytes(bool vf32) { return vf32 ? 4 : 2; }

// FMT 0 = FP8 e4m3 (16 elements per 16-byte chunk), 1 = NVFP4 (32 elements per chunk, 2 scales), 2 = bf16 (8
// elements per chunk, no scale; always with fp32 vectors, the bf16 weights widened exactly).
// VF32: the vectors are staged (and multiplied) in fp32; otherwise as prescaled f16.
template <int FMT, int MODE, int CPL, int M, bool VF32>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_kernel(GemvArgs a, int rows_per_cta) {
    constexpr int EPC = FMT == 1 ? 32 : FMT == 2 ? 8 : 16;   // elements per chunk
    static_assert(FMT != 2 || VF32, "bf16 weights take fp32 vectors");
    constexpr int EPU = VF32 ? 4 : 8;                 // vector elements per uint4
    constexpr int Q = EPC / EPU;                      // uint4 of the vector per chunk
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint4 *xs = reinterpret_cast<uint4 *>(smem_raw);
    __shared__ float red[GEMV_WARPS][M];
    __shared__ float vscale[M];

    const int K = a.K;
    const int KB = FMT == 1 ? K / 2 : FMT == 2 ? K * 2 : K;
    const int nch = KB / 16;   // chunks per row
    const int item = blockIdx.y;
    const int row0 = blockIdx.x * rows_per_cta;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // ---- item descriptor
    const uint8_t *W;
    const uint8_t *S = nullptr;
    float mult;
    int nrows = a.N;
    bool bad = false;
    if (MODE == GM_DENSE) {
        W = a.w;
        S = a.sc;
        mult = FMT == 2 ? 1.f : *a.s;
    } else {
        int64_t slot = a.sidx[item];
        bad = slot < 0 || slot >= a.nslots;
        if (MODE == GM_PAIR_UP) bad = bad || a.ptok[item] < 0 || a.ptok[item] >= a.T;
        if (bad) slot = 0;
        const uint8_t *blk = a.slots + slot * a.slot_bytes;
        if (MODE == GM_PAIR_UP) {
            W = blk + O_UW;
            S = blk + O_US;
            mult = a.s2[2 * item];
        } else {
            W = blk + O_DW;
            S = blk + O_DS;
            mult = a.coef[item] * a.s2[2 * item + 1];
        }
    }
    if (bad) mult = __int_as_float(0x7fc00000);

    auto vec = [&](int m, int i) -> float {   // element i of vector m
        if (MODE == GM_DENSE) return load_act(a.x, a.x_dtype, (int64_t)m * K + i);
        if (MODE == GM_PAIR_UP) return bad ? 0.f : load_act(a.x, a.x_dtype, (int64_t)a.ptok[item] * K + i);
        return a.hin[(int64_t)item * K + i];
    };

    // ---- vectors -> shared memory (f16x2 prescaled by 2^E, exact; or fp32 as given)
    if constexpr (!VF32) {
        float am[M];
#pragma unroll
        for (int m = 0; m < M; ++m) am[m] = 0.f;
        for (int i = tid; i < K; i += GEMV_THREADS) {
#pragma unroll
            for (int m = 0; m < M; ++m) am[m] = fmaxf(am[m], fabsf(vec(m, i)));
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float v = am[m];
            for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
            if (lane == 0) red[warp][m] = v;
        }
        __syncthreads();
        if (tid < M) {
            float v = 0.f;
            for (int i = 0; i < GEMV_WARPS; ++i) v = fmaxf(v, red[i][tid]);
            vscale[tid] = (float)prescale_exp(v, 9);
        }
        __syncthreads();
        // xs[m][q][c] as 32-bit words: element pair i (elements 2i, 2i+1) -> chunk c = i / (EPC/2),
        // q = (i % (EPC/2)) / 4, word i % 4
        uint32_t *xs32 = reinterpret_cast<uint32_t *>(smem_raw);
        for (int i = tid; i < K / 2; i += GEMV_THREADS) {
            const int c = i / (EPC / 2), r = i % (EPC / 2), q = r / 4, wi = r % 4;
#pragma unroll
            for (int m = 0; m < M; ++m) {
                const float pe = pow2f((int)vscale[m]);
                const __half2 hv = __halves2half2(__float2half_rn(vec(m, 2 * i) * pe), __float2half_rn(vec(m, 2 * i + 1) * pe));
                xs32[(((size_t)m * Q + q) * nch + c) * 4 + wi] = h2_as_u(hv);
            }
        }
    } else {
        // xs[m][q][c] as float2: element pair i -> chunk c = i / (EPC/2), q = (i % (EPC/2)) / 2, pair i % 2
        float2 *xs2 = reinterpret_cast<float2 *>(smem_raw);
        for (int i = tid; i < K / 2; i += GEMV_THREADS) {
            const int c = i / (EPC / 2), r = i % (EPC / 2), q = r / 2, wi = r % 2;
#pragma unroll
            for (int m = 0; m < M; ++m) xs2[(((size_t)m * Q + q) * nch + c) * 2 + wi] = make_float2(vec(m, 2 * i), vec(m, 2 * i + 1));
        }
        if (tid < M) vscale[tid] = 0.f;
    }
    __syncthreads();
    float inv[M];
#pragma unroll
    for (int m = 0; m < M; ++m) inv[m] = pow2f(-(int)vscale[m]);

    // ---- rows: each warp takes rows warp, warp+8, ... two at a time
    const int row_end = min(row0 + rows_per_cta, nrows);
    for (int r = row0 + warp * 2; r < row_end; r += GEMV_WARPS * 2) {
        const bool two = (r + 1) < row_end;
        float acc[2][M];
#pragma unroll
        for (int rr = 0; rr < 2; ++rr)
#pragma unroll
            for (int m = 0; m < M; ++m) acc[rr][m] = 0.f;
        for (int cb = 0; cb < nch; cb += 32 * CPL) {
            uint4 wv[2][CPL];
            uint16_t sv[2][CPL];
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                const int row = two ? r + rr : r;
                const uint8_t *wrow = W + (int64_t)row * KB;
                const uint8_t *srow = FMT == 1 ? S + (int64_t)row * (K / 16) : nullptr;
#pragma unroll
                for (int i = 0; i < CPL; ++i) {
                    const int c = cb + lane + 32 * i;
                    if (c < nch) {
                        wv[rr][i] = ldg_stream(wrow + 16 * c);
                        if (FMT == 1) sv[rr][i] = __ldg(reinterpret_cast<const uint16_t *>(srow) + c);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < CPL; ++i) {
                const int c = cb + lane + 32 * i;
                if (c < nch) {
#pragma unroll
                    for (int m = 0; m < M; ++m) {
                        uint4 xq[Q];
#pragma unroll
                        for (int q = 0; q < Q; ++q) xq[q] = xs[((size_t)m * Q + q) * nch + c];
                        const uint32_t *xw = reinterpret_cast<const uint32_t *>(xq);   // f16x2 words
                        const float2 *xf = reinterpret_cast<const float2 *>(xq);       // fp32 pairs
#pragma unroll
                        for (int rr = 0; rr < 2; ++rr) {
                            const uint32_t *ww = reinterpret_cast<const uint32_t *>(&wv[rr][i]);
                            // g[group][lo/hi]: fp32 partial sums of the chunk's one or two 16-element groups
                            float g[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
                            if (FMT == 1) {
#pragma unroll
                                for (int wd = 0; wd < 4; ++wd) {   // word wd: elements 8wd .. 8wd+7
                                    uint32_t o[4];
                                    e2m1x8_f16x2(ww[wd], o);
#pragma unroll
                                    for (int k = 0; k < 4; ++k) {
                                        float &lo = g[wd >> 1][0], &hi = g[wd >> 1][1];
                                        if constexpr (VF32) {
                                            const float2 cv = __half22float2(as_h2(o[k]));
                                            const float2 xv = xf[4 * wd + k];
                                            lo = fmaf(cv.x, xv.x, lo);
                                            hi = fmaf(cv.y, xv.y, hi);
                                        } else {
                                            fma2_f16_f32(o[k], xw[4 * wd + k], lo, hi);
                                        }
                                    }
                                }
                                const float2 sf = __half22float2(as_h2(e4m3x2_f16x2(sv[rr][i])));
                                acc[rr][m] = fmaf(g[0][0] + g[0][1], sf.x, acc[rr][m]);
                                acc[rr][m] = fmaf(g[1][0] + g[1][1], sf.y, acc[rr][m]);
                            } else if (FMT == 2) {
#pragma unroll
                                for (int wd = 0; wd < 4; ++wd) {   // word wd: elements 2wd, 2wd+1 (bf16 -> fp32 exact)
                                    const float2 xv = xf[wd];
                                    g[0][0] = fmaf(__uint_as_float(ww[wd] << 16), xv.x, g[0][0]);
                                    g[0][1] = fmaf(__uint_as_float(ww[wd] & 0xFFFF0000u), xv.y, g[0][1]);
                                }
                                acc[rr][m] += g[0][0] + g[0][1];
                            } else {
#pragma unroll
                                for (int wd = 0; wd < 4; ++wd) {   // word wd: elements 4wd .. 4wd+3
                                    uint32_t lo2, hi2;
                                    e4m3x4_f16x2(ww[wd], lo2, hi2);
                                    if constexpr (VF32) {
                                        const float2 c0 = __half22float2(as_h2(lo2)), c1 = __half22float2(as_h2(hi2));
                                        const float2 x0 = xf[2 * wd], x1 = xf[2 * wd + 1];
                                        g[0][0] = fmaf(c0.x, x0.x, g[0][0]);
                                        g[0][1] = fmaf(c0.y, x0.y, g[0][1]);
                                        g[1][0] = fmaf(c1.x, x1.x, g[1][0]);
                                        g[1][1] = fmaf(c1.y, x1.y, g[1][1]);
                                    } else {
                                        fma2_f16_f32(lo2, xw[2 * wd], g[0][0], g[0][1]);
                                        fma2_f16_f32(hi2, xw[2 * wd + 1], g[1][0], g[1][1]);
                                    }
                                }
                                acc[rr][m] += (g[0][0] + g[0][1]) + (g[1][0] + g[1][1]);
                            }
                        }
                    }
                }
            }
        }
        // warp reduction of both rows
#pragma unroll
        for (int rr = 0; rr < 2; ++rr)
#pragma unroll
            for (int m = 0; m < M; ++m)
                for (int o = 16; o; o >>= 1) acc[rr][m] += __shfl_xor_sync(0xffffffffu, acc[rr][m], o);
        if (lane < 2 && (lane == 0 || two)) {
            const int row = r + lane;
#pragma unroll
            for (int m = 0; m < M; ++m) {
                const float v = (lane == 0 ? acc[0][m] : acc[1][m]) * inv[m];
                if (MODE == GM_DENSE) {
                    const int64_t o = (int64_t)m * a.N + row;
                    if (a.out_op == 0) {
                        a.y[o] = v * mult;
                    } else {
                        // the linear's output as torch leaves it (bf16), then relu^2 or the residual add, each
                        // computed in fp32 and rounded to bf16 as torch's bf16 operators do
                        float b = __bfloat162float(__float2bfloat16_rn(v * mult));
                        if (a.out_op == 1) {
                            b = b > 0.f ? b : (b != b ? b : 0.f);   // relu, NaN kept
                            b = b * b;
                        } else if (a.out_op == 2) {
                            b = b + __bfloat162float(__ushort_as_bfloat16(a.res[o]));
                        }   // 3: the bf16 cast alone
                        a.ybf[o] = __bfloat16_as_ushort(__float2bfloat16_rn(b));
                    }
                } else if (MODE == GM_PAIR_UP) {
                    float u = v * mult;
                    u = fmaxf(u, 0.f);
                    a.hout[(int64_t)item * a.N + row] = u * u;
                } else {
                    a.y[(int64_t)item * a.N + row] = v * mult;
                }
            }
        }
    }
}

// shared-memory bytes of the vector copy
inline size_t gemv_smem_bytes(bool vf32, int M, int K) { return (size_t)M * (size_t)K * gemv_vec_bytes(vf32); }

} // namespace qmoe
