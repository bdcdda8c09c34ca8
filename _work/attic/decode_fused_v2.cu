// Fused decode-step routed-expert layer for sm_100a: `moe_decode_groups` (qmoe_ns.py:245-255) as one
// cooperative kernel (one CTA per SM): up GEMV + ReLU^2, the live-group down GEMV and the sum over
// experts in a single launch.
//
// CTA c owns the 16-neuron groups q = c + k*grid (k = 0, 1, ...) of the layer's K experts.
//   Phase 1 (`_up`, qmoe_ns.py:24-44): its 16 warps stream the groups' 8-row halves exactly as the
//     stand-alone up kernel does (16-byte streaming loads, cvt.e2m1x2 + HFMA2, fp32 scales, butterfly,
//     ReLU^2), write h and the half's live mask, and keep mask and the 8 values of h in shared memory.
//   Phase 2 (`_down_groups`, qmoe_ns.py:209-239), after a CTA barrier: warp w takes the CTA's groups
//     w, w+16, ...; for a group with a live neuron it loads the T-layout scale row dnT_s[g, :] (lane l:
//     32 B = rows 32l..32l+31) and, 4 at a time, the 512-byte rows dnT_w[n, :] of its live neurons, and
//     accumulates coef_j*s2d_j * D_j[:, n] * h_j[n] into the warp's register slice of the output.
//   Phase 3: the 16 warp slices are summed in warp order into the CTA partial, all CTAs meet at a
//     bounded grid barrier, and each CTA sums a slice of output rows over all CTA partials in CTA order;
//     CTAs also compact the live groups of experts j = c (mod grid) into gidx / gcnt (qmoe_ns.py:249-251).
// Every summation order is fixed by the static schedule, so the result is bit-reproducible.
#include "common.cuh"
#include "host.h"

namespace qmoe {
namespace fused {

constexpr int NW = 16;                  // warps per CTA
constexpr int THREADS = 32 * NW;
constexpr int MAXK = 64;
constexpr int MAX_GRID = 256;
constexpr int DNB = 4;                  // live neurons per down batch (loads in flight together)

// workspace layout (zero-filled once by the caller; the barrier words are self-restoring)
constexpr size_t WS_STATUS = 0;
constexpr size_t WS_BAR = 64;           // int count, int epoch
constexpr size_t WS_GMASK = 256;        // u8 [K, 336]
__host__ __device__ inline size_t ws_partials(int K) { return (WS_GMASK + (size_t)K * 336 + 255) / 256 * 256; }
__host__ __device__ inline size_t ws_bytes(int K) { return ws_partials(K) + (size_t)MAX_GRID * LAT * 4; }

struct Args {
    const uint8_t *slots;
    int64_t slot_bytes, nslots;
    const int32_t *sidx;
    const int64_t *tab;
    const float *s2, *coef;
    const void *x;
    int x_dtype, K;
    float *h;
    int32_t *gidx, *gcnt;
    float *y;
    uint8_t *ws;
};

__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// Sense-reversing barrier over all CTAs of a cooperative launch; bounded (records a timeout).
__device__ bool grid_barrier(int *count, int *epoch, int *status) {
    __threadfence();                                          // this CTA's writes before its arrival
    const int e = *reinterpret_cast<volatile int *>(epoch);
    __threadfence();                                          // the epoch read before the arrival
    if (atomicAdd(count, 1) == (int)gridDim.x - 1) {
        *reinterpret_cast<volatile int *>(count) = 0;
        __threadfence();
        atomicAdd(epoch, 1);
        return true;
    }
    const long long t0 = clock64();
    while (*reinterpret_cast<volatile int *>(epoch) == e) {
        if (clock64() - t0 > WAIT_CYCLES) {
            set_error(status, QMOE_ERR_TIMEOUT);
            return false;
        }
        __nanosleep(32);
    }
    __threadfence();
    return true;
}

__global__ void __launch_bounds__(THREADS, 1) decode_layer_kernel(Args a) {
    __shared__ const uint8_t *s_up[MAXK];     // up block of expert j (nullptr: slot out of range)
    __shared__ const uint8_t *s_dn[MAXK];     // T block of expert j (nullptr: null or misaligned)
    __shared__ float s_s2u[MAXK], s_dmul[MAXK];
    __shared__ int s_ok;
    extern __shared__ __align__(16) float dyn[];   // red [NW][1024] | hh [nhalf][8] | mk [nhalf]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = a.K;
    const int G = gridDim.x;
    int *status = reinterpret_cast<int *>(a.ws + WS_STATUS);
    uint8_t *gmask8 = a.ws + WS_GMASK;
    float *partial = reinterpret_cast<float *>(a.ws + ws_partials(K));
    const int ngroups = K * G_DN;
    const int my_groups = (int)blockIdx.x < ngroups ? (ngroups - 1 - (int)blockIdx.x) / G + 1 : 0;
    const int nhalf = 2 * my_groups;
    float *red = dyn;
    float *hh = dyn + NW * LAT;
    int *mk = reinterpret_cast<int *>(hh + 8 * nhalf);

    for (int j = threadIdx.x; j < K; j += blockDim.x) {
        const int64_t slot = a.sidx[j];
        const int64_t tb = a.tab[j];
        s_up[j] = (slot < 0 || slot >= a.nslots) ? nullptr : a.slots + slot * a.slot_bytes;
        s_dn[j] = (tb == 0 || (tb & 15)) ? nullptr : reinterpret_cast<const uint8_t *>(tb);
        s_s2u[j] = a.s2[2 * j];
        s_dmul[j] = a.coef[j] * a.s2[2 * j + 1];
    }
    __syncthreads();

    // x slice [32*lane, 32*lane+32) as f16x2 scaled by 2^E (amax*2^E in [256, 512))
    float xv[32];
    if (a.x_dtype == QMOE_DT_BF16 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0) {
        const uint4 *xp = reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(a.x) + 32 * lane);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 v = __ldg(xp + i);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                xv[8 * i + 2 * k] = __uint_as_float(w[k] << 16);
                xv[8 * i + 2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) xv[i] = load_act(a.x, a.x_dtype, 32 * lane + i);
    }
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) am = fmaxf(am, fabsf(xv[i]));
#pragma unroll
    for (int o = 16; o; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    const int E = prescale_exp(am, 9);
    const float pe = pow2f(E);
    uint32_t xr[16];
#pragma unroll
    for (int k = 0; k < 16; ++k)
        xr[k] = h2_as_u(__halves2half2(__float2half_rn(xv[2 * k] * pe), __float2half_rn(xv[2 * k + 1] * pe)));
    const float inv = pow2f(-E);

    // ================= phase 1: up GEMV over the CTA's half groups
    for (int sidx = warp; sidx < nhalf; sidx += NW) {
        const int q = blockIdx.x + (sidx >> 1) * G;
        const int j = q / G_DN, g = q - j * G_DN, hg = 2 * g + (sidx & 1);
        const uint8_t *ub = s_up[j];
        const float mult = s_s2u[j] * inv;
        uint4 wv[8];
        uint16_t sv[8];
        if (ub) {
            const uint8_t *wr = ub + O_UW + (int64_t)hg * (8 * KB_UP) + 16 * lane;
            const uint8_t *sr = ub + O_US + (int64_t)hg * (8 * G_UP) + 2 * lane;
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                wv[r] = ldg_stream(wr + r * KB_UP);
                sv[r] = __ldg(reinterpret_cast<const uint16_t *>(sr + r * G_UP));
            }
        }
        float part[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            const uint4 w = wv[r];
            __half2 a0 = __float2half2_rn(0.f), a1 = a0, b0 = a0, b1 = a0;
            uint32_t o[4];
            e2m1x8_f16x2(w.x, o);
            a0 = __hfma2(as_h2(o[0]), as_h2(xr[0]), a0);
            b0 = __hfma2(as_h2(o[1]), as_h2(xr[1]), b0);
            a0 = __hfma2(as_h2(o[2]), as_h2(xr[2]), a0);
            b0 = __hfma2(as_h2(o[3]), as_h2(xr[3]), b0);
            e2m1x8_f16x2(w.y, o);
            a0 = __hfma2(as_h2(o[0]), as_h2(xr[4]), a0);
            b0 = __hfma2(as_h2(o[1]), as_h2(xr[5]), b0);
            a0 = __hfma2(as_h2(o[2]), as_h2(xr[6]), a0);
            b0 = __hfma2(as_h2(o[3]), as_h2(xr[7]), b0);
            e2m1x8_f16x2(w.z, o);
            a1 = __hfma2(as_h2(o[0]), as_h2(xr[8]), a1);
            b1 = __hfma2(as_h2(o[1]), as_h2(xr[9]), b1);
            a1 = __hfma2(as_h2(o[2]), as_h2(xr[10]), a1);
            b1 = __hfma2(as_h2(o[3]), as_h2(xr[11]), b1);
            e2m1x8_f16x2(w.w, o);
            a1 = __hfma2(as_h2(o[0]), as_h2(xr[12]), a1);
            b1 = __hfma2(as_h2(o[1]), as_h2(xr[13]), b1);
            a1 = __hfma2(as_h2(o[2]), as_h2(xr[14]), a1);
            b1 = __hfma2(as_h2(o[3]), as_h2(xr[15]), b1);
            const float2 sf = __half22float2(as_h2(e4m3x2_f16x2(sv[r])));
            const float2 fa = __half22float2(__hadd2(a0, b0));
            const float2 fb = __half22float2(__hadd2(a1, b1));
            part[r] = (fa.x + fa.y) * sf.x + (fb.x + fb.y) * sf.y;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const bool up = lane & 16;
            const float send = up ? part[i] : part[i + 4];
            part[i] = (up ? part[i + 4] : part[i]) + __shfl_xor_sync(0xffffffffu, send, 16);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const bool up = lane & 8;
            const float send = up ? part[i] : part[i + 2];
            part[i] = (up ? part[i + 2] : part[i]) + __shfl_xor_sync(0xffffffffu, send, 8);
        }
        {
            const bool up = lane & 4;
            const float send = up ? part[0] : part[1];
            part[0] = (up ? part[1] : part[0]) + __shfl_xor_sync(0xffffffffu, send, 4);
        }
        part[0] += __shfl_xor_sync(0xffffffffu, part[0], 2);
        part[0] += __shfl_xor_sync(0xffffffffu, part[0], 1);
        const float u = fmaxf(part[0] * mult, 0.f);   // ReLU^2 (qmoe_ns.py:42-44)
        float hv = u * u;
        if (!ub) hv = __int_as_float(0x7fc00000);
        const bool lead = (lane & 3) == 0;
        if (lead) {
            a.h[(int64_t)j * INTER + hg * 8 + (lane >> 2)] = hv;
            hh[sidx * 8 + (lane >> 2)] = hv;
        }
        const unsigned m = __reduce_or_sync(0xffffffffu, (lead && (hv > 0.f || !ub)) ? (1u << (lane >> 2)) : 0u);
        if (lane == 0) {
            gmask8[(int64_t)j * (2 * G_DN) + hg] = (uint8_t)m;
            mk[sidx] = (int)m;
        }
    }
    __syncthreads();

    // ================= phase 2: down GEMV over the live neurons of the CTA's groups
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.f;
    for (int k = warp; k < my_groups; k += NW) {
        const unsigned mask = (unsigned)mk[2 * k] | ((unsigned)mk[2 * k + 1] << 8);   // 16 neurons of the group
        if (!mask) continue;
        const int q = blockIdx.x + k * G;
        const int j = q / G_DN, g = q - j * G_DN;
        const uint8_t *db = s_dn[j];
        if (!db) {
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[i] = __int_as_float(0x7fc00000);
            continue;
        }
        const float dmul = s_dmul[j];
        const uint8_t *srow = db + O_DS + (int64_t)g * LAT + 32 * lane;
        const uint4 s0 = __ldg(reinterpret_cast<const uint4 *>(srow));
        const uint4 s1 = __ldg(reinterpret_cast<const uint4 *>(srow + 16));
        unsigned mm = mask;
        bool first = true;
        uint32_t scl[16];
        while (mm) {
            uint4 dw[DNB];
            float hn[DNB];
            int cnt = 0;
#pragma unroll
            for (int b = 0; b < DNB; ++b) {
                hn[b] = 0.f;
                if (mm) {
                    const int i = __ffs(mm) - 1;
                    mm &= mm - 1;
                    const int n = 16 * g + i;
                    dw[b] = ldg_stream(db + O_DW + (int64_t)n * (LAT / 2) + 16 * lane);
                    hn[b] = hh[(2 * k + (i >> 3)) * 8 + (i & 7)] * dmul;
                    cnt = b + 1;
                }
            }
            if (first) {   // scales of this lane's 32 rows as f16x2 pairs (rows 2i, 2i+1)
                const uint32_t sw8[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
                for (int c = 0; c < 8; ++c) e4m3x4_f16x2(sw8[c], scl[2 * c], scl[2 * c + 1]);
                first = false;
            }
#pragma unroll
            for (int b = 0; b < DNB; ++b) {
                if (b >= cnt) break;
                const uint32_t ww[4] = {dw[b].x, dw[b].y, dw[b].z, dw[b].w};
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t o[4];
                    e2m1x8_f16x2(ww[c], o);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        // e2m1 * e4m3 is exact in f16
                        const float2 f = __half22float2(__hmul2(as_h2(o[e]), as_h2(scl[4 * c + e])));
                        acc[8 * c + 2 * e] = fmaf(f.x, hn[b], acc[8 * c + 2 * e]);
                        acc[8 * c + 2 * e + 1] = fmaf(f.y, hn[b], acc[8 * c + 2 * e + 1]);
                    }
                }
            }
        }
    }

    // ================= phase 3: CTA partial, grid barrier, distributed sum over CTAs
#pragma unroll
    for (int i = 0; i < 32; ++i) red[warp * LAT + 32 * lane + i] = acc[i];
    __syncthreads();
    for (int r = threadIdx.x; r < LAT; r += THREADS) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) v += red[w * LAT + r];
        partial[(int64_t)blockIdx.x * LAT + r] = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) s_ok = grid_barrier(reinterpret_cast<int *>(a.ws + WS_BAR), reinterpret_cast<int *>(a.ws + WS_BAR + 4), status);
    __syncthreads();
    if (!s_ok) return;
    for (int r = blockIdx.x + G * warp; r < LAT; r += G * NW) {
        float v = 0.f;
        for (int c = lane; c < G; c += 32) v += __ldcg(&partial[(int64_t)c * LAT + r]);
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) a.y[r] = v;
    }
    if (warp == 0) {
        for (int j = blockIdx.x; j < K; j += G) {
            int base = 0, total = 0;
            unsigned b[6];
            int m6[6];
#pragma unroll
            for (int c = 0; c < 6; ++c) {
                const int g = 32 * c + lane;
                m6[c] = g < G_DN ? (int)__ldcg(reinterpret_cast<const unsigned short *>(gmask8 + (int64_t)j * 2 * G_DN + 2 * g)) : 0;
                b[c] = __ballot_sync(0xffffffffu, m6[c] != 0);
                total += __popc(b[c]);
            }
#pragma unroll
            for (int c = 0; c < 6; ++c) {
                const int g = 32 * c + lane;
                const int rank = base + __popc(b[c] & ((1u << lane) - 1u));
                if (g < G_DN) a.gidx[(int64_t)j * G_DN + (m6[c] ? rank : total + (g - rank))] = g;
                base += __popc(b[c]);
            }
            if (lane == 0) a.gcnt[j] = total;
        }
    }
}

} // namespace fused

static std::atomic<uint64_t> g_fused_smem{0};

int launch_decode_fused(const fused::Args &a, cudaStream_t st) {
    int dev;
    DeviceInfo *di;
    if (int e = current_device(&dev, &di)) return e;
    int grid = di->sms;
    if (grid > fused::MAX_GRID) grid = fused::MAX_GRID;
    const int ngroups = a.K * G_DN;
    const int max_groups = (ngroups + grid - 1) / grid;
    const size_t smem = (size_t)fused::NW * LAT * sizeof(float) + (size_t)2 * max_groups * (8 * sizeof(float) + sizeof(int));
    if (!ensure_smem(fused::decode_layer_kernel, smem, dev, g_fused_smem)) return QMOE_ERR_LAUNCH;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(fused::THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, fused::decode_layer_kernel, a) != cudaSuccess) return QMOE_ERR_LAUNCH;
    return launch_status();
}

size_t decode_fused_ws_bytes(int K) { return fused::ws_bytes(K); }
int decode_fused_max_k() { return fused::MAXK; }

} // namespace qmoe
