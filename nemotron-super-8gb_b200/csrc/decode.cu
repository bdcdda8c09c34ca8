// Decode-step routed-expert kernels (bs = 1) for sm_100a.
//
//   decode_up_kernel    — `_up` (qmoe_ns.py:24-44): persistent CTAs; one producer thread streams 16-row
//                         tiles (8 KB codes + 1 KB scales, both contiguous in the block) into a 16-stage
//                         shared-memory ring with 1-D bulk copies (TMA engine) completing on mbarriers;
//                         eight consumer warps each own whole tiles, keep their 32-element slice of x in
//                         registers as prescaled f16x2, decode with cvt.e2m1x2 and reduce 16 rows with a
//                         16-shuffle butterfly. Fused epilogue: ReLU^2, and the tile (= one 16-neuron group)
//                         writes its 16-bit live-neuron mask, so no separate liveness pass is needed.
//   live_groups_kernel  — the torch glue of moe_decode_groups (qmoe_ns.py:249-251).
//   decode_down_kernel  — `_down_groups` (qmoe_ns.py:209-239) over the T layout: CTA = (expert, split,
//                         128-row chunk); compacts the live groups and live neurons into shared memory,
//                         streams 64 B of codes per live neuron and 128 B of scales per live group, and
//                         reduces the 64 neuron slots in a fixed order. In the fused form the last CTA of
//                         each chunk (arrival counter) sums the K experts in slot order into y, so the
//                         result is deterministic without float atomics.
#include "common.cuh"
#include "gemv.cuh"
#include "host.h"

namespace qmoe {

// ------------------------------------------------------------------ up
constexpr int UP_ROWS = 16;
constexpr int UP_TILE_W = UP_ROWS * KB_UP;       // 8192 B of codes
constexpr int UP_TILE_S = UP_ROWS * G_UP;        // 1024 B of scales
constexpr int UP_STAGE = UP_TILE_W + UP_TILE_S;  // 9216 B
constexpr int UP_CONSUMERS = 8;
constexpr int UP_THREADS = 32 * (UP_CONSUMERS + 1);
constexpr int UP_STAGES = 16;  // multiple of UP_CONSUMERS: stage s is always consumed by warp s % 8
constexpr size_t UP_SMEM = (size_t)UP_STAGES * UP_STAGE + 2 * UP_STAGES * sizeof(uint64_t);
static_assert(UP_STAGES % UP_CONSUMERS == 0, "stage/warp ownership");

struct UpArgs {
    const uint8_t *slots;
    int64_t slot_bytes;
    int64_t nslots;
    const int32_t *sidx;
    int K;
    const float *s2;
    const void *x;
    int x_dtype;
    float *h;
    uint16_t *gmask;    // [K, 168] live-neuron mask per group (nullable)
    int *status;        // device status word (nullable)
    int *zero_words;    // words to zero before the dependent kernel runs (nullable)
    int nzero;
};

__global__ void __launch_bounds__(UP_THREADS, 1) decode_up_kernel(UpArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)UP_STAGES * UP_STAGE);
    uint64_t *empty = full + UP_STAGES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = a.K * G_DN;  // 168 tiles of 16 rows per expert

    if (threadIdx.x == 0) {
        for (int s = 0; s < UP_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_mbar_init();
    }
    if (blockIdx.x == 0 && a.zero_words && (int)threadIdx.x < a.nzero) a.zero_words[threadIdx.x] = 0;
    __syncthreads();
    pdl_launch_dependents();

    if (warp == UP_CONSUMERS) {
        // ---------------- producer: one thread issues the bulk copies
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
                const int s = it % UP_STAGES;
                if (it >= UP_STAGES && !mbar_wait(&empty[s], ((it / UP_STAGES) & 1) ^ 1)) {
                    ok = false;
                    break;
                }
                const int j = t / G_DN, g = t - j * G_DN;
                int64_t slot = a.sidx[j];
                if (slot < 0 || slot >= a.nslots) slot = -1;
                uint8_t *dst = smem + (size_t)s * UP_STAGE;
                if (slot >= 0) {
                    const uint8_t *base = a.slots + slot * a.slot_bytes;
                    mbar_expect_tx(&full[s], UP_STAGE);
                    bulk_g2s(dst, base + O_UW + (int64_t)g * UP_TILE_W, UP_TILE_W, &full[s], pol);
                    bulk_g2s(dst + UP_TILE_W, base + O_US + (int64_t)g * UP_TILE_S, UP_TILE_S, &full[s], pol);
                } else {
                    mbar_arrive(&full[s]);  // bad slot: no copy; the consumer writes NaN
                }
            }
            if (!ok) set_error(a.status, DEV_ERR_TIMEOUT);
            // every copy this thread issued must land before the CTA exits
            const int n = it;
            for (int i = n > UP_STAGES ? n - UP_STAGES : 0; i < n; ++i)
                if (!mbar_wait(&full[i % UP_STAGES], (i / UP_STAGES) & 1)) set_error(a.status, DEV_ERR_TIMEOUT);
        }
        return;
    }

    // ---------------- consumers: x slice [32*lane, 32*lane+32) as prescaled f16x2 in registers
    float xv[32];
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        xv[i] = load_act(a.x, a.x_dtype, 32 * lane + i);
        am = fmaxf(am, fabsf(xv[i]));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    const int E = prescale_exp(am, 9);  // amax * 2^E in [256, 512): 16 products of |e2m1| <= 6 stay < 2^16
    uint32_t xr[16];
#pragma unroll
    for (int k = 0; k < 16; ++k)
        xr[k] = h2_as_u(__halves2half2(__float2half_rn(ldexpf(xv[2 * k], E)), __float2half_rn(ldexpf(xv[2 * k + 1], E))));
    const float inv = ldexpf(1.f, -E);

    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
        if ((it % UP_CONSUMERS) != warp) continue;
        const int s = it % UP_STAGES;
        if (!mbar_wait(&full[s], (it / UP_STAGES) & 1)) {
            set_error(a.status, DEV_ERR_TIMEOUT);
            break;
        }
        const int j = t / G_DN, g = t - j * G_DN;
        const int32_t slot = a.sidx[j];
        const bool bad = slot < 0 || (int64_t)slot >= a.nslots;
        const uint8_t *sw = smem + (size_t)s * UP_STAGE;
        const uint8_t *ss = sw + UP_TILE_W;
        float part[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            const uint4 w = *reinterpret_cast<const uint4 *>(sw + r * KB_UP + 16 * lane);
            const uint16_t sc = *reinterpret_cast<const uint16_t *>(ss + r * G_UP + 2 * lane);
            __half2 a0 = __float2half2_rn(0.f), a1 = __float2half2_rn(0.f);
            uint32_t o[4];
            e2m1x8_f16x2(w.x, o);
#pragma unroll
            for (int k = 0; k < 4; ++k) a0 = __hfma2(as_h2(o[k]), as_h2(xr[k]), a0);
            e2m1x8_f16x2(w.y, o);
#pragma unroll
            for (int k = 0; k < 4; ++k) a0 = __hfma2(as_h2(o[k]), as_h2(xr[4 + k]), a0);
            e2m1x8_f16x2(w.z, o);
#pragma unroll
            for (int k = 0; k < 4; ++k) a1 = __hfma2(as_h2(o[k]), as_h2(xr[8 + k]), a1);
            e2m1x8_f16x2(w.w, o);
#pragma unroll
            for (int k = 0; k < 4; ++k) a1 = __hfma2(as_h2(o[k]), as_h2(xr[12 + k]), a1);
            const float2 sf = __half22float2(as_h2(e4m3x2_f16x2(sc)));
            part[r] = h2sum_f32(a0) * sf.x + h2sum_f32(a1) * sf.y;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // the stage's bytes are in registers now

        // butterfly: 16 row partials over 32 lanes -> lanes 2r, 2r+1 hold row r
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const bool up = lane & 16;
            const float send = up ? part[i] : part[i + 8];
            const float keep = up ? part[i + 8] : part[i];
            part[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const bool up = lane & 8;
            const float send = up ? part[i] : part[i + 4];
            const float keep = up ? part[i + 4] : part[i];
            part[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const bool up = lane & 4;
            const float send = up ? part[i] : part[i + 2];
            const float keep = up ? part[i + 2] : part[i];
            part[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
        }
        {
            const bool up = lane & 2;
            const float send = up ? part[0] : part[1];
            const float keep = up ? part[1] : part[0];
            part[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
        }
        part[0] += __shfl_xor_sync(0xffffffffu, part[0], 1);

        float u = part[0] * (a.s2[2 * j] * inv);
        u = fmaxf(u, 0.f);
        float hv = u * u;
        if (bad) hv = __int_as_float(0x7fc00000);
        const bool even = (lane & 1) == 0;
        if (even) a.h[(int64_t)j * INTER + g * UP_ROWS + (lane >> 1)] = hv;
        if (a.gmask) {
            const unsigned m = __reduce_or_sync(0xffffffffu, (even && (hv > 0.f || bad)) ? (1u << (lane >> 1)) : 0u);
            if (lane == 0) a.gmask[(int64_t)j * G_DN + g] = (uint16_t)m;
        }
    }
}

// ------------------------------------------------------------------ live groups (qmoe_ns.py:249-251)
__global__ void __launch_bounds__(192) live_groups_kernel(const float *__restrict__ h, int32_t *__restrict__ gidx,
                                                          int32_t *__restrict__ gcnt) {
    __shared__ int wsum[6];
    const int j = blockIdx.x, g = threadIdx.x, warp = g >> 5, lane = g & 31;
    int live = 0;
    if (g < G_DN) {
        const float4 *p = reinterpret_cast<const float4 *>(h + (int64_t)j * INTER + 16 * g);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 v = p[i];
            live |= (v.x > 0.f) | (v.y > 0.f) | (v.z > 0.f) | (v.w > 0.f);
        }
    }
    const unsigned b = __ballot_sync(0xffffffffu, live);
    if (lane == 0) wsum[warp] = __popc(b);
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < 6; ++w) {
        if (w < warp) before += wsum[w];
        total += wsum[w];
    }
    const int rank = before + __popc(b & ((1u << lane) - 1u));  // live groups before g
    if (g < G_DN) {
        const int pos = live ? rank : total + (g - rank);
        gidx[(int64_t)j * G_DN + pos] = g;
    }
    if (g == 0) gcnt[j] = total;
}

// ------------------------------------------------------------------ down over live groups (T layout)
constexpr int DN_THREADS = 256;
constexpr int DN_CHUNK = 128;                  // output rows per CTA
constexpr int DN_NCHUNK = LAT / DN_CHUNK;      // 8
constexpr int DN_SLOTS = DN_THREADS / 4;       // 64 neuron slots (4 threads x 16 B = 64 B of a neuron's row chunk)
constexpr int DN_RED_LD = DN_THREADS + 1;
constexpr size_t DN_SMEM = (size_t)INTER * 4 * 2 + (size_t)32 * DN_RED_LD * 4 + (size_t)G_DN * 8 + 64;

struct DownArgs {
    const int64_t *tab;
    const float *h;
    const uint16_t *gmask;   // fused: live masks from the up kernel
    const int32_t *gidx_in;  // reference form
    const int32_t *gcnt_in;
    const float *s2;
    const float *coef;
    int K, KS;
    float *part;        // reference form: [KS, K, 1024]; fused: [K, 1024]
    int32_t *gidx_out;  // fused: written by the chunk-0 CTA of each expert
    int32_t *gcnt_out;
    float *y;           // fused: [1024]
    int *counters;      // fused: [DN_NCHUNK] arrival counters (zeroed by the up kernel)
    int *status;
};

template <bool FUSED>
__global__ void __launch_bounds__(DN_THREADS) decode_down_kernel(DownArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    int *nl = reinterpret_cast<int *>(smem);                       // live neuron ids
    float *hv = reinterpret_cast<float *>(smem + INTER * 4);       // their h
    float *red = reinterpret_cast<float *>(smem + INTER * 8);      // [32][257]
    int *gl = reinterpret_cast<int *>(smem + INTER * 8 + 32 * DN_RED_LD * 4);  // listed groups
    int *gm = gl + G_DN;                                           // their live masks
    __shared__ int s_wsum[8];
    __shared__ int s_ng, s_last;

    const int rc = blockIdx.x, sp = blockIdx.y, j = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    pdl_wait();  // the up kernel's h / masks are complete and visible

    const uint8_t *blk = reinterpret_cast<const uint8_t *>(a.tab[j]);
    const bool bad = (reinterpret_cast<uintptr_t>(blk) & 15u) != 0 || blk == nullptr;

    // ---- 1. groups handled by this CTA, with their live-neuron masks
    if (FUSED) {
        if (warp == 0) {
            int base = 0;
            unsigned b[6];
            int m[6];
#pragma unroll
            for (int c = 0; c < 6; ++c) {
                const int g = 32 * c + lane;
                m[c] = g < G_DN ? (int)a.gmask[(int64_t)j * G_DN + g] : 0;
                b[c] = __ballot_sync(0xffffffffu, m[c] != 0);
            }
            int total = 0;
#pragma unroll
            for (int c = 0; c < 6; ++c) total += __popc(b[c]);
#pragma unroll
            for (int c = 0; c < 6; ++c) {
                const int g = 32 * c + lane;
                const int rank = base + __popc(b[c] & ((1u << lane) - 1u));
                if (m[c]) {
                    gl[rank] = g;
                    gm[rank] = m[c];
                }
                if (rc == 0 && g < G_DN) a.gidx_out[(int64_t)j * G_DN + (m[c] ? rank : total + (g - rank))] = g;
                base += __popc(b[c]);
            }
            if (lane == 0) {
                s_ng = total;
                if (rc == 0) a.gcnt_out[j] = total;
            }
        }
    } else {
        int gc = a.gcnt_in[j];
        gc = gc < 0 ? 0 : (gc > G_DN ? G_DN : gc);   // caller data: never index past the [K,168] list
        const int ng = gc > sp ? (gc - sp + a.KS - 1) / a.KS : 0;
        if (tid < ng) {
            const int g = a.gidx_in[(int64_t)j * G_DN + sp + tid * a.KS];
            int m = 0;
            if (g >= 0 && g < G_DN) {
                const float *hp = a.h + (int64_t)j * INTER + 16 * g;
#pragma unroll
                for (int i = 0; i < 16; ++i) m |= (hp[i] > 0.f) ? (1 << i) : 0;
            }
            gl[tid] = g;
            gm[tid] = m;   // an out-of-range group id contributes nothing
        }
        if (tid == 0) s_ng = ng;
    }
    __syncthreads();
    const int ng = s_ng;

    // ---- 2. compact live neurons of the listed groups (exclusive scan of the mask popcounts)
    const int cnt = tid < ng ? __popc(gm[tid]) : 0;
    int inc = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
    }
    if (lane == 31) s_wsum[warp] = inc;
    __syncthreads();
    int off = inc - cnt, L = 0;
    for (int w = 0; w < DN_THREADS / 32; ++w) {
        if (w < warp) off += s_wsum[w];
        L += s_wsum[w];
    }
    if (tid < ng) {
        int m = gm[tid];
        const int g = gl[tid];
        while (m) {
            const int i = __ffs(m) - 1;
            m &= m - 1;
            const int n = 16 * g + i;
            nl[off] = n;
            hv[off] = a.h[(int64_t)j * INTER + n];
            ++off;
        }
    }
    __syncthreads();

    // ---- 3. stream live neurons: thread (p = tid/4, q = tid%4) covers rows rc*128 + q*32 + [0,32)
    const int q = tid & 3, p = tid >> 2;
    float acc[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) acc[k] = 0.f;
    if (!bad) {
        const uint8_t *wb = blk + O_DW + rc * (DN_CHUNK / 2) + q * 16;
        const uint8_t *sb = blk + O_DS + rc * DN_CHUNK + q * 32;
        int i = p;
        uint4 wv, s0, s1;
        float hn = 0.f;
        if (i < L) {
            const int n = nl[i];
            hn = hv[i];
            wv = ldg_stream(wb + (int64_t)n * (LAT / 2));
            s0 = __ldg(reinterpret_cast<const uint4 *>(sb + (int64_t)(n >> 4) * LAT));
            s1 = __ldg(reinterpret_cast<const uint4 *>(sb + (int64_t)(n >> 4) * LAT + 16));
        }
        while (i < L) {
            const int inext = i + DN_SLOTS;
            uint4 wn, t0, t1;
            float hnn = 0.f;
            if (inext < L) {  // prefetch the next neuron of this slot
                const int n = nl[inext];
                hnn = hv[inext];
                wn = ldg_stream(wb + (int64_t)n * (LAT / 2));
                t0 = __ldg(reinterpret_cast<const uint4 *>(sb + (int64_t)(n >> 4) * LAT));
                t1 = __ldg(reinterpret_cast<const uint4 *>(sb + (int64_t)(n >> 4) * LAT + 16));
            }
            const uint32_t *ww = reinterpret_cast<const uint32_t *>(&wv);
            const uint32_t *sw0 = reinterpret_cast<const uint32_t *>(&s0);
            const uint32_t *sw1 = reinterpret_cast<const uint32_t *>(&s1);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                uint32_t o[4];
                e2m1x8_f16x2(ww[k], o);  // rows 8k .. 8k+7 of this thread's 32
                uint32_t slo, shi;
                e4m3x4_f16x2(k < 2 ? sw0[2 * k] : sw1[2 * (k - 2)], slo, shi);        // scales rows 8k..8k+3
                uint32_t slo2, shi2;
                e4m3x4_f16x2(k < 2 ? sw0[2 * k + 1] : sw1[2 * (k - 2) + 1], slo2, shi2);  // rows 8k+4..8k+7
                const uint32_t sc[4] = {slo, shi, slo2, shi2};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    // e2m1 * e4m3 is exact in f16
                    const float2 f = __half22float2(__hmul2(as_h2(o[e]), as_h2(sc[e])));
                    acc[8 * k + 2 * e] = fmaf(f.x, hn, acc[8 * k + 2 * e]);
                    acc[8 * k + 2 * e + 1] = fmaf(f.y, hn, acc[8 * k + 2 * e + 1]);
                }
            }
            i = inext;
            wv = wn;
            s0 = t0;
            s1 = t1;
            hn = hnn;
        }
    }

    // ---- 4. fixed-order reduction over the 64 neuron slots
#pragma unroll
    for (int k = 0; k < 32; ++k) red[k * DN_RED_LD + tid] = acc[k];
    __syncthreads();
    float out = 0.f;
    if (tid < DN_CHUNK) {
        const int qq = tid >> 5, k = tid & 31;
        float v = 0.f;
        for (int pp = 0; pp < DN_SLOTS; ++pp) v += red[k * DN_RED_LD + 4 * pp + qq];
        out = v * (a.coef[j] * a.s2[2 * j + 1]);
        if (bad) out = __int_as_float(0x7fc00000);
    }
    const int row = rc * DN_CHUNK + tid;
    if (!FUSED) {
        if (tid < DN_CHUNK) a.part[((int64_t)sp * a.K + j) * LAT + row] = out;
        return;
    }
    if (bad) set_error(a.status, QMOE_ERR_ALIGN);
    if (tid < DN_CHUNK) a.part[(int64_t)j * LAT + row] = out;
    // ---- 5. last CTA of this chunk sums the K experts in slot order
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&a.counters[rc], 1) == a.K - 1;
    __syncthreads();
    if (s_last) {
        __threadfence();
        if (tid < DN_CHUNK) {
            float v = 0.f;
            for (int jj = 0; jj < a.K; ++jj) v += __ldcg(&a.part[(int64_t)jj * LAT + row]);
            a.y[row] = v;
        }
        if (tid == 0) a.counters[rc] = 0;
    }
}

// ------------------------------------------------------------------ sum over experts (orig-layout path)
__global__ void sum_rows_kernel(const float *__restrict__ out, int K, float *__restrict__ y) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= LAT) return;
    float v = 0.f;
    for (int j = 0; j < K; ++j) v += out[(int64_t)j * LAT + r];
    y[r] = v;
}

// ------------------------------------------------------------------ host launchers
static std::atomic<uint64_t> g_up_smem{0}, g_dn_smem_f{0}, g_dn_smem_r{0};

static int launch_up(const UpArgs &a, cudaStream_t st, int dev, const DeviceInfo &di) {
    if (!ensure_smem(decode_up_kernel, UP_SMEM, dev, g_up_smem)) return QMOE_ERR_LAUNCH;
    const int ntiles = a.K * G_DN;
    const int grid = ntiles < di.sms ? ntiles : di.sms;
    decode_up_kernel<<<grid, UP_THREADS, UP_SMEM, st>>>(a);
    return launch_status();
}

template <bool FUSED>
static int launch_down(const DownArgs &a, cudaStream_t st, int dev, bool pdl) {
    auto kern = decode_down_kernel<FUSED>;
    if (!ensure_smem(kern, DN_SMEM, dev, FUSED ? g_dn_smem_f : g_dn_smem_r)) return QMOE_ERR_LAUNCH;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(DN_NCHUNK, FUSED ? 1 : a.KS, a.K);
    cfg.blockDim = dim3(DN_THREADS);
    cfg.dynamicSmemBytes = DN_SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, kern, a) != cudaSuccess) return QMOE_ERR_LAUNCH;
    return launch_status();
}

// Workspace of qmoe_decode_groups: [status int][pad to 64][counters DN_NCHUNK ints][pad][gmask K*168 u16]
constexpr size_t WS_STATUS = 0;
constexpr size_t WS_COUNTERS = 64;
constexpr size_t WS_GMASK = 256;

} // namespace qmoe

using namespace qmoe;

extern "C" {

int qmoe_decode_up(const uint8_t *slots, int64_t slot_bytes, int64_t nslots, const int32_t *sidx, int K,
                   const float *s2, const void *x, int x_dtype, float *h, void *stream) {
    if (!slots || !sidx || !s2 || !x || !h) return QMOE_ERR_NULL;
    if (K < 1 || K > QMOE_MAX_K || nslots < 1) return QMOE_ERR_SHAPE;
    if (slot_bytes < UPB || (slot_bytes & 15) || !aligned16(slots)) return QMOE_ERR_ALIGN;
    if (!valid_dtype(x_dtype)) return QMOE_ERR_DTYPE;
    int dev;
    DeviceInfo *di;
    if (int e = current_device(&dev, &di)) return e;
    UpArgs a{slots, slot_bytes, nslots, sidx, K, s2, x, x_dtype, h, nullptr, nullptr, nullptr, 0};
    return launch_up(a, as_stream(stream), dev, *di);
}

int qmoe_live_groups(const float *h, int K, int32_t *gidx, int32_t *gcnt, void *stream) {
    if (!h || !gidx || !gcnt) return QMOE_ERR_NULL;
    if (K < 1 || K > QMOE_MAX_K) return QMOE_ERR_SHAPE;
    if (!aligned16(h)) return QMOE_ERR_ALIGN;
    if (int e = current_device(nullptr, nullptr)) return e;
    live_groups_kernel<<<K, 192, 0, as_stream(stream)>>>(h, gidx, gcnt);
    return launch_status();
}

int qmoe_decode_down_groups(const int64_t *tab, const float *h, const int32_t *gidx, const int32_t *gcnt,
                            const float *s2, const float *coef, int K, int KS, float *part, void *stream) {
    if (!tab || !h || !gidx || !gcnt || !s2 || !coef || !part) return QMOE_ERR_NULL;
    if (K < 1 || K > QMOE_MAX_K || KS < 1 || KS > 8) return QMOE_ERR_SHAPE;
    int dev;
    if (int e = current_device(&dev, nullptr)) return e;
    DownArgs a{tab, h, nullptr, gidx, gcnt, s2, coef, K, KS, part, nullptr, nullptr, nullptr, nullptr, nullptr};
    return launch_down<false>(a, as_stream(stream), dev, false);
}

size_t qmoe_decode_groups_workspace_bytes(int K) {
    if (K < 1 || K > QMOE_MAX_K) return 0;
    return WS_GMASK + (size_t)K * G_DN * sizeof(uint16_t);
}

int qmoe_decode_groups(const uint8_t *slots_up, int64_t slot_bytes, int64_t nslots, const int32_t *sidx,
                       const int64_t *tab, const float *s2, const float *coef, const void *x, int x_dtype, int K,
                       float *h, int32_t *gidx, int32_t *gcnt, float *part, float *y, void *workspace,
                       size_t workspace_bytes, void *stream) {
    if (!slots_up || !sidx || !tab || !s2 || !coef || !x || !h || !gidx || !gcnt || !part || !y || !workspace)
        return QMOE_ERR_NULL;
    if (K < 1 || K > QMOE_MAX_K || nslots < 1) return QMOE_ERR_SHAPE;
    if (slot_bytes < UPB || (slot_bytes & 15) || !aligned16(slots_up) || !aligned16(workspace)) return QMOE_ERR_ALIGN;
    if (!valid_dtype(x_dtype)) return QMOE_ERR_DTYPE;
    if (workspace_bytes < qmoe_decode_groups_workspace_bytes(K)) return QMOE_ERR_WORKSPACE;
    int dev;
    DeviceInfo *di;
    if (int e = current_device(&dev, &di)) return e;
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    int *status = reinterpret_cast<int *>(ws + WS_STATUS);
    int *counters = reinterpret_cast<int *>(ws + WS_COUNTERS);
    uint16_t *gmask = reinterpret_cast<uint16_t *>(ws + WS_GMASK);
    cudaStream_t st = as_stream(stream);
    UpArgs ua{slots_up, slot_bytes, nslots, sidx, K, s2, x, x_dtype, h, gmask, status, counters, DN_NCHUNK};
    if (int e = launch_up(ua, st, dev, *di)) return e;
    DownArgs da{tab, h, gmask, nullptr, nullptr, s2, coef, K, 1, part, gidx, gcnt, y, counters, status};
    return launch_down<true>(da, st, dev, true);
}

int qmoe_decode(const uint8_t *slots, int64_t slot_bytes, int64_t nslots, const int32_t *sidx, const float *s2,
                const float *coef, const void *x, int x_dtype, int K, float *h, float *out, float *y, void *stream) {
    if (!slots || !sidx || !s2 || !coef || !x || !h || !out || !y) return QMOE_ERR_NULL;
    if (K < 1 || K > QMOE_MAX_K || nslots < 1) return QMOE_ERR_SHAPE;
    if (slot_bytes < BLOCK || (slot_bytes & 15) || !aligned16(slots)) return QMOE_ERR_ALIGN;
    if (!valid_dtype(x_dtype)) return QMOE_ERR_DTYPE;
    int dev;
    DeviceInfo *di;
    if (int e = current_device(&dev, &di)) return e;
    cudaStream_t st = as_stream(stream);
    UpArgs ua{slots, slot_bytes, nslots, sidx, K, s2, x, x_dtype, h, nullptr, nullptr, nullptr, 0};
    if (int e = launch_up(ua, st, dev, *di)) return e;
    GemvArgs g{};
    g.slots = slots;
    g.slot_bytes = slot_bytes;
    g.nslots = nslots;
    g.sidx = sidx;
    g.s2 = s2;
    g.coef = coef;
    g.hin = h;
    g.y = out;
    g.M = 1;
    g.N = LAT;
    g.K = INTER;
    static std::atomic<uint64_t> smem_done{0};
    auto kern = gemv_kernel<1, GM_EXPERT_DOWN, 3, 1>;
    const size_t smem = gemv_smem_bytes(1, 1, INTER);
    if (!ensure_smem(kern, smem, dev, smem_done)) return QMOE_ERR_LAUNCH;
    const int rows = 64;
    kern<<<dim3(LAT / rows, K), GEMV_THREADS, smem, st>>>(g, rows);
    if (int e = launch_status()) return e;
    sum_rows_kernel<<<LAT / 256, 256, 0, st>>>(out, K, y);
    return launch_status();
}

int qmoe_pairs(const uint8_t *slots, int64_t slot_bytes, int64_t nslots, const int32_t *pslot, const int32_t *ptok,
               const float *s2p, const float *coefp, const void *X, int x_dtype, int T, int P, float *h, float *out,
               void *stream) {
    if (!slots || !pslot || !ptok || !s2p || !coefp || !X || !h || !out) return QMOE_ERR_NULL;
    if (P < 0 || T < 1 || nslots < 1) return QMOE_ERR_SHAPE;
    if (slot_bytes < BLOCK || (slot_bytes & 15) || !aligned16(slots)) return QMOE_ERR_ALIGN;
    if (!valid_dtype(x_dtype)) return QMOE_ERR_DTYPE;
    if (P == 0) return QMOE_OK;
    if (P > 65535) return QMOE_ERR_SHAPE;
    int dev;
    if (int e = current_device(&dev, nullptr)) return e;
    cudaStream_t st = as_stream(stream);
    GemvArgs g{};
    g.slots = slots;
    g.slot_bytes = slot_bytes;
    g.nslots = nslots;
    g.sidx = pslot;
    g.ptok = ptok;
    g.s2 = s2p;
    g.coef = coefp;
    g.x = X;
    g.x_dtype = x_dtype;
    g.T = T;
    g.hout = h;
    g.M = 1;
    g.N = INTER;
    g.K = LAT;
    static std::atomic<uint64_t> up_done{0}, dn_done{0};
    auto kup = gemv_kernel<1, GM_PAIR_UP, 1, 1>;
    const size_t smem_up = gemv_smem_bytes(1, 1, LAT);
    if (!ensure_smem(kup, smem_up, dev, up_done)) return QMOE_ERR_LAUNCH;
    kup<<<dim3(INTER / 128, P), GEMV_THREADS, smem_up, st>>>(g, 128);
    if (int e = launch_status()) return e;
    GemvArgs d = g;
    d.hin = h;
    d.y = out;
    d.N = LAT;
    d.K = INTER;
    auto kdn = gemv_kernel<1, GM_PAIR_DOWN, 3, 1>;
    const size_t smem_dn = gemv_smem_bytes(1, 1, INTER);
    if (!ensure_smem(kdn, smem_dn, dev, dn_done)) return QMOE_ERR_LAUNCH;
    kdn<<<dim3(LAT / 64, P), GEMV_THREADS, smem_dn, st>>>(d, 64);
    return launch_status();
}

} // extern "C"
