// Decode-step routed-expert kernels (bs = 1) for sm_100a. Every sum is fp32, as in the reference's kernels.
//
//   decode_layer_kernel — `moe_decode_groups` (qmoe_ns.py:245-255) for K <= SMs, one kernel per layer: each expert's
//                         neurons split over a cluster of S CTAs; a CTA streams its up rows (`_up`, qmoe_ns.py:24-44),
//                         keeps h and the live masks on chip and adds its own live neurons' down rows (`_down_groups`,
//                         qmoe_ns.py:209-239, T layout); the cluster's sums meet in rank 0 over distributed shared
//                         memory, which writes part[j] and the expert's live-group lists (qmoe_ns.py:249-251).
//   decode_finish_kernel — its programmatic dependent: y = the experts' outputs summed in slot order.
//   decode_up_kernel    — `_up` alone (qmoe_decode_up, qmoe_decode, and the layer for K above the SM count): one CTA
//                         per SM, 12 warps; a warp takes whole 8-row tiles, a lane 16 B of each row and a 32-element
//                         slice of x, the next tile's loads in flight during the current tile's math; ReLU^2, h and
//                         the tile's 8-bit live-neuron mask; live neurons' down rows prefetched to L2.
//   live_groups_kernel  — the torch glue of moe_decode_groups (qmoe_ns.py:249-251).
//   decode_down_kernel  — `_down_groups` over the T layout for the reference form (qmoe_decode_down_groups, KS splits)
//                         and for the layer above the SM count: CTA = (128-row chunk, split, expert); live neurons
//                         compacted into shared memory; in the fused form the last CTA of each chunk (arrival counter)
//                         sums the K experts in slot order into y.
#include "common.cuh"
#include "gemv.cuh"
#include "host.h"

namespace qmoe {

// ------------------------------------------------------------------ up
constexpr int UP_ROWS = 8;                          // rows per tile: half of a 16-neuron group
constexpr int UP_HALVES = INTER / UP_ROWS;          // 336 tiles per expert
constexpr int UP_NW = 12;                           // warps per CTA (one CTA per SM)
constexpr int UP_THREADS = 32 * UP_NW;
constexpr int UP_MAXK = 64;                         // experts whose metadata is staged in shared memory

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
    uint8_t *gmask8;    // [K, 336] live-neuron mask per 8-row half group (nullable)
    int *status;        // device status word (nullable)
    int *zero_words;    // words zeroed for the dependent kernel (nullable)
    int nzero;
    const int64_t *tab; // T-layout blocks the down kernel reads (nullable): live rows are prefetched to L2
};

struct UpTile {      // one lane's share of an 8-row tile: 16 B of codes and 2 scale bytes per row
    uint4 w[UP_ROWS];
    uint16_t sc[UP_ROWS];
};

// A lane's slice [32*lane, 32*lane+32) of x: as f16x2 scaled by 2^E (bf16 / f16 activations, exact) or as
// fp32 pairs (fp32 activations, kept exact).
template <bool XF32>
struct UpX {
    uint32_t h[16];
};
template <>
struct UpX<true> {
    float2 f[16];
};

__device__ __forceinline__ void up_load(const uint8_t *base, int hg, int lane, UpTile &T) {
    const uint8_t *wr = base + O_UW + (int64_t)hg * (UP_ROWS * KB_UP) + 16 * lane;
    const uint8_t *sr = base + O_US + (int64_t)hg * (UP_ROWS * G_UP) + 2 * lane;
#pragma unroll
    for (int r = 0; r < UP_ROWS; ++r) {
        T.w[r] = ldg_stream(wr + r * KB_UP);
        T.sc[r] = __ldg(reinterpret_cast<const uint16_t *>(sr + r * G_UP));
    }
}

// One row's partial for a lane: its two 16-element groups (codes of words x, y and of words z, w), each summed
// in fp32 from exact e2m1 * x products (fma.rn.f32.f16, or f32 FMAs for fp32 x), times its e4m3 scale.
template <bool XF32>
__device__ __forceinline__ float up_row(const uint4 w, uint16_t sc, const UpX<XF32> &x) {
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    float g[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t o[4];
        e2m1x8_f16x2(ww[q], o);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            if constexpr (XF32) {
                const float2 c = __half22float2(as_h2(o[e]));
                g[q >> 1][0] = fmaf(c.x, x.f[4 * q + e].x, g[q >> 1][0]);
                g[q >> 1][1] = fmaf(c.y, x.f[4 * q + e].y, g[q >> 1][1]);
            } else {
                fma2_f16_f32(o[e], x.h[4 * q + e], g[q >> 1][0], g[q >> 1][1]);
            }
        }
    }
    const float2 sf = __half22float2(as_h2(e4m3x2_f16x2(sc)));
    return (g[0][0] + g[0][1]) * sf.x + (g[1][0] + g[1][1]) * sf.y;
}

// The 8 row dot products of a tile: each lane's two fp32 group partials per row, reduced over the warp by a
// 9-shuffle butterfly; lanes 4r .. 4r+3 return row r (unscaled).
template <bool XF32>
__device__ __forceinline__ float up_tile_dot(const UpTile &cur, const UpX<XF32> &x, int lane) {
    float part[UP_ROWS];
#pragma unroll
    for (int r = 0; r < UP_ROWS; ++r) part[r] = up_row<XF32>(cur.w[r], cur.sc[r], x);
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
    return part[0];
}

// One 8-row tile of `_up` (qmoe_ns.py:24-44) from a lane's share of its codes and scales: per row the lane's two
// 16-element groups in fp32 (as the reference accumulates), a 9-shuffle butterfly over the 8 rows, then ReLU^2,
// h, the tile's 8-bit live-neuron mask and the L2 prefetch of the live neurons' down rows.
template <bool XF32>
__device__ __forceinline__ void up_tile(const UpArgs &a, const UpTile &cur, int j, int hg, float mult, bool bad,
                                        const UpX<XF32> &x, int lane, const uint8_t *const *s_tab) {
    const float u = fmaxf(up_tile_dot<XF32>(cur, x, lane) * mult, 0.f);   // ReLU^2 (qmoe_ns.py:42-44)
    float hv = u * u;
    if (bad) hv = __int_as_float(0x7fc00000);
    const bool lead = (lane & 3) == 0;
    if (lead) a.h[(int64_t)j * INTER + hg * UP_ROWS + (lane >> 2)] = hv;
    if (a.gmask8 || a.tab) {
        const unsigned m = __reduce_or_sync(0xffffffffu, (lead && (hv > 0.f || bad)) ? (1u << (lane >> 2)) : 0u);
        if (a.gmask8 && lane == 0) a.gmask8[(int64_t)j * UP_HALVES + hg] = (uint8_t)m;
        // The down kernel reads, per live neuron, its 512-byte row of dnT_w and, per live group, the
        // group's 1024-byte row of dnT_s: start bringing them into L2 now, while the up stream runs.
        const uint8_t *tb = a.tab ? (j < UP_MAXK ? s_tab[j] : reinterpret_cast<const uint8_t *>(a.tab[j])) : nullptr;
        // a null or unaligned block address is the down kernel's error case: nothing to bring in
        if (tb && (reinterpret_cast<uintptr_t>(tb) & 15u) == 0 && !bad && m) {
            if (lead && hv > 0.f) {
                const uint8_t *row = tb + O_DW + (int64_t)(hg * UP_ROWS + (lane >> 2)) * (LAT / 2);
#pragma unroll
                for (int l = 0; l < 4; ++l) prefetch_l2(row + 128 * l);
            }
            if (lane >= 24) prefetch_l2(tb + O_DS + (int64_t)(hg >> 1) * LAT + 128 * (lane - 24));
        }
    }
}

// A lane's 32-element slice [32*lane, 32*lane+32) of x. bf16 / f16: as f16x2 scaled by 2^E with amax*2^E in
// [256, 512) (exact: a bf16 or f16 value scaled by a power of two stays an f16 value), inv = 2^-E. fp32: as is.
template <bool XF32>
__device__ __forceinline__ void up_prep_x(const UpArgs &a, int lane, UpX<XF32> &x, float &inv) {
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
    if constexpr (XF32) {
#pragma unroll
        for (int k = 0; k < 16; ++k) x.f[k] = make_float2(xv[2 * k], xv[2 * k + 1]);
        inv = 1.f;
    } else {
        float am = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) am = fmaxf(am, fabsf(xv[i]));
#pragma unroll
        for (int o = 16; o; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
        const int E = prescale_exp(am, 9);
        const float pe = pow2f(E);
#pragma unroll
        for (int k = 0; k < 16; ++k)
            x.h[k] = h2_as_u(__halves2half2(__float2half_rn(xv[2 * k] * pe), __float2half_rn(xv[2 * k + 1] * pe)));
        inv = pow2f(-E);
    }
}

struct UpRef {   // where a tile's data lives: expert j, half group hg, block base (nullptr: bad slot), multiplier
    int j, hg;
    const uint8_t *base;
    float mult;
};

// `_up` (qmoe_ns.py:24-44) for bs = 1. One CTA per SM of 12 warps; warp w of CTA c takes tiles c + (w + 12k)*grid
// (tile = 8 rows). A lane owns a 32-element slice of x and 16 bytes of each row of a tile; the loads of the
// warp's next tile are issued before the current tile is computed (two tiles of codes in flight per lane), so
// the fp32 arithmetic overlaps the stream. Epilogue: ReLU^2, h, and the tile's 8-bit live-neuron mask for the
// down kernel. (Measured on B200 with 22 experts: fp32 accumulation at 12 warps with the next tile in flight runs
// as fast as f16 group sums did at 16 warps without it; 16 and 24 warps, or no look-ahead, are 1.5-4 us slower.)
template <bool XF32>
__global__ void __launch_bounds__(UP_THREADS, 1) decode_up_kernel(UpArgs a) {
    __shared__ const uint8_t *s_base[UP_MAXK];   // slot base of expert j (nullptr: slot out of range)
    __shared__ float s_s2u[UP_MAXK];
    __shared__ const uint8_t *s_tab[UP_MAXK];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = a.K * UP_HALVES;
    // Launched as a programmatic dependent of the previous layer's kernels: everything below may read their
    // outputs (sidx, x) or rewrite buffers they still read (the workspace counters), so wait first.
    pdl_wait();
    for (int j = threadIdx.x; j < a.K && j < UP_MAXK; j += blockDim.x) {
        const int64_t slot = a.sidx[j];
        s_base[j] = (slot < 0 || slot >= a.nslots) ? nullptr : a.slots + slot * a.slot_bytes;
        s_s2u[j] = a.s2[2 * j];
        s_tab[j] = a.tab ? reinterpret_cast<const uint8_t *>(a.tab[j]) : nullptr;
    }
    if (blockIdx.x == 0 && a.zero_words && (int)threadIdx.x < a.nzero) a.zero_words[threadIdx.x] = 0;
    __syncthreads();
    pdl_launch_dependents();

    UpX<XF32> x;
    float inv;
    up_prep_x<XF32>(a, lane, x, inv);

    auto ref = [&](int t) {
        UpRef r;
        r.j = t / UP_HALVES;
        r.hg = t - r.j * UP_HALVES;
        if (r.j < UP_MAXK) {
            r.base = s_base[r.j];
            r.mult = s_s2u[r.j] * inv;
        } else {
            const int64_t slot = a.sidx[r.j];
            r.base = (slot < 0 || slot >= a.nslots) ? nullptr : a.slots + slot * a.slot_bytes;
            r.mult = a.s2[2 * r.j] * inv;
        }
        return r;
    };
    const int tstep = UP_NW * gridDim.x;
    int t = blockIdx.x + warp * gridDim.x;
    UpRef rn{};
    UpTile tn;
    if (t < ntiles) {
        rn = ref(t);
        if (rn.base) up_load(rn.base, rn.hg, lane, tn);
    }
    for (; t < ntiles; t += tstep) {
        const UpRef rc = rn;
        const UpTile tc = tn;
        if (t + tstep < ntiles) {   // the next tile's loads go out before this tile's math
            rn = ref(t + tstep);
            if (rn.base) up_load(rn.base, rn.hg, lane, tn);
        }
        up_tile<XF32>(a, tc, rc.j, rc.hg, rc.mult, rc.base == nullptr, x, lane, s_tab);
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
constexpr int DN_NB = 4;                       // neurons per thread with all loads in flight at once
constexpr int DN_RED_LD = DN_THREADS + 1;
constexpr size_t DN_SMEM = (size_t)INTER * 4 + (size_t)32 * DN_RED_LD * 4;

struct DownArgs {
    const int64_t *tab;
    const float *h;
    const uint8_t *gmask8;   // fused form: half-group live masks from the up kernel
    const int32_t *gidx_in;  // reference form
    const int32_t *gcnt_in;
    const float *s2;
    const float *coef;
    int K, KS;
    float *part;        // reference form: [KS, K, 1024]; fused form: [K, 1024] per-expert outputs
    int32_t *gidx_out;  // fused form: written by the chunk-0 CTA of each expert
    int32_t *gcnt_out;
    float *y;           // fused form: [1024]
    int *counters;      // fused form: [DN_NCHUNK] arrival counters (zeroed by the up kernel)
    int *status;
};

// One CTA = (128-row chunk rc, split sp, expert j). Warp 0 lists the live neurons of the CTA's groups
// (ascending) in shared memory; then thread (p, q) takes neurons p, p+64, ... and output rows
// rc*128 + 32q .. +31, loading for up to DN_NB neurons at once 16 B of codes, 32 B of the group's
// scales and h before computing, so a batch costs one memory round trip.
template <bool FUSED>
__global__ void __launch_bounds__(DN_THREADS) decode_down_kernel(DownArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    int *nl = reinterpret_cast<int *>(smem);                       // live neuron ids
    float *red = reinterpret_cast<float *>(smem + INTER * 4);      // [32][257]
    __shared__ int s_last;

    const int rc = blockIdx.x, sp = blockIdx.y, j = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    const uint8_t *blk = reinterpret_cast<const uint8_t *>(a.tab[j]);
    const bool bad = (reinterpret_cast<uintptr_t>(blk) & 15u) != 0 || blk == nullptr;
    const float cmul = a.coef[j] * a.s2[2 * j + 1];

    pdl_launch_dependents();   // the next kernel (the next layer's up) may start its launch now
    pdl_wait();  // the up kernel's h and masks are complete and visible

    // ---- 1. live neurons of this CTA's groups, ascending: thread t < 168 takes the t-th listed group;
    // one block scan of packed (live-group count << 16 | live-neuron count) gives every thread its
    // group rank and its neurons' offset in nl.
    __shared__ int s_wsum[DN_THREADS / 32];
    int g = -1, m = 0;
    if (FUSED) {
        if (tid < G_DN) {
            g = tid;
            m = *reinterpret_cast<const uint16_t *>(a.gmask8 + (int64_t)j * 2 * G_DN + 2 * g);  // 16 neurons of group g
        }
    } else {
        int gc = a.gcnt_in[j];
        gc = gc < 0 ? 0 : (gc > G_DN ? G_DN : gc);   // caller data: never index past the [K,168] list
        const int ng = gc > sp ? (gc - sp + a.KS - 1) / a.KS : 0;
        if (tid < ng) {
            g = a.gidx_in[(int64_t)j * G_DN + sp + tid * a.KS];
            if (g >= 0 && g < G_DN) {   // an out-of-range group id contributes nothing
                const float4 *hp = reinterpret_cast<const float4 *>(a.h + (int64_t)j * INTER + 16 * g);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float4 v = hp[i];
                    m |= ((v.x > 0.f) << (4 * i)) | ((v.y > 0.f) << (4 * i + 1)) | ((v.z > 0.f) << (4 * i + 2)) |
                         ((v.w > 0.f) << (4 * i + 3));
                }
            }
        }
    }
    const int packed = ((m != 0) << 16) | __popc(m);
    int inc = packed;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
    }
    if (lane == 31) s_wsum[warp] = inc;
    __syncthreads();
    int excl = inc - packed, tot = 0;
#pragma unroll
    for (int w = 0; w < DN_THREADS / 32; ++w) {
        if (w < warp) excl += s_wsum[w];
        tot += s_wsum[w];
    }
    {
        int off = excl & 0xFFFF, mm = m;
        while (mm) {
            const int i = __ffs(mm) - 1;
            mm &= mm - 1;
            nl[off++] = 16 * g + i;
        }
    }
    if (FUSED && rc == 0) {
        const int total_groups = tot >> 16, grank = excl >> 16;
        if (tid < G_DN) a.gidx_out[(int64_t)j * G_DN + (m ? grank : total_groups + (tid - grank))] = tid;
        if (tid == 0) a.gcnt_out[j] = total_groups;
    }
    __syncthreads();
    const int L = tot & 0xFFFF;

    // ---- 2. stream the live neurons
    const int q = tid & 3, p = tid >> 2;
    float acc[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) acc[k] = 0.f;
    if (!bad) {
        const uint8_t *wb = blk + O_DW + rc * (DN_CHUNK / 2) + q * 16;
        const uint8_t *sb = blk + O_DS + rc * DN_CHUNK + q * 32;
        const float *hj = a.h + (int64_t)j * INTER;
        for (int i0 = p; i0 < L; i0 += DN_SLOTS * DN_NB) {
            uint4 wv[DN_NB], s0[DN_NB], s1[DN_NB];
            float hn[DN_NB];
#pragma unroll
            for (int u = 0; u < DN_NB; ++u) {
                const int i = i0 + u * DN_SLOTS;
                if (i < L) {
                    const int n = nl[i];
                    wv[u] = ldg_stream(wb + (int64_t)n * (LAT / 2));
                    s0[u] = __ldg(reinterpret_cast<const uint4 *>(sb + (int64_t)(n >> 4) * LAT));
                    s1[u] = __ldg(reinterpret_cast<const uint4 *>(sb + (int64_t)(n >> 4) * LAT + 16));
                    hn[u] = hj[n];
                } else {
                    hn[u] = 0.f;
                }
            }
#pragma unroll
            for (int u = 0; u < DN_NB; ++u) {
                if (i0 + u * DN_SLOTS >= L) break;
                const uint32_t *ww = reinterpret_cast<const uint32_t *>(&wv[u]);
                const uint32_t sw8[8] = {s0[u].x, s0[u].y, s0[u].z, s0[u].w, s1[u].x, s1[u].y, s1[u].z, s1[u].w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    uint32_t o[4];
                    e2m1x8_f16x2(ww[k], o);  // rows 8k .. 8k+7 of this thread's 32
                    uint32_t sc[4];
                    e4m3x4_f16x2(sw8[2 * k], sc[0], sc[1]);
                    e4m3x4_f16x2(sw8[2 * k + 1], sc[2], sc[3]);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        // e2m1 * e4m3 is exact in f16
                        const float2 f = __half22float2(__hmul2(as_h2(o[e]), as_h2(sc[e])));
                        acc[8 * k + 2 * e] = fmaf(f.x, hn[u], acc[8 * k + 2 * e]);
                        acc[8 * k + 2 * e + 1] = fmaf(f.y, hn[u], acc[8 * k + 2 * e + 1]);
                    }
                }
            }
        }
    }

    // ---- 3. fixed-order reduction over the 64 neuron slots
#pragma unroll
    for (int k = 0; k < 32; ++k) red[k * DN_RED_LD + tid] = acc[k];
    __syncthreads();
    float out = 0.f;
    if (tid < DN_CHUNK) {
        const int qq = tid >> 5, k = tid & 31;
        float v = 0.f;
        for (int pp = 0; pp < DN_SLOTS; ++pp) v += red[k * DN_RED_LD + 4 * pp + qq];
        out = v * cmul;
        if (bad) out = __int_as_float(0x7fc00000);
    }
    const int row = rc * DN_CHUNK + tid;
    if (!FUSED) {
        if (tid < DN_CHUNK) a.part[((int64_t)sp * a.K + j) * LAT + row] = out;
        return;
    }
    if (bad && tid == 0) set_error(a.status, QMOE_ERR_ALIGN);
    if (tid < DN_CHUNK) a.part[(int64_t)j * LAT + row] = out;
    // ---- 4. the last CTA of this chunk sums the K experts in slot order. The CTA barrier orders every
    // thread's part[] store before thread 0's GPU-scope fence and arrival (fences are cumulative), and
    // the last arriver's fence before the barrier orders its readers after all arrivals.
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const bool last = atomicAdd(&a.counters[rc], 1) == a.K - 1;
        if (last) __threadfence();
        s_last = last;
    }
    __syncthreads();
    if (s_last) {
        if (tid < DN_CHUNK) {
            float v = 0.f;
            for (int jj = 0; jj < a.K; ++jj) v += __ldcg(&a.part[(int64_t)jj * LAT + row]);
            a.y[row] = v;
        }
        if (tid == 0) a.counters[rc] = 0;
    }
}

// ------------------------------------------------------------------ thread-block-cluster helpers
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Cluster barrier (split): every CTA arrives at kernel entry and waits just before its first access to another CTA's
// shared memory, which must not happen before all CTAs of the cluster have started; the release / acquire pair at the
// end publishes the pushed sums to rank 0.
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_wait_acquire() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ------------------------------------------------------------------ the decode-step layer fused per CTA
// `moe_decode_groups` (qmoe_ns.py:245-255) with each expert's neurons split over a cluster of S CTAs (S*K <= SMs):
// CTA s of expert j owns neurons [s*2688/S, (s+1)*2688/S). It streams their up rows (`_up`, qmoe_ns.py:24-44, the
// tiles of decode_up_kernel with the next tile's loads in flight), keeps h and the live masks in shared memory
// (and writes h out), lists its live neurons, and at once adds their down contributions (`_down_groups`,
// qmoe_ns.py:209-239, over the T layout: a neuron's 512-byte row of dnT_w covers all 1024 output rows): warp w
// takes live neurons w, w+12, ..., lane l the rows 32l .. 32l+31, fp32 accumulation of (e2m1 * e4m3, exact in f16)
// * h. So no CTA waits for another's up tiles, and the down work of early CTAs overlaps the up tail of late ones.
// The CTA's 1024 partial sums (its 12 warps in order) and its groups' live flags go to cluster rank 0's shared
// memory; rank 0 sums the S CTAs in rank order into part[j] (x coef_j * s2d_j) and writes gidx / gcnt for the
// expert. decode_finish_kernel, its programmatic dependent, sums the experts in slot order into y.
constexpr int FL_NW = UP_NW;                   // 12 warps, as the up kernel
constexpr int FL_THREADS = 32 * FL_NW;
constexpr int FL_MAXS = 8;                     // CTAs per expert (portable cluster size)
constexpr int FL_NB = 4;                       // live neurons per warp with all loads in flight at once
// dynamic shared memory of the fused layer kernel (byte offsets)
constexpr int FL_OFF_H = 0;                                   // h of the CTA's neurons, f32 [<= 2688]
constexpr int FL_OFF_NL = FL_OFF_H + INTER * 4;               // live neurons (CTA-local index), u16 [<= 2688]
constexpr int FL_OFF_MASK = FL_OFF_NL + INTER * 2;            // live mask per 8-row tile, u8 [<= 336]
constexpr int FL_OFF_TMASK = FL_OFF_MASK + 352;               // rank 0: the expert's 336 tile masks (all CTAs)
constexpr int FL_OFF_WSUM = FL_OFF_TMASK + 352;               // the live-neuron count
constexpr int FL_RED_LD = 33;                                 // per-warp down sums: lane l's 32 rows at 33 l + k
constexpr int FL_RED_W = 32 * FL_RED_LD;                      //   (no bank conflicts on either side)
constexpr int FL_OFF_RED = FL_OFF_WSUM + 64;                  // per-warp down sums, f32 [12][32][33]
constexpr int FL_OFF_GATHER = FL_OFF_RED + FL_NW * FL_RED_W * 4;   // rank 0: each CTA's 1024 sums, f32 [S][1024]
constexpr size_t FL_SMEM = FL_OFF_GATHER + (size_t)FL_MAXS * LAT * 4;
static_assert(FL_OFF_RED % 16 == 0 && FL_OFF_GATHER % 16 == 0, "fused layer smem alignment");

struct LayerArgs {
    const uint8_t *slots;
    int64_t slot_bytes;
    int64_t nslots;
    const int32_t *sidx;
    const int64_t *tab;
    const float *s2;
    const float *coef;
    const void *x;
    int x_dtype;
    int K, S;
    float *h;
    int32_t *gidx;
    int32_t *gcnt;
    float *part;
    int *status;
};

__device__ __forceinline__ void st_cluster_f32x4(float *local, uint32_t rank, float4 v) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(remote), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

__device__ __forceinline__ void st_cluster_u8(uint8_t *local, uint32_t rank, uint32_t v) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
    asm volatile("st.shared::cluster.u8 [%0], %1;" ::"r"(remote), "r"(v) : "memory");
}

template <bool XF32>
__global__ void __launch_bounds__(FL_THREADS, 1) decode_layer_kernel(LayerArgs a) {
    extern __shared__ __align__(16) uint8_t fsm[];
    float *hs = reinterpret_cast<float *>(fsm + FL_OFF_H);
    uint16_t *nl = reinterpret_cast<uint16_t *>(fsm + FL_OFF_NL);
    uint8_t *mk = fsm + FL_OFF_MASK;
    uint8_t *tmask = fsm + FL_OFF_TMASK;
    int *wsum = reinterpret_cast<int *>(fsm + FL_OFF_WSUM);
    float *red = reinterpret_cast<float *>(fsm + FL_OFF_RED);
    float *gather = reinterpret_cast<float *>(fsm + FL_OFF_GATHER);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int sr = (int)cluster_ctarank(), j = blockIdx.y, S = a.S;
    const int npc = INTER / S, ntile = npc / UP_ROWS, ngrp = npc / 16, n0 = sr * npc;
    cluster_arrive_relaxed();

    pdl_launch_dependents();   // the finish kernel may become resident now; it waits for this grid
    pdl_wait();                // the layer inputs may be outputs of the preceding kernels
    const int64_t slot = a.sidx[j];
    const uint8_t *base = (slot < 0 || slot >= a.nslots) ? nullptr : a.slots + slot * a.slot_bytes;
    const bool bad = base == nullptr;                 // bad slot: h and every output of the expert NaN
    const uint8_t *blk = reinterpret_cast<const uint8_t *>(a.tab[j]);
    const bool bad_tab = blk == nullptr || (reinterpret_cast<uintptr_t>(blk) & 15u) != 0;

    // Each warp's first tile is requested before x is prepared, so that the two latencies overlap.
    UpTile tn;
    if (warp < ntile && !bad) up_load(base, n0 / UP_ROWS + warp, lane, tn);

    UpArgs xa{};
    xa.x = a.x;
    xa.x_dtype = a.x_dtype;
    UpX<XF32> x;
    float inv;
    up_prep_x<XF32>(xa, lane, x, inv);
    const float mult = a.s2[2 * j] * inv;

    // ---- U: the CTA's up tiles (8 rows each), warp w takes tiles w, w+12, ..., the next tile's loads in flight
    {
        int t = warp;
        for (; t < ntile; t += FL_NW) {
            const UpTile tc = tn;
            if (t + FL_NW < ntile && !bad) up_load(base, n0 / UP_ROWS + t + FL_NW, lane, tn);
            const float u = fmaxf(up_tile_dot<XF32>(tc, x, lane) * mult, 0.f);   // ReLU^2 (qmoe_ns.py:42-44)
            float hv = u * u;
            if (bad) hv = __int_as_float(0x7fc00000);
            const int nloc = t * UP_ROWS + (lane >> 2);
            const bool lead = (lane & 3) == 0;
            if (lead) {
                hs[nloc] = hv;
                a.h[(int64_t)j * INTER + n0 + nloc] = hv;
            }
            const unsigned m = __reduce_or_sync(0xffffffffu, (lead && (hv > 0.f || bad)) ? (1u << (lane >> 2)) : 0u);
            if (lane == 0) mk[t] = (uint8_t)m;
            // start bringing the live neurons' dnT_w rows and their groups' dnT_s rows into L2
            if (!bad_tab && !bad && m) {
                if (lead && hv > 0.f) {
                    const uint8_t *row = blk + O_DW + (int64_t)(n0 + nloc) * (LAT / 2);
#pragma unroll
                    for (int l = 0; l < 4; ++l) prefetch_l2(row + 128 * l);
                }
                if (lane >= 24) prefetch_l2(blk + O_DS + (int64_t)((n0 + t * UP_ROWS) >> 4) * LAT + 128 * (lane - 24));
            }
        }
    }
    __syncthreads();

    // ---- C: warp 0 lists the CTA's live neurons, ascending (lane l: groups G*l .. G*l + G - 1)
    if (warp == 0) {
        const int G = (ngrp + 31) / 32;
        int cnt = 0;
        for (int q = 0; q < G; ++q) {
            const int g = G * lane + q;
            if (g < ngrp) cnt += __popc((uint32_t)mk[2 * g] | ((uint32_t)mk[2 * g + 1] << 8));
        }
        int inc = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += t;
        }
        int o = inc - cnt;
        for (int q = 0; q < G; ++q) {
            const int g = G * lane + q;
            uint32_t mm = g < ngrp ? ((uint32_t)mk[2 * g] | ((uint32_t)mk[2 * g + 1] << 8)) : 0u;
            while (mm) {
                const int i = __ffs(mm) - 1;
                mm &= mm - 1;
                nl[o++] = (uint16_t)(16 * g + i);
            }
        }
        if (lane == 31) wsum[0] = inc;
    }
    __syncthreads();
    const int L = wsum[0];

    // ---- D: the live neurons' down contributions to all 1024 rows; lane l: rows 32l .. 32l+31
    float acc[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) acc[k] = 0.f;
    if (!bad_tab) {
        const uint8_t *wb = blk + O_DW + lane * 16;
        const uint8_t *sb = blk + O_DS + lane * 32;
        for (int i0 = warp; i0 < L; i0 += FL_NW * FL_NB) {
            uint4 wv[FL_NB], s0[FL_NB], s1[FL_NB];
            float hn[FL_NB];
#pragma unroll
            for (int b = 0; b < FL_NB; ++b) {
                const int i = i0 + b * FL_NW;
                if (i < L) {
                    const int nloc = nl[i], n = n0 + nloc;
                    wv[b] = ldg_stream(wb + (int64_t)n * (LAT / 2));
                    s0[b] = __ldg(reinterpret_cast<const uint4 *>(sb + (int64_t)(n >> 4) * LAT));
                    s1[b] = __ldg(reinterpret_cast<const uint4 *>(sb + (int64_t)(n >> 4) * LAT + 16));
                    hn[b] = hs[nloc];
                }
            }
#pragma unroll
            for (int b = 0; b < FL_NB; ++b) {
                if (i0 + b * FL_NW >= L) break;
                const uint32_t *ww = reinterpret_cast<const uint32_t *>(&wv[b]);
                const uint32_t sw8[8] = {s0[b].x, s0[b].y, s0[b].z, s0[b].w, s1[b].x, s1[b].y, s1[b].z, s1[b].w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    uint32_t o[4];
                    e2m1x8_f16x2(ww[k], o);   // rows 32l + 8k .. 32l + 8k + 7
                    uint32_t sc[4];
                    e4m3x4_f16x2(sw8[2 * k], sc[0], sc[1]);
                    e4m3x4_f16x2(sw8[2 * k + 1], sc[2], sc[3]);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f = __half22float2(__hmul2(as_h2(o[e]), as_h2(sc[e])));   // exact in f16
                        acc[8 * k + 2 * e] = fmaf(f.x, hn[b], acc[8 * k + 2 * e]);
                        acc[8 * k + 2 * e + 1] = fmaf(f.y, hn[b], acc[8 * k + 2 * e + 1]);
                    }
                }
            }
        }
    }
    {
        float *rw = red + warp * FL_RED_W + lane * FL_RED_LD;
#pragma unroll
        for (int k = 0; k < 32; ++k) rw[k] = acc[k];
    }
    cluster_wait();   // every CTA of the cluster has started: rank 0's shared memory may be written
    __syncthreads();
    // the CTA's sums (warps in order) into rank 0's gather[sr]: thread t sums rows 4t .. 4t+3 (lane t/8 of each warp,
    // rows 4(t%8) .. 4(t%8)+3 of its 32) and stores them with one 16-byte remote store
    if (tid < LAT / 4) {
        const float *rr = red + (tid >> 3) * FL_RED_LD + 4 * (tid & 7);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < FL_NW; ++w) {
            const float *t = rr + w * FL_RED_W;
            v.x += t[0], v.y += t[1], v.z += t[2], v.w += t[3];
        }
        st_cluster_f32x4(gather + sr * LAT + 4 * tid, 0u, v);
    }
    if (tid < ntile) st_cluster_u8(tmask + sr * ntile + tid, 0u, mk[tid]);   // the CTA's tile masks, for gidx
    cluster_arrive_release();
    if (sr != 0) return;   // nothing left for this CTA; rank 0's shared memory is the only one written remotely
    cluster_wait_acquire();

    // ---- rank 0: part[j], the S CTAs in rank order
    const float cmul = bad_tab ? __int_as_float(0x7fc00000) : a.coef[j] * a.s2[2 * j + 1];
    if (tid < LAT / 4) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int q = 0; q < S; ++q) {
            const float4 t = reinterpret_cast<const float4 *>(gather + q * LAT)[tid];
            v.x += t.x, v.y += t.y, v.z += t.z, v.w += t.w;
        }
        reinterpret_cast<float4 *>(a.part + (int64_t)j * LAT)[tid] = make_float4(v.x * cmul, v.y * cmul, v.z * cmul, v.w * cmul);
    }
    if (warp == FL_NW - 1) {
        // the expert's live-group list (qmoe_ns.py:249-251): live groups ascending, then dead groups ascending;
        // lane l takes groups 6l .. 6l+5, a group live if either of its two tiles has a live neuron
        int f[6], cnt = 0;
#pragma unroll
        for (int q = 0; q < 6; ++q) {
            const int g = 6 * lane + q;
            f[q] = g < G_DN ? ((tmask[2 * g] | tmask[2 * g + 1]) != 0) : 0;
            cnt += f[q];
        }
        int inc = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += t;
        }
        const int total = __shfl_sync(0xffffffffu, inc, 31);
        int before = inc - cnt;   // live groups before group 6l
#pragma unroll
        for (int q = 0; q < 6; ++q) {
            const int g = 6 * lane + q;
            if (g < G_DN) a.gidx[(int64_t)j * G_DN + (f[q] ? before : total + (g - before))] = g;
            before += f[q];
        }
        if (lane == 0) a.gcnt[j] = total;
    }
    if (bad_tab && tid == 0) set_error(a.status, QMOE_ERR_ALIGN);

}

// y[r] = sum over experts, in slot order, of part[j][r]: a programmatic dependent of decode_layer_kernel, all K loads
// of a row in flight at once (32 at a time).
__global__ void __launch_bounds__(128) decode_finish_kernel(const float *__restrict__ part, int K, float *__restrict__ y) {
    pdl_launch_dependents();
    pdl_wait();
    const int r = blockIdx.x * 128 + threadIdx.x;
    float v = 0.f;
    for (int j0 = 0; j0 < K; j0 += 32) {
        float t[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) t[k] = j0 + k < K ? __ldcg(part + (int64_t)(j0 + k) * LAT + r) : 0.f;
#pragma unroll
        for (int k = 0; k < 32; ++k)
            if (j0 + k < K) v += t[k];
    }
    y[r] = v;
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
static std::atomic<uint64_t> g_dn_smem_f{0}, g_dn_smem_r{0};

// The up kernel is launched as a programmatic dependent of whatever precedes it on the stream (for a decode
// step, the previous layer's down kernel): its CTAs are resident and waiting in griddepcontrol.wait when
// that kernel finishes, instead of being launched only then.
static int launch_up(const UpArgs &a, cudaStream_t st, int dev, const DeviceInfo &di) {
    (void)dev;
    const int ntiles = a.K * UP_HALVES;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ntiles < di.sms ? ntiles : di.sms);
    cfg.blockDim = dim3(UP_THREADS);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = a.x_dtype == QMOE_DT_F32 ? cudaLaunchKernelEx(&cfg, decode_up_kernel<true>, a)
                                                   : cudaLaunchKernelEx(&cfg, decode_up_kernel<false>, a);
    if (e != cudaSuccess) return QMOE_ERR_LAUNCH;
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

// CTAs per expert of the fused layer: the largest of 8, 7, 6, 4, 3, 2, 1 (2688 / S a multiple of 16) with S * K
// CTAs fitting the SMs at once; 0 when K exceeds the SMs (the two-kernel form then runs).
static int layer_split(int K, int sms) {
    const int opts[7] = {8, 7, 6, 4, 3, 2, 1};
    for (int i = 0; i < 7; ++i)
        if (opts[i] * K <= sms) return opts[i];
    return 0;
}

static std::atomic<uint64_t> g_fl_smem_b{0}, g_fl_smem_f{0};

// The fused decode-step layer: decode_layer_kernel (clusters of S CTAs per expert) and decode_finish_kernel, both
// programmatic dependents of what precedes them on the stream.
static int launch_layer(const LayerArgs &a, float *y, cudaStream_t st, int dev) {
    const bool f32 = a.x_dtype == QMOE_DT_F32;
    auto kern = f32 ? decode_layer_kernel<true> : decode_layer_kernel<false>;
    if (!ensure_smem(kern, FL_SMEM, dev, f32 ? g_fl_smem_f : g_fl_smem_b)) return QMOE_ERR_LAUNCH;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.S, a.K, 1);
    cfg.blockDim = dim3(FL_THREADS);
    cfg.dynamicSmemBytes = FL_SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = a.S;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (cudaLaunchKernelEx(&cfg, kern, a) != cudaSuccess) return QMOE_ERR_LAUNCH;
    if (int e = launch_status()) return e;
    cudaLaunchConfig_t cf = {};
    cf.gridDim = dim3(LAT / 128);
    cf.blockDim = dim3(128);
    cf.stream = st;
    cf.attrs = attr;
    cf.numAttrs = 1;
    if (cudaLaunchKernelEx(&cf, decode_finish_kernel, static_cast<const float *>(a.part), a.K, y) != cudaSuccess)
        return QMOE_ERR_LAUNCH;
    return launch_status();
}

// Workspace of qmoe_decode_groups: [status int][pad to 64][counters DN_NCHUNK ints][pad][gmask8 K*336 u8]
constexpr size_t WS_STATUS = 0;
constexpr size_t WS_COUNTERS = 64;
constexpr size_t WS_GMASK = 256;

// ------------------------------------------------------------------ allocation-free variant
// Scratch of qmoe_decode_groups_static: a file-scope device array instead of a caller workspace. Every
// GPU that loads this library holds it until the process exits. In host code the symbol is only a
// stand-in for the device array, never a device address: kernels get the address looked up below.
static __device__ __align__(256) uint8_t g_static_scratch[QMOE_STATIC_SCRATCH_BYTES];

// Device address of g_static_scratch on device `dev`, looked up once per device (the caller has made
// `dev` current). nullptr if the lookup failed.
static uint8_t *static_scratch(int dev) {
    static uint8_t *addr[MAX_DEVICES];
    static cudaError_t err[MAX_DEVICES];
    static std::once_flag once[MAX_DEVICES];
    std::call_once(once[dev], [dev] {
        void *p = nullptr;
        err[dev] = cudaGetSymbolAddress(&p, g_static_scratch);
        addr[dev] = static_cast<uint8_t *>(p);
    });
    return err[dev] == cudaSuccess ? addr[dev] : nullptr;
}
static_assert(WS_GMASK + (size_t)QMOE_STATIC_MAX_K * UP_HALVES <= QMOE_STATIC_SCRATCH_BYTES, "static scratch size");

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
    return WS_GMASK + (size_t)K * UP_HALVES;
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
    uint8_t *gmask8 = ws + WS_GMASK;
    cudaStream_t st = as_stream(stream);
    if (const int S = layer_split(K, di->sms)) {   // one fused kernel per layer (+ the expert sum)
        LayerArgs la{slots_up, slot_bytes, nslots, sidx, tab, s2, coef, x, x_dtype, K, S, h, gidx, gcnt, part, status};
        return launch_layer(la, y, st, dev);
    }
    UpArgs ua{slots_up, slot_bytes, nslots, sidx, K, s2, x, x_dtype, h, gmask8, status, counters, DN_NCHUNK, tab};
    if (int e = launch_up(ua, st, dev, *di)) return e;
    DownArgs da{tab, h, gmask8, nullptr, nullptr, s2, coef, K, 1, part, gidx, gcnt, y, counters, status};
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
    auto kern = gemv_kernel<1, GM_EXPERT_DOWN, 3, 1, true>;   // h stays fp32
    const size_t smem = gemv_smem_bytes(true, 1, INTER);
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
    static std::atomic<uint64_t> up_done{0}, up32_done{0}, dn_done{0};
    const bool xf32 = x_dtype == QMOE_DT_F32;   // fp32 tokens are multiplied in fp32, bf16 / f16 as exact f16
    auto kup = xf32 ? gemv_kernel<1, GM_PAIR_UP, 1, 1, true> : gemv_kernel<1, GM_PAIR_UP, 1, 1, false>;
    const size_t smem_up = gemv_smem_bytes(xf32, 1, LAT);
    if (!ensure_smem(kup, smem_up, dev, xf32 ? up32_done : up_done)) return QMOE_ERR_LAUNCH;
    kup<<<dim3(INTER / 128, P), GEMV_THREADS, smem_up, st>>>(g, 128);
    if (int e = launch_status()) return e;
    GemvArgs d = g;
    d.hin = h;
    d.y = out;
    d.N = LAT;
    d.K = INTER;
    auto kdn = gemv_kernel<1, GM_PAIR_DOWN, 3, 1, true>;   // h stays fp32
    const size_t smem_dn = gemv_smem_bytes(true, 1, INTER);
    if (!ensure_smem(kdn, smem_dn, dev, dn_done)) return QMOE_ERR_LAUNCH;
    kdn<<<dim3(LAT / 64, P), GEMV_THREADS, smem_dn, st>>>(d, 64);
    return launch_status();
}

// For callers that cannot allocate device memory: the decode-step layer of qmoe_decode_groups, with the
// scratch in the library's static device array instead of a caller workspace. No allocation of any kind.
int qmoe_decode_groups_static(const uint8_t *slots_up, int64_t slot_bytes, int64_t nslots, const int32_t *sidx,
                              const int64_t *tab, const float *s2, const float *coef, const void *x, int x_dtype,
                              int K, float *h, int32_t *gidx, int32_t *gcnt, float *part, float *y, void *stream) {
    if (!slots_up || !sidx || !tab || !s2 || !coef || !x || !h || !gidx || !gcnt || !part || !y) return QMOE_ERR_NULL;
    if (K < 1 || nslots < 1) return QMOE_ERR_SHAPE;
    if (K > QMOE_STATIC_MAX_K) return QMOE_ERR_SCRATCH_LIMIT;   // its workspace would not fit the static array
    if (slot_bytes < UPB || (slot_bytes & 15) || !aligned16(slots_up)) return QMOE_ERR_ALIGN;
    if (!valid_dtype(x_dtype)) return QMOE_ERR_DTYPE;
    int dev;
    DeviceInfo *di;
    if (int e = current_device(&dev, &di)) return e;
    uint8_t *ws = static_scratch(dev);
    if (!ws) return QMOE_ERR_LAUNCH;
    int *status = reinterpret_cast<int *>(ws + WS_STATUS);
    int *counters = reinterpret_cast<int *>(ws + WS_COUNTERS);   // zeroed by the up kernel on every call
    uint8_t *gmask8 = ws + WS_GMASK;                              // rewritten in full on every call
    cudaStream_t st = as_stream(stream);
    if (const int S = layer_split(K, di->sms)) {   // one fused kernel per layer (+ the expert sum)
        LayerArgs la{slots_up, slot_bytes, nslots, sidx, tab, s2, coef, x, x_dtype, K, S, h, gidx, gcnt, part, status};
        return launch_layer(la, y, st, dev);
    }
    UpArgs ua{slots_up, slot_bytes, nslots, sidx, K, s2, x, x_dtype, h, gmask8, status, counters, DN_NCHUNK, tab};
    if (int e = launch_up(ua, st, dev, *di)) return e;
    DownArgs da{tab, h, gmask8, nullptr, nullptr, s2, coef, K, 1, part, gidx, gcnt, y, counters, status};
    return launch_down<true>(da, st, dev, true);
}

// The status word at the start of the static array: the first device-side error of the calls since it was last
// cleared, read (and with `clear`, reset) on `stream` after that stream's earlier work has finished.
int qmoe_decode_groups_static_status(int clear, void *stream) {
    int dev;
    if (int e = current_device(&dev, nullptr)) return e;
    uint8_t *ws = static_scratch(dev);
    if (!ws) return QMOE_ERR_LAUNCH;
    return qmoe_workspace_status(ws + WS_STATUS, clear, stream);
}

} // extern "C"
