// Prefill: the routed-expert forward for T tokens at once, as an expert-grouped GEMM on the 5th-generation
// tensor cores (block-scaled NVFP4 tcgen05.mma, accumulators in tensor memory).
//
// Replaces the reference's prompt path (nem_super.py:295-348): the pair path moe_pairs
// (qmoe_ns.py:79-133, used for T <= 64) and the per-expert CPU/fp32 path (block_deq + two F.linear per
// expert, nem_super.py:342-346), including the fixed-order combine over top-k (nem_super.py:309, :347).
//
// Pipeline (all on the caller's stream, nothing allocated):
//   1. pf_hist / pf_chunkscan / pf_scan / pf_place: a deterministic counting sort of the T*topk (token, k)
//      pairs by expert. Pairs of one expert are contiguous and ordered by token; tiles of <= 128 pairs per
//      expert.
//   2. pf_xtok / pf_xplanes: x[token] * 2^E as three NVFP4 residual planes (once per token), copied to each
//      pair's rows, their scales as tcgen05 scale atoms of the pair's tile.
//   3. (T layout only) pf_dnT_codes / pf_dnT_scales: the used experts' down halves converted to the orig
//      (K-major) layout in the workspace.
//   4. pfb_gemm<UP>: per (tile, 128 up rows): D = W_up (NVFP4 as stored) x planes^T, block-scaled MMA;
//      epilogue u = D * 2^-E * s2u, h = relu(u)^2 stored as f32.
//   5. pf_hplanes: h in its tile's frame as three NVFP4 planes.
//   6. pfb_gemm<DOWN>: per (tile, 128 output rows), K = 2688; epilogue y = D * 2^(4 - S0) * s2d * coef.
//   7. pf_combine: out[t] = sum_k Op[pos(t, k)] in k order (deterministic, as nem_super.py:309-347).
#include <cuda.h>

#include "common.cuh"
#include "host.h"

namespace qmoe {
namespace pf {

constexpr int NT = 128;                 // pairs per tile = largest MMA N used
constexpr int BM = 128;                 // MMA M (rows of the weight tile)
constexpr int MT_UP = INTER / BM;       // 21
constexpr int MT_DN = LAT / BM;         // 8
constexpr int CHUNK_T = 16;             // tokens per routing chunk (one placement warp each)
constexpr int MAX_NE = 1024;
constexpr int MAX_TOPK = 32;
constexpr int MAX_T = 65536;
// Row offsets of the block regions in the TMA views of the store (row pitch 512, 1024, 1344 bytes).
constexpr int ROW1344_DW = (int)(O_DW / 1344);    // 1152: dn_w
constexpr int64_t DC_W = (int64_t)LAT * KB_DN;      // 1,376,256 B: orig-layout down codes
constexpr int64_t DC_STRIDE = DC_W + (int64_t)LAT * G_DN;   // + 172,032 B of scales: one converted down half
static_assert(O_DW % 1344 == 0 && BLOCK % 1344 == 0, "dn_w on 1344-byte view rows");

// Shared memory carve-up, from a 1024-byte aligned base (the 128B swizzle repeats every 1024 bytes).
enum { PH_UP = 0, PH_DN_O = 2 };

struct Params {
    const uint8_t *store;   // expert e's block at store + e * bstride
    int64_t bstride;
    int ne;
    const int32_t *ids;     // [T, topk]
    const float *wts;       // [T, topk]
    const float *s2;        // [ne, 2]: (up, down) weight_scale_2
    const void *x;          // [T, 1024]
    int x_dtype;
    int T, topk, P, nchunks, tiles_cap;
    float *out;             // [T, 1024] f32
    int *status;
    long long wait_cycles;  // bound on each wait of the GEMM roles, in SM clock cycles
    int *tile_count;
    int *cnt;               // [ne]
    int *eoff;              // [ne + 1]
    int *chunk_hist;        // [nchunks, ne] counts, then per-chunk offsets
    int4 *tiles;            // [tiles_cap] (expert, first pair, pairs, rank of the expert among those used)
    int *pair_tok;          // [P]
    float *pair_coef;       // [P]
    int *pair_pos;          // [T * topk] sorted position of (t, k), -1 if the id was invalid
    int *pair_exp;          // [P]
    int *tile_scale;        // [tiles_cap, 21]
    float *hs;              // [P, 2688] h = relu(u)^2 of every pair, f32 (the h planes read it)
    const uint8_t *dn_w;    // down codes [1024 rows][1344 B] of expert e at dn_w + e * dn_bstride (row dn_row0)
    const uint8_t *dn_sc;   // down scales [1024][168] of expert e at dn_sc + e * dn_bstride
    int64_t dn_bstride;
    int dn_row0;
    uint8_t *dconv;         // T layout: the used experts' down halves converted to the orig layout,
                            // [used experts][1376256 B codes | 172032 B scales], in ascending expert order
    int *ecomp;             // [ne] rank of expert e among the experts with pairs (-1: no pair)
    int dn_compact;         // 1: the down GEMM addresses its weights by the rank (tile .w), not the id
    float *op;              // [P, 1024]
    int *pair_tile;         // [P] tile of each sorted pair
    int *toff;              // [ne] index of the expert's first tile
    uint8_t *xq, *hq;       // [NP, P, 512], [NP, P, 1344] e2m1 codes: x, h (x 2^S0 of its tile) as NVFP4 planes
    uint8_t *xtq, *xtsc;    // [NP, T, 512] codes, [NP, T, 64] scales: x planes per token
    int *xt_exp;            // [T] prescale exponent per token
    uint8_t *sfbx, *sfbh;   // [tiles_cap, k-steps 16 | 42, NP, 512] the planes' e4m3 scales as tcgen05 atoms
};

// ------------------------------------------------------------------------------------------ routing
// Per chunk of CHUNK_T tokens: histogram of expert ids. Id -1 means "no expert" (an expert-parallel block
// row whose expert lives on another rank): the pair is skipped and contributes nothing. Any other id outside
// [0, ne) is recorded as a shape error and its pair dropped (its (t, k) slot then yields NaN in the combine).
__global__ void __launch_bounds__(256) pf_hist_kernel(const Params p) {
    __shared__ int hist[MAX_NE];
    for (int e = threadIdx.x; e < p.ne; e += blockDim.x) hist[e] = 0;
    __syncthreads();
    const int t0 = blockIdx.x * CHUNK_T;
    const int t1 = min(p.T, t0 + CHUNK_T);
    const int n = (t1 - t0) * p.topk;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int e = p.ids[(int64_t)t0 * p.topk + i];
        if (e == -1) continue;
        if (e < 0 || e >= p.ne) {
            set_error(p.status, QMOE_ERR_SHAPE);
            continue;
        }
        atomicAdd(&hist[e], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < p.ne; e += blockDim.x) p.chunk_hist[(int64_t)blockIdx.x * p.ne + e] = hist[e];
}

// One warp per expert: the running offset of each chunk (in place, chunks in order) and the expert's pair
// count.
__global__ void __launch_bounds__(256) pf_chunkscan_kernel(const Params p) {
    const int lane = threadIdx.x & 31;
    const int e = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (e >= p.ne) return;
    int carry = 0;
    for (int c0 = 0; c0 < p.nchunks; c0 += 32) {
        const int c = c0 + lane;
        const int v = c < p.nchunks ? p.chunk_hist[(int64_t)c * p.ne + e] : 0;
        int inc = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += y;
        }
        if (c < p.nchunks) p.chunk_hist[(int64_t)c * p.ne + e] = carry + inc - v;
        carry += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) p.cnt[e] = carry;
}

// One CTA: per expert (thread), the offset of its pairs and the tile list (tiles of NT pairs, experts in
// ascending order).
__global__ void __launch_bounds__(1024) pf_scan_kernel(const Params p) {
    __shared__ int warp_sum[3][32];
    const int e = threadIdx.x;
    const int run = e < p.ne ? p.cnt[e] : 0;
    const int cnt = run;
    const int ntile = (cnt + NT - 1) / NT;
    const int used = cnt > 0;
    // block exclusive scans of (cnt, ntile, used) in thread (= expert) order
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int a = cnt, b = ntile, c = used;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int ya = __shfl_up_sync(0xffffffffu, a, o), yb = __shfl_up_sync(0xffffffffu, b, o),
                  yc = __shfl_up_sync(0xffffffffu, c, o);
        if (lane >= o) { a += ya; b += yb; c += yc; }
    }
    if (lane == 31) { warp_sum[0][warp] = a; warp_sum[1][warp] = b; warp_sum[2][warp] = c; }
    __syncthreads();
    if (warp == 0) {
        int wa = warp_sum[0][lane], wb = warp_sum[1][lane], wc = warp_sum[2][lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int ya = __shfl_up_sync(0xffffffffu, wa, o), yb = __shfl_up_sync(0xffffffffu, wb, o),
                      yc = __shfl_up_sync(0xffffffffu, wc, o);
            if (lane >= o) { wa += ya; wb += yb; wc += yc; }
        }
        warp_sum[0][lane] = wa;
        warp_sum[1][lane] = wb;
        warp_sum[2][lane] = wc;
    }
    __syncthreads();
    const int off = a - cnt + (warp ? warp_sum[0][warp - 1] : 0);
    const int toff = b - ntile + (warp ? warp_sum[1][warp - 1] : 0);
    const int rank = c - used + (warp ? warp_sum[2][warp - 1] : 0);
    if (e < p.ne) {
        p.eoff[e] = off;
        p.toff[e] = toff;
        p.ecomp[e] = used ? rank : -1;
        for (int i = 0; i < ntile; i++) {
            const int n0 = off + i * NT;
            p.tiles[toff + i] = make_int4(e, n0, min(NT, cnt - i * NT), rank);
        }
    }
    if (threadIdx.x == blockDim.x - 1) {
        p.eoff[p.ne] = warp_sum[0][31];
        *p.tile_count = warp_sum[1][31];
    }
}

// One warp per chunk: walks the chunk's tokens in order and gives each (t, k) its position inside its
// expert's run, and the pair its tile. Equal ids inside one token (not produced by a top-k router) are ranked
// by k.
__global__ void __launch_bounds__(32) pf_place_kernel(const Params p) {
    __shared__ int base[MAX_NE];
    __shared__ int sid[CHUNK_T * MAX_TOPK];
    __shared__ float swt[CHUNK_T * MAX_TOPK];
    const int lane = threadIdx.x;
    const int c = blockIdx.x;
    for (int e = lane; e < p.ne; e += 32) base[e] = p.eoff[e] + p.chunk_hist[(int64_t)c * p.ne + e];
    const int t0 = c * CHUNK_T;
    const int t1 = min(p.T, t0 + CHUNK_T);
    const int n = (t1 - t0) * p.topk;
    for (int i = lane; i < n; i += 32) {
        sid[i] = p.ids[(int64_t)t0 * p.topk + i];
        swt[i] = p.wts[(int64_t)t0 * p.topk + i];
    }
    __syncwarp();
    const uint32_t lt = (1u << lane) - 1u;
    for (int t = t0; t < t1; t++) {
        const bool valid = lane < p.topk;
        const int e = valid ? sid[(t - t0) * p.topk + lane] : -1;
        const bool ok = valid && e >= 0 && e < p.ne;
        const uint32_t mask = __match_any_sync(0xffffffffu, ok ? e : -1 - lane);
        const int64_t tk = (int64_t)t * p.topk + lane;
        if (ok) {
            const int pos = base[e] + __popc(mask & lt);
            p.pair_tok[pos] = t;
            p.pair_coef[pos] = swt[(t - t0) * p.topk + lane];
            p.pair_pos[tk] = pos;
            p.pair_tile[pos] = p.toff[e] + (pos - p.eoff[e]) / NT;
        } else if (valid) {
            p.pair_pos[tk] = e == -1 ? -2 : -1;   // -2: no expert (skipped), -1: invalid id (NaN)
        }
        __syncwarp();
        if (ok && (mask & lt) == 0) base[e] += __popc(mask);
        __syncwarp();
    }
}

// out[t] = sum over k (in order) of Op[pos(t, k)]; an invalid (t, k) contributes NaN, a skipped one nothing.
__global__ void __launch_bounds__(256) pf_combine_kernel(const Params p) {
    const int t = blockIdx.x;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < p.topk; k++) {
        const int pos = p.pair_pos[(int64_t)t * p.topk + k];
        if (pos == -2) continue;
        float4 v;
        if (pos >= 0) {
            v = reinterpret_cast<const float4 *>(p.op + (int64_t)pos * LAT)[threadIdx.x];
        } else {
            const float nan = __int_as_float(0x7fc00000);
            v = make_float4(nan, nan, nan, nan);
        }
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    reinterpret_cast<float4 *>(p.out + (int64_t)t * LAT)[threadIdx.x] = acc;
}

// ------------------------------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("barrier.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Shared-memory matrix descriptor (tcgen05 "matrix descriptor", version 1): start, leading and stride
// byte offsets in 16-byte units, layout type in bits 61-63 (0 = no swizzle, 2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}

// Arrives on `bar` once every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 consecutive f32 columns of tensor memory -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// 3-D tiled TMA load (box {x, y, 1}) into this CTA's shared memory, completing on `bar`.
// 1-D bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16), completing on bar.
__device__ __forceinline__ void bulk_g2s_nohint(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// 32 lanes x 16 consecutive f32 columns of tensor memory -> 16 registers per thread.
// 16 consecutive 32-bit columns of this warp's 32 TMEM lanes from registers (thread i -> lane base + i).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}


// Bounded wait for the phase with the given parity: false after `limit` SM clock cycles.
__device__ __forceinline__ bool mbar_wait_for(uint64_t *bar, uint32_t parity, long long limit) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > limit) return false;
    }
    return true;
}

__device__ __forceinline__ bool lane_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *status,
                                          long long limit) {
    if (mbar_try_wait(bar, parity)) return true;   // ready: no need to look at the abort flag
    const bool ok = !*abort_flag && mbar_wait_for(bar, parity, limit);
    if (!ok) {
        set_error(status, DEV_ERR_TIMEOUT);
        *abort_flag = 1;
    }
    return ok;
}

// ------------------------------------------------------------------------------------------ block-scaled
// The NVFP4 block-scaled path: tcgen05.mma.kind::mxf4nvf4.block_scale.block16 takes the weights exactly as
// stored (e2m1 codes, one e4m3 scale per 16 along k, K-major: up_w and the orig-layout dn_w) straight from
// TMA, with no decode. The other operand, the pairs' activations, is given as NP "residual planes": plane 0
// is the NVFP4 quantization of the row (per-16 e4m3 scale = amax/6), plane p+1 quantizes what plane p left
// over, so the sum of the planes is the row to ~amax/6^NP per 16-element group (measured output rel-L2
// ~8e-4 for x and ~2e-4 for h at NP = 3). Each k-step of 64 is NP MMAs into one fp32 accumulator.
constexpr int NP = 3;                    // activation planes
constexpr int HSHIFT = 4;                // h planes carry h * 2^(S0 - HSHIFT): block amax <= 2^11, scale <= 2^11 / 6
constexpr int BS_BK = 128;               // k per stage: two MMA k-steps of 64
constexpr int BS_KS = BS_BK / 64;        // MMA k-steps per stage
constexpr int BS_A = BM * BS_BK / 2;     // 8 KB: 128 weight rows x 64 B, 64-byte swizzle
constexpr int BS_B = NP * NT * BS_BK / 2;   // 24 KB: NP planes x up to 128 pair rows x 64 B
constexpr int BS_ATOM = 512;             // scale-factor atom: 128 rows x 4 scales, byte (r%32)*16 + (r/32)*4 + k
constexpr int BS_SFB = BS_KS * NP * BS_ATOM;   // 3 KB: the planes' atoms of a stage, (k-step, plane) order
constexpr int BS_SFA = BS_KS * BS_ATOM;        // 1 KB: the weights' atoms of a stage
constexpr int BS_STAGE = BS_A + BS_B + BS_SFB + BS_SFA;
constexpr int KS_UP = LAT / 64, KS_DN = INTER / 64;   // MMA k-steps of a row: 16 (up), 42 (down)
// Wide stages: a tile of h <= 32 pair rows (its planes run as one MMA) moves 256 k-elements per stage in the
// same 36 KB - weights [2 halves][128 rows][64 B] at 0, planes [2][NP][h][64 B] at 16 KB, plane atoms
// [4 k-steps][NP][512 B] at 28 KB, weight atoms [4][512 B] at 34 KB - so twice the weight bytes are in
// flight per stage and the per-stage hand-offs are paid once per 256. Other tiles use 128-element stages
// laid out as A | B | plane atoms | weight atoms (BS_A, BS_B, BS_SFB, BS_SFA).
constexpr int BW_B = 2 * BS_A;
constexpr int BW_SFB = BW_B + 2 * NP * 32 * (BS_BK / 2);
constexpr int BW_SFA = BW_SFB + 2 * BS_SFB;
static_assert(BS_STAGE % 1024 == 0 && BS_A % 512 == 0, "TMA destinations and swizzle atoms");
static_assert(BW_SFA + 2 * BS_SFA == BS_STAGE && BW_B % 512 == 0 && (NP * 16 * (BS_BK / 2)) % 512 == 0,
              "a wide stage fills the stage; its plane halves start on 64-byte swizzle atoms");

// Shared-memory plan of pfb_gemm_kernel<PH>: the stage ring, two slabs of the item's weight scales (128 rows
// x all of K: 8 KB up, 21 KB down), epilogue staging, barriers: five stages for both halves (the down half's
// five stages and two 21 KB slabs take 224 KB of the 227 KB opt-in).
template <int PH>
struct BsPlan {
    static constexpr int STAGES = 5;
    static constexpr int SLAB = BM * (PH == PH_UP ? G_UP : G_DN);
    static constexpr int OFF_SLAB = STAGES * BS_STAGE;
    static constexpr int OFF_COLSC = OFF_SLAB + 2 * SLAB;
    static constexpr int OFF_RED = OFF_COLSC + 2 * NT * 4;
    static constexpr int OFF_BAR = OFF_RED + 32;
    static constexpr int NBAR = 4 * STAGES + 8;
    static constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
    static constexpr int OFF_ABORT = OFF_TMEM + 16;
    static constexpr int OFF_REC = OFF_ABORT + 16;   // [STAGES][8] ints: the last use each role armed / arrived for
    static constexpr int SMEM = OFF_REC + STAGES * 32 + 1024;
    static_assert(SMEM <= 232448, "fits the 227 KB opt-in");
    static_assert(SLAB % 16 == 0, "bulk copy size");
};
constexpr int BS_NA = 2, BS_NB = 2;                   // A issuers, B issuers
constexpr int BS_W_A = 4, BS_W_B = BS_W_A + BS_NA, BS_W_SF = BS_W_B + BS_NB, BS_W_MMA = BS_W_SF + 1;
constexpr int BS_NSS = 4;                             // scale-store warps: one per TMEM lane quarter
constexpr int BS_W_SS = BS_W_MMA + 1;
constexpr int BS_THREADS = (BS_W_SS + BS_NSS) * 32;
constexpr int BS_TMEM_COLS = 512;                     // accumulators at 0 and NT; stage s's scale factors at
constexpr int BS_SF_COL = 2 * NT;                     // 2*NT + 32 s (per k-step: 4 columns SFA, 4 per plane)
static_assert(BS_SF_COL + 32 * 5 <= BS_TMEM_COLS && BS_KS * (1 + NP) * 4 <= 32, "TMEM plan");

// Pair rows loaded for a tile of n pairs (the TMA box heights): 16 or 32 for the fused-plane tiles, else n
// rounded up to a multiple of 16, so that a tile reads at most 15 rows of planes it does not use.
__host__ __device__ __forceinline__ int b_rows(int n) { return n <= 16 ? 16 : n <= 32 ? 32 : (n + 15) & ~15; }
constexpr int NBOX = NT / 16;   // box heights 16, 32, ..., NT

// The plane tensor maps of one GEMM, one per box height (16 * (k + 1) rows).
struct PlaneMaps {
    CUtensorMap m[NBOX];
};

// 16 fp32 values -> NP NVFP4 planes: codes[p] = 8 bytes (element 2i in the low nibble of byte i), scale
// byte sc[p] (e4m3, round to nearest; the e2m1 codes saturate, the residual carries the difference).
__device__ __forceinline__ void nvfp4_planes16(float (&v)[16], uint32_t (&codes)[NP][2], uint8_t (&sc)[NP]) {
#pragma unroll
    for (int pl = 0; pl < NP; ++pl) {
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
        uint32_t s16;
        asm("{\n\t.reg .b16 t;\n\tcvt.rn.satfinite.e4m3x2.f32 t, %1, %2;\n\tcvt.u32.u16 %0, t;\n\t}"
            : "=r"(s16) : "f"(0.f), "f"(amax * (1.f / 6.f)));
        const uint8_t sb = (uint8_t)(s16 & 0xFFu);
        const float s = e4m3_f32(sb);
        sc[pl] = sb;
        codes[pl][0] = codes[pl][1] = 0u;
        if (!(s > 0.f)) continue;
        // Any rounding of 1/s only moves a code choice; the residual below subtracts the exact value q * s
        // that the code and scale encode, so an approximate reciprocal keeps the planes consistent.
        float inv;
        asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(inv) : "f"(s));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            uint32_t b;
            asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u32.u8 %0, t;\n\t}"
                : "=r"(b) : "f"(v[2 * i + 1] * inv), "f"(v[2 * i] * inv));
            codes[pl][i >> 2] |= b << (8 * (i & 3));
            if (pl + 1 < NP) {   // the last plane leaves no residual to carry
                uint32_t h2;
                asm("{\n\t.reg .b8 t;\n\tcvt.u8.u32 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}" : "=r"(h2) : "r"(b));
                const float2 q = __half22float2(as_h2(h2));   // (element 2i, element 2i+1)
                v[2 * i] -= q.x * s;
                v[2 * i + 1] -= q.y * s;
            }
        }
    }
}

// A tile of h = b_rows(n) <= 32 pair rows runs its NP planes as ONE MMA of N = NP * h: B row pl * h + j is
// pair j of plane pl (the planes lie contiguous in the stage), and its scales sit in the tile's plane-0 atom
// at that row. Larger tiles run one MMA per plane with plane pl's scales in atom pl at row j.
__device__ __forceinline__ bool fused_planes(int h) { return h <= 32; }

// Byte of the tile's atoms holding the 4 scales of k-step ks, plane pl, pair j (atom row r:
// (r % 32) * 16 + (r / 32) * 4).
__device__ __forceinline__ int sfb_byte(int ks, int pl, int j, int h) {
    const bool f = fused_planes(h);
    const int r = f ? pl * h + j : j;
    return (ks * NP + (f ? 0 : pl)) * BS_ATOM + (r & 31) * 16 + (r >> 5) * 4;
}

// One warp per token: x[t] * 2^E (amax in [2^8, 2^9)) as NP planes, once per token (every pair of the token
// uses the same planes): codes [NP][T][512 B], scales [NP][T][64 B] (lane l: groups 2l, 2l+1), E per token.
__global__ void __launch_bounds__(256) pf_xtok_kernel(const Params p) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= p.T) return;
    float v[32];
    if (p.x_dtype == QMOE_DT_BF16) {
        const uint4 *src = reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(p.x) +
                                                          (int64_t)t * LAT + lane * 32);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint4 w = src[i];
            const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                v[i * 8 + 2 * j] = __uint_as_float(u[j] << 16);
                v[i * 8 + 2 * j + 1] = __uint_as_float(u[j] & 0xFFFF0000u);
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = load_act(p.x, p.x_dtype, (int64_t)t * LAT + lane * 32 + i);
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const int E = prescale_exp(amax, 9);
    const float scl = pow2f(E);
    uint32_t sc2[NP] = {};
#pragma unroll
    for (int g = 0; g < 2; ++g) {
        float w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = v[16 * g + i] * scl;
        uint32_t codes[NP][2];
        uint8_t sc[NP];
        nvfp4_planes16(w, codes, sc);
        const int grp = 2 * lane + g;
#pragma unroll
        for (int pl = 0; pl < NP; ++pl) {
            *reinterpret_cast<uint2 *>(p.xtq + ((int64_t)pl * p.T + t) * (LAT / 2) + grp * 8) = make_uint2(codes[pl][0], codes[pl][1]);
            sc2[pl] |= (uint32_t)sc[pl] << (8 * g);
        }
    }
#pragma unroll
    for (int pl = 0; pl < NP; ++pl)
        *reinterpret_cast<uint16_t *>(p.xtsc + ((int64_t)pl * p.T + t) * G_UP + 2 * lane) = (uint16_t)sc2[pl];
    if (lane == 0) p.xt_exp[t] = E;
}

// One warp per sorted pair: its token's planes copied into the pair's rows of xq (the GEMM's B operand) and
// the token's scales placed into the tile's atoms (sfbx), so that the GEMM moves a stage's scales with one bulk
// copy; E per pair for the epilogue.
__global__ void __launch_bounds__(256) pf_xplanes_kernel(const Params p) {
    const int lane = threadIdx.x & 31;
    const int pr = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (pr >= p.eoff[p.ne]) return;
    const int tile = p.pair_tile[pr];
    const int4 td = p.tiles[tile];
    const int jrow = pr - td.y, h = b_rows(td.z);
    uint8_t *sfb = p.sfbx + (int64_t)tile * KS_UP * NP * BS_ATOM;
    const int t = p.pair_tok[pr];
#pragma unroll
    for (int pl = 0; pl < NP; ++pl) {
        const uint4 c = *reinterpret_cast<const uint4 *>(p.xtq + ((int64_t)pl * p.T + t) * (LAT / 2) + 16 * lane);
        *reinterpret_cast<uint4 *>(p.xq + ((int64_t)pl * p.P + pr) * (LAT / 2) + 16 * lane) = c;
        // k-step ks = lane / 2 holds groups 4ks .. 4ks+3: the even lane stores all four bytes
        const uint32_t sc2 = *reinterpret_cast<const uint16_t *>(p.xtsc + ((int64_t)pl * p.T + t) * G_UP + 2 * lane);
        const uint32_t hi = __shfl_down_sync(0xffffffffu, sc2, 1);
        if (!(lane & 1)) *reinterpret_cast<uint32_t *>(sfb + sfb_byte(lane >> 1, pl, jrow, h)) = sc2 | (hi << 16);
    }
    if (lane == 0) p.pair_exp[pr] = p.xt_exp[t];
}

// One warp per sorted pair: its f32 h row times 2^(S0 - HSHIFT), S0 the tile's smallest block exponent (the
// exponent that puts a 128-row block's amax in [2^14, 2^15), recorded by the up epilogue), as NP planes: one
// frame for the whole row, the largest block amax in [2^10, 2^11), inside the e4m3 range of the plane scales.
__global__ void __launch_bounds__(256) pf_hplanes_kernel(const Params p) {
    const int lane = threadIdx.x & 31;
    const int pr = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (pr >= p.eoff[p.ne]) return;
    const int tile = p.pair_tile[pr];
    const int4 td = p.tiles[tile];
    const int jrow = pr - td.y, h = b_rows(td.z);
    uint8_t *sfb = p.sfbh + (int64_t)tile * KS_DN * NP * BS_ATOM;
    int s0 = lane < MT_UP ? p.tile_scale[(int64_t)tile * MT_UP + lane] : INT_MAX;
#pragma unroll
    for (int o = 16; o; o >>= 1) s0 = min(s0, __shfl_xor_sync(0xffffffffu, s0, o));
    for (int g0 = 0; g0 < G_DN; g0 += 32) {   // G_DN = 168 = 4 * 42: lanes of one k-step are all in or all out
        const int grp = g0 + lane;
        const bool live = grp < G_DN;
        uint8_t sc[NP] = {};
        if (live) {
            float w[16];
            const int d = s0 - HSHIFT;   // h as computed, in the tile's frame 2^(S0 - HSHIFT)
            const float f = d >= -126 ? pow2f(d) : 0.f;
            const float4 *src = reinterpret_cast<const float4 *>(p.hs + (int64_t)pr * INTER + grp * 16);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 v = src[i];
                w[4 * i] = v.x * f;
                w[4 * i + 1] = v.y * f;
                w[4 * i + 2] = v.z * f;
                w[4 * i + 3] = v.w * f;
            }
            uint32_t codes[NP][2];
            nvfp4_planes16(w, codes, sc);
#pragma unroll
            for (int pl = 0; pl < NP; ++pl)
                *reinterpret_cast<uint2 *>(p.hq + ((int64_t)pl * p.P + pr) * KB_DN + grp * 8) = make_uint2(codes[pl][0], codes[pl][1]);
        }
        // the four groups of k-step grp / 4 sit in lanes 4i .. 4i+3: gather their scale bytes in lane 4i
#pragma unroll
        for (int pl = 0; pl < NP; ++pl) {
            uint32_t v = sc[pl];
            v |= __shfl_down_sync(0xffffffffu, v, 1) << 8;
            v |= __shfl_down_sync(0xffffffffu, v, 2) << 16;
            if (live && !(lane & 3)) *reinterpret_cast<uint32_t *>(sfb + sfb_byte(grp >> 2, pl, jrow, h)) = v;
        }
    }
}

__device__ __forceinline__ void mma_nvfp4(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc,
                                          uint32_t tsfa, uint32_t tsfb) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(tsfa), "r"(tsfb)
        : "memory");
}

// Instruction descriptor of kind::mxf4nvf4: A, B e2m1 (format 1), K-major, e4m3 scales, M = 128, N = n, K = 64.
__device__ __forceinline__ uint32_t instr_desc_nvfp4(int n) {
    return (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// The grouped GEMM on block-scaled NVFP4 MMA; persistent: one CTA per SM walks the items (tile, 128 weight
// rows) i = blockIdx.x, blockIdx.x + gridDim.x, ... (consecutive items share a tile, whose planes stay in L2).
// Roles: warps 4..5 load the weight stages (TMA, 8 KB, 64-byte swizzle); warps 6..7 the NP activation planes
// of the stage (one 3-D TMA box: planes x pair rows x 64 B) and the planes' scale atoms (one 3 KB bulk copy,
// laid out by the plane kernels); warp 8 bulk-copies the item's 128 weight-scale rows into a slab and
// rearranges each stage's two weight atoms from it; warps 10..13 store the stage's atoms into its TMEM scale
// slot; warp 9 issues the MMAs into one of two TMEM accumulators while warps 0..3 drain the other (epilogue).
// Waits of the producer and epilogue roles: between polls the thread sleeps, so that polling warps leave the
// issue slots of their SM sub-partition to the MMA-issuing warp.
__device__ __forceinline__ bool mbar_wait_bo(uint64_t *bar, uint32_t parity, long long limit) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        __nanosleep(200);
        if (clock64() - t0 > limit) return false;
    }
    return true;
}

__device__ __forceinline__ bool lane_wait_bo(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *status,
                                             long long limit) {
    if (mbar_try_wait(bar, parity)) return true;
    const bool ok = !*abort_flag && mbar_wait_bo(bar, parity, limit);
    if (!ok) {
        set_error(status, DEV_ERR_TIMEOUT);
        *abort_flag = 1;
    }
    return ok;
}

__device__ __forceinline__ bool warp_wait_bo(uint64_t *bar, uint32_t parity, int lane, volatile int *abort_flag,
                                             int *status, long long limit) {
    bool ok = true;
    if (lane == 0) ok = lane_wait_bo(bar, parity, abort_flag, status, limit);
    return __shfl_sync(0xffffffffu, ok, 0);
}

template <int PH>
__global__ void __launch_bounds__(BS_THREADS, 1)
    pfb_gemm_kernel(const Params p, const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ PlaneMaps tm_b) {
    constexpr int MT = PH == PH_UP ? MT_UP : MT_DN;
    constexpr int K = PH == PH_UP ? LAT : INTER;
    constexpr int NST = K / BS_BK;                     // stages per item
    constexpr int GP = PH == PH_UP ? G_UP : G_DN;      // scale bytes per weight row
    constexpr int KS = K / 64;                         // MMA k-steps per row
    using Plan = BsPlan<PH>;
    constexpr int S = Plan::STAGES;
    const int nitems = *p.tile_count * MT;

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_u32(smem_raw);
    uint8_t *sm = smem_raw + (((raw_base + 1023u) & ~1023u) - raw_base);
    const uint32_t sbase = smem_u32(sm);
    float *colsc = reinterpret_cast<float *>(sm + Plan::OFF_COLSC);
    float *red = reinterpret_cast<float *>(sm + Plan::OFF_RED);
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + Plan::OFF_BAR);
    uint64_t *empty = full + S;
    uint64_t *acc_full = empty + S;
    uint64_t *acc_empty = acc_full + 2;
    uint64_t *slab_full = acc_empty + 2;
    uint64_t *sf_src = slab_full + 2;    // [S] the stage's scale atoms are in shared memory (bulk copy + weight atoms)
    uint64_t *mma_drain = sf_src + S;    // after an abort: every MMA issued has completed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + Plan::OFF_TMEM);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sm + Plan::OFF_ABORT);
    // rec[s][r]: the last use (running stage count q) of stage s that role r armed or arrived for: 0 the weight
    // issuers (full, expect_tx), 1 the plane issuers (full and sf_src, expect_tx), 2 the weight-atom warp (sf_src),
    // 3.. the scale-store warps (full). Read only after an abort, to let every copy in flight land before the exit.
    int *rec = reinterpret_cast<int *>(sm + Plan::OFF_REC);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < S; s++) {
            // A and B expect_tx arrivals (codes) and one arrival per scale-store warp (the stage's scale factors
            // are in TMEM): the MMA thread waits on this one barrier per stage
            mbar_init(&full[s], 2 + BS_NSS);
            mbar_init(&sf_src[s], 2);   // B issuer's expect_tx for the planes' atoms, the weight-atom warp
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], 4);
            mbar_init(&slab_full[a], 1);
        }
        mbar_init(mma_drain, 1);
        *abort_flag = 0;
        for (int k = 0; k < S * 8; k++) rec[k] = -1;
        fence_mbar_init();
    }
    if (warp == BS_W_MMA) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(BS_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp >= BS_W_A && warp < BS_W_B) {
        // ------------------------------------------------------------ weights: codes [128 rows][64 B] per stage
        const int pr = warp - BS_W_A;
        if (lane == 0) {
            uint32_t q = 0;
            int4 td_next = blockIdx.x < nitems ? p.tiles[blockIdx.x / MT] : make_int4(0, 0, 0, 0);
            for (int i = blockIdx.x; i < nitems && !*abort_flag; i += gridDim.x) {
                const int4 td = td_next;
                if (i + (int)gridDim.x < nitems) td_next = p.tiles[(i + gridDim.x) / MT];
                const int mt = i % MT, e = PH == PH_DN_O && p.dn_compact ? td.w : td.x;
                const bool wide = fused_planes(b_rows(td.z));
                const int nst = wide ? (NST + 1) / 2 : NST;
                bool ok = true;
                for (int kt = 0; kt < nst; kt++, q++) {
                    if ((int)(q % BS_NA) != pr) continue;
                    const int s = q % S;
                    if (!lane_wait_bo(&empty[s], ((q / S) & 1) ^ 1, abort_flag, p.status, p.wait_cycles)) {
                        ok = false;
                        break;
                    }
                    const int nh = wide ? min(2, NST - 2 * kt) : 1, k0 = wide ? 2 * kt : kt;
                    mbar_expect_tx(&full[s], (uint32_t)(nh * BS_A));
                    for (int hh = 0; hh < nh; hh++)
                        tma_load_3d(sm + s * BS_STAGE + hh * BS_A, &tm_w, (k0 + hh) * (BS_BK / 2),
                                    (PH == PH_UP ? 0 : p.dn_row0) + mt * BM, e, &full[s]);
                    atomicMax(&rec[s * 8 + 0], (int)q);
                }
                if (!ok) break;
            }
        }
        __syncwarp();
    } else if (warp >= BS_W_B && warp < BS_W_SF) {
        // ------------------------------------------------------------ activation planes [NP][rows][64 B] per stage
        //                                                              and their scale atoms [k-step][plane][512 B]
        const int pb = warp - BS_W_B;
        if (lane == 0) {
            const uint8_t *sfb = PH == PH_UP ? p.sfbx : p.sfbh;
            uint32_t q = 0;
            int4 td_next = blockIdx.x < nitems ? p.tiles[blockIdx.x / MT] : make_int4(0, 0, 0, 0);
            for (int i = blockIdx.x; i < nitems && !*abort_flag; i += gridDim.x) {
                const int4 td = td_next;
                if (i + (int)gridDim.x < nitems) td_next = p.tiles[(i + gridDim.x) / MT];
                const int n0 = td.y, np_ = b_rows(td.z);
                const CUtensorMap *map = &tm_b.m[(np_ >> 4) - 1];
                const uint8_t *sfb_tile = sfb + (int64_t)(i / MT) * KS * NP * BS_ATOM;
                const bool wide = fused_planes(np_);
                const int nst = wide ? (NST + 1) / 2 : NST;
                const int pbytes = NP * np_ * (BS_BK / 2);   // one 128-element half of the planes
                bool ok = true;
                for (int kt = 0; kt < nst; kt++, q++) {
                    if ((int)(q % BS_NB) != pb) continue;
                    const int s = q % S;
                    if (!lane_wait_bo(&empty[s], ((q / S) & 1) ^ 1, abort_flag, p.status, p.wait_cycles)) {
                        ok = false;
                        break;
                    }
                    const int nh = wide ? min(2, NST - 2 * kt) : 1, k0 = wide ? 2 * kt : kt;
                    uint8_t *st = sm + s * BS_STAGE;
                    // the atoms first, on their own barrier: the scale stores into TMEM need not wait for codes
                    mbar_expect_tx(&sf_src[s], (uint32_t)(nh * BS_SFB));
                    bulk_g2s_nohint(st + (wide ? BW_SFB : BS_A + BS_B), sfb_tile + (int64_t)k0 * BS_SFB,
                                    (uint32_t)(nh * BS_SFB), &sf_src[s]);
                    mbar_expect_tx(&full[s], (uint32_t)(nh * pbytes));
                    for (int hh = 0; hh < nh; hh++)
                        tma_load_3d(st + (wide ? BW_B + hh * pbytes : BS_A), map, (k0 + hh) * (BS_BK / 2), n0, 0,
                                    &full[s]);
                    atomicMax(&rec[s * 8 + 1], (int)q);
                }
                if (!ok) break;
            }
        }
        __syncwarp();
    } else if (warp == BS_W_SF) {
        // ------------------------------------------------------------ weight-scale atoms
        // The item's scale rows (128 rows x GP bytes, contiguous in the block) arrive by one bulk copy into one
        // of two slabs, the next item's copy in flight while this item is built. Stage kt takes bytes
        // 8kt .. 8kt+7 of each row: atom kk, lane L = rows L, L+32, L+64, L+96, 4 bytes each.
        uint8_t *slab = sm + Plan::OFF_SLAB;
        const uint8_t *wsc0 = PH == PH_UP ? p.store + O_US : p.dn_sc;
        const int64_t wstride = PH == PH_UP ? p.bstride : p.dn_bstride;
        // the weight block of a tile: the expert id, or for converted down halves the expert's rank among those used
        auto wexp = [&](const int4 &td) { return PH == PH_DN_O && p.dn_compact ? td.w : td.x; };
        uint32_t issued[2] = {0, 0}, done[2] = {0, 0};
        if (blockIdx.x < nitems) {
            if (lane == 0) {
                const int i = blockIdx.x;
                mbar_expect_tx(&slab_full[0], Plan::SLAB);
                bulk_g2s_nohint(slab, wsc0 + (int64_t)wexp(p.tiles[i / MT]) * wstride + (int64_t)(i % MT) * Plan::SLAB,
                                Plan::SLAB, &slab_full[0]);
            }
            issued[0] = 1;
        }
        uint32_t q = 0;
        for (int i = blockIdx.x, j = 0; i < nitems; i += gridDim.x, j++) {
            if (__shfl_sync(0xffffffffu, *abort_flag, 0)) break;   // one decision for the whole warp
            const int b = j & 1;
            const int inext = i + (int)gridDim.x;
            if (inext < nitems) {   // slab b ^ 1 was last read while building item j - 1
                __syncwarp();
                if (lane == 0) {
                    fence_async_smem();
                    mbar_expect_tx(&slab_full[b ^ 1], Plan::SLAB);
                    bulk_g2s_nohint(slab + (b ^ 1) * Plan::SLAB,
                                    wsc0 + (int64_t)wexp(p.tiles[inext / MT]) * wstride + (int64_t)(inext % MT) * Plan::SLAB,
                                    Plan::SLAB, &slab_full[b ^ 1]);
                }
                issued[b ^ 1]++;
            }
            if (!warp_wait_bo(&slab_full[b], (j >> 1) & 1, lane, abort_flag, p.status, p.wait_cycles)) break;
            mbar_try_wait(&slab_full[b], (j >> 1) & 1);   // completed phase: acquire for every lane
            done[b]++;
            const uint8_t *sl = slab + b * Plan::SLAB;
            const bool wide = fused_planes(b_rows(p.tiles[i / MT].z));
            const int nst = wide ? (NST + 1) / 2 : NST;
            bool ok = true;
            for (int kt = 0; kt < nst; kt++, q++) {
                const int s = q % S;
                if (!warp_wait_bo(&empty[s], ((q / S) & 1) ^ 1, lane, abort_flag, p.status, p.wait_cycles)) {
                    ok = false;
                    break;
                }
                const int nh = wide ? min(2, NST - 2 * kt) : 1, k0 = wide ? 2 * kt : kt;
                uint8_t *at = sm + s * BS_STAGE + (wide ? BW_SFA : BS_A + BS_B + BS_SFB);
                for (int hh = 0; hh < nh; hh++) {   // 128-element half: k-steps 2(k0+hh), 2(k0+hh)+1
                    uint2 w[4];
#pragma unroll
                    for (int g = 0; g < 4; g++)
                        w[g] = *reinterpret_cast<const uint2 *>(sl + (lane + 32 * g) * GP + 8 * (k0 + hh));
                    *reinterpret_cast<uint4 *>(at + (2 * hh) * BS_ATOM + lane * 16) = make_uint4(w[0].x, w[1].x, w[2].x, w[3].x);
                    *reinterpret_cast<uint4 *>(at + (2 * hh + 1) * BS_ATOM + lane * 16) = make_uint4(w[0].y, w[1].y, w[2].y, w[3].y);
                }
                fence_async_smem();   // generic-proxy atom stores, ordered before the async proxy's next use
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&sf_src[s]);
                    rec[s * 8 + 2] = (int)q;
                }
            }
            if (!ok) break;
        }
        // after an abort: let every slab copy still in flight land before the CTA exits (bounded waits)
        if (lane == 0)
            for (int b = 0; b < 2; b++)
                for (; done[b] < issued[b]; done[b]++)
                    if (!mbar_wait(&slab_full[b], done[b] & 1)) break;
        __syncwarp();
    } else if (warp == BS_W_MMA) {
        // ------------------------------------------------------------ scale factors -> TMEM, NP MMAs per k-step
        if (lane == 0) {
            // descriptors of 64-byte-swizzled K-major tiles (LBO 16, SBO 512): the constant part once, plus the
            // tile address / 16 (14 bits, shared memory < 256 KB)
            const uint64_t dbase = smem_desc(0, 16, 512, 4);
            int s = 0;
            uint32_t ph = 0;   // stage s and the parity of its current use, advanced per stage
            int n_next = blockIdx.x < nitems ? p.tiles[blockIdx.x / MT].z : 0;
            for (int i = blockIdx.x, j = 0; i < nitems && !*abort_flag; i += gridDim.x, j++) {
                const int n = n_next;
                if (i + (int)gridDim.x < nitems) n_next = p.tiles[(i + gridDim.x) / MT].z;
                const int np_ = b_rows(n);
                const bool fused = fused_planes(np_);
                const int a = j & 1;
                if (!lane_wait(&acc_empty[a], ((j >> 1) & 1) ^ 1, abort_flag, p.status, p.wait_cycles)) break;
                tc_fence_after();
                const uint32_t idesc = instr_desc_nvfp4(fused ? NP * np_ : (n + 15) & ~15);
                const uint32_t d = tmem + a * NT;
                const int nst = fused ? (NST + 1) / 2 : NST;   // fused tiles use wide stages
                const uint32_t pstride = (uint32_t)(np_ * (BS_BK / 2)) >> 4;   // one plane of B, in 16-byte units
                bool ok = true;
                for (int kt = 0; kt < nst; kt++) {
                    if (!lane_wait(&full[s], ph, abort_flag, p.status, p.wait_cycles)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t dst0 = dbase + ((sbase + (uint32_t)s * BS_STAGE) >> 4);
                    const uint32_t slot = tmem + BS_SF_COL + s * 32;
                    if (fused) {   // all planes as one MMA: N = NP * np_ rows of B, scales in the plane-0 atom
                        const int nk = 2 * min(2, NST - 2 * kt);
                        for (int kk = 0; kk < nk; kk++) {
                            const uint32_t half = (uint32_t)(kk >> 1), kb = (uint32_t)(kk & 1) * 2;
                            const uint64_t ad = dst0 + half * (BS_A >> 4) + kb;
                            const uint64_t bd = dst0 + (BW_B >> 4) + half * NP * pstride + kb;
                            mma_nvfp4(d, ad, bd, idesc, (kt | kk) != 0, slot + kk * 8, slot + kk * 8 + 4);
                        }
                    } else {
#pragma unroll
                        for (int kk = 0; kk < BS_KS; kk++) {
                            const uint32_t sfa = slot + kk * 16;
                            const uint64_t ad = dst0 + kk * 2;
#pragma unroll
                            for (int pl = 0; pl < NP; pl++) {
                                const uint64_t bd = dst0 + (BS_A >> 4) + pl * pstride + kk * 2;
                                mma_nvfp4(d, ad, bd, idesc, (kt | kk | pl) != 0, sfa, sfa + 4 + 4 * pl);
                            }
                        }
                    }
                    mma_commit(&empty[s]);
                    if (++s == S) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                mma_commit(&acc_full[a]);   // also after a failed wait: tracks every MMA issued
                if (!ok) break;
            }
        }
        __syncwarp();
    } else if (warp >= BS_W_SS) {
        // ------------------------------------------------------------ scale-factor atoms -> TMEM slot of the stage
        // tcgen05.st from four warps, warp w writing lane quarter w % 4: each quarter gets the 32-row pattern of
        // every atom (lane L, column c = bytes 16L + 4c .. 16L + 4c + 3), the layout a 32x128b.warpx4 copy
        // makes, without occupying the tensor pipe. Slot s is rewritten only after sf_src[s] of its next use,
        // which follows empty[s] (the MMAs that read the slot completed) through its producers.
        const uint32_t quarter = (uint32_t)(warp & 3) << 21;   // TMEM lane 32 * (warp % 4), in bits 16..
        uint32_t q = 0;
        for (int i = blockIdx.x; i < nitems; i += gridDim.x) {
            if (__shfl_sync(0xffffffffu, *abort_flag, 0)) break;   // one decision for the whole warp
            const bool wide = fused_planes(b_rows(p.tiles[i / MT].z));
            const int nst = wide ? (NST + 1) / 2 : NST;
            bool ok = true;
            for (int kt = 0; kt < nst; kt++, q++) {
                const int s = q % S;
                if (!warp_wait_bo(&sf_src[s], (q / S) & 1, lane, abort_flag, p.status, p.wait_cycles)) {
                    ok = false;
                    break;
                }
                mbar_try_wait(&sf_src[s], (q / S) & 1);   // completed phase: acquire for every lane
                if (wide) {
                    // per k-step kk: columns 8kk .. 8kk+3 weight atom, 8kk+4 .. 8kk+7 the plane-0 (all-plane) atom
                    const uint8_t *at = sm + s * BS_STAGE;
                    const int nh = min(2, NST - 2 * kt);
                    for (int hh = 0; hh < nh; hh++) {
                        uint32_t r[16];
#pragma unroll
                        for (int u = 0; u < 2; u++) {
                            const int kk = 2 * hh + u;
                            const uint4 a = *reinterpret_cast<const uint4 *>(at + BW_SFA + kk * BS_ATOM + lane * 16);
                            const uint4 b = *reinterpret_cast<const uint4 *>(at + BW_SFB + kk * NP * BS_ATOM + lane * 16);
                            r[8 * u + 0] = a.x, r[8 * u + 1] = a.y, r[8 * u + 2] = a.z, r[8 * u + 3] = a.w;
                            r[8 * u + 4] = b.x, r[8 * u + 5] = b.y, r[8 * u + 6] = b.z, r[8 * u + 7] = b.w;
                        }
                        tmem_st16(tmem + quarter + BS_SF_COL + s * 32 + hh * 16, r);
                    }
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&full[s]);
                        rec[s * 8 + 3 + (warp - BS_W_SS)] = (int)q;
                    }
                    continue;
                }
                const uint8_t *at = sm + s * BS_STAGE + BS_A + BS_B;
#pragma unroll
                for (int kk = 0; kk < BS_KS; kk++) {
                    uint32_t r[16];
                    const uint4 a = *reinterpret_cast<const uint4 *>(at + BS_SFB + kk * BS_ATOM + lane * 16);
                    r[0] = a.x, r[1] = a.y, r[2] = a.z, r[3] = a.w;
#pragma unroll
                    for (int pl = 0; pl < NP; pl++) {
                        const uint4 b = *reinterpret_cast<const uint4 *>(at + (kk * NP + pl) * BS_ATOM + lane * 16);
                        r[4 + 4 * pl] = b.x, r[5 + 4 * pl] = b.y, r[6 + 4 * pl] = b.z, r[7 + 4 * pl] = b.w;
                    }
                    tmem_st16(tmem + quarter + BS_SF_COL + s * 32 + kk * 16, r);
                }
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&full[s]);
                    rec[s * 8 + 3 + (warp - BS_W_SS)] = (int)q;
                }
            }
            if (!ok) break;
        }
    } else {
        // ------------------------------------------------------------ epilogue (warps 0..3 = TMEM lanes)
        const int m = tid;
        // The column scales of an item (one per pair: thread c < n owns pair c) are fetched into registers
        // while the previous item is drained and published to colsc[a] after it, so their global loads
        // stay off the path between two accumulators.
        int4 tdn = make_int4(0, 0, 0, 0);
        float vn = 0.f, s2n = 0.f;
        int tsn = INT_MAX;
        auto fetch = [&](int ii) {
            tdn = p.tiles[ii / MT];
            s2n = p.s2[(int64_t)tdn.x * 2 + (PH == PH_UP ? 0 : 1)];
            vn = 0.f;
            if (tid < tdn.z) vn = PH == PH_UP ? pow2f(-p.pair_exp[tdn.y + tid]) : p.pair_coef[tdn.y + tid];
            tsn = (PH != PH_UP && lane < MT_UP) ? p.tile_scale[(int64_t)(ii / MT) * MT_UP + lane] : INT_MAX;
        };
        auto publish = [&](int buf) {
            int s0 = tsn;   // down: the tile's smallest block exponent (tile_s0)
#pragma unroll
            for (int o = 16; o; o >>= 1) s0 = min(s0, __shfl_xor_sync(0xffffffffu, s0, o));
            if (tid < tdn.z)
                colsc[buf * NT + tid] = PH == PH_UP ? vn * s2n : vn * s2n * pow2f(min(HSHIFT - s0, 127));
        };
        if (blockIdx.x < nitems) {
            fetch(blockIdx.x);
            publish(0);
        }
        for (int i = blockIdx.x, j = 0; i < nitems; i += gridDim.x, j++) {
            const int tile = i / MT, mt = i % MT;
            const int4 td = tdn;
            const int n0 = td.y, n = td.z;
            const int a = j & 1;
            float *cs = colsc + a * NT;
            named_sync(1, 128);   // this item's column scales are visible; colsc[a ^ 1] is free
            const bool more = i + (int)gridDim.x < nitems;
            if (more) fetch(i + gridDim.x);
            const bool acc_ok = warp_wait_bo(&acc_full[a], (j >> 1) & 1, lane, abort_flag, p.status, p.wait_cycles);
            tc_fence_after();
            const uint32_t trow = tmem + a * NT + ((uint32_t)(warp * 32) << 16);
            // a fused-plane tile holds plane pl of pair c in column pl * h + c: the pair's value is the sum
            const int h = b_rows(n);
            const bool fused = fused_planes(h);
            auto acc32 = [&](int c0, float(&v)[32]) {
                tmem_ld32(trow + c0, v);
                if (fused) {
#pragma unroll
                    for (int pl = 1; pl < NP; pl++) {
                        float w[32];
                        tmem_ld32(trow + pl * h + c0, w);
#pragma unroll
                        for (int jj = 0; jj < 32; jj++) v[jj] += w[jj];
                    }
                }
            };
            bool released = false;
            if (PH == PH_UP) {
                // one pass: h = relu(u)^2 stored as f32 straight from registers (thread m -> neuron m: each
                // column is one coalesced 512-byte row segment), the block max tracked on the way; the
                // accumulator is released as soon as its last TMEM read is done
                float mx = 0.f;
                float *hrow = p.hs + (int64_t)n0 * INTER + mt * BM + m;
                if (acc_ok) {
                    for (int c0 = 0; c0 < n; c0 += 32) {
                        float v[32];
                        acc32(c0, v);
#pragma unroll
                        for (int jj = 0; jj < 32; jj++) {
                            if (c0 + jj < n) {
                                const float u = v[jj] * cs[c0 + jj];
                                const float hv = u > 0.f ? u * u : 0.f;
                                mx = fmaxf(mx, hv);
                                hrow[(int64_t)(c0 + jj) * INTER] = hv;
                            }
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[a]);
                released = true;
#pragma unroll
                for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                if (lane == 0) red[a * 4 + warp] = mx;
                named_sync(1, 128);
                mx = fmaxf(fmaxf(red[a * 4 + 0], red[a * 4 + 1]), fmaxf(red[a * 4 + 2], red[a * 4 + 3]));
                if (tid == 0) p.tile_scale[(int64_t)tile * MT_UP + mt] = mx > 0.f ? prescale_exp(mx, 15) : 127;
            } else if (acc_ok) {
                float *dst = p.op + (int64_t)n0 * LAT + mt * BM + m;
                for (int c0 = 0; c0 < n; c0 += 32) {
                    float v[32];
                    acc32(c0, v);
#pragma unroll
                    for (int jj = 0; jj < 32; jj++)
                        if (c0 + jj < n) dst[(int64_t)(c0 + jj) * LAT] = v[jj] * cs[c0 + jj];
                }
            }
            if (!released) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[a]);
            }
            if (more) publish(a ^ 1);
        }
    }
    tc_fence_before();
    __syncthreads();
    const bool aborted = *abort_flag != 0;
    if (warp == BS_W_MMA) {
        // after an abort an accumulator may not have been waited for (two commits to one acc_full barrier can
        // then be pending, which a parity wait cannot tell apart): one more commit, on a barrier of its own,
        // arrives once every MMA this thread issued has completed
        if (aborted && lane == 0) {
            mma_commit(mma_drain);
            mbar_wait(mma_drain, 0);
        }
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BS_TMEM_COLS) : "memory");
    } else if (aborted && tid == 0) {
        // After an abort, copies may still be in flight into stages whose barrier phase will never complete.
        // Each stage has at most one pending phase per barrier (a producer arms use q + S only after the
        // consumers released use q). Its use is the largest one any role recorded; the roles that have not
        // arrived for it are arrived for here, so the phase completes exactly when the bytes still in flight
        // have landed, and that completion is waited for (bounded) before the CTA's shared memory is released.
        for (int s = 0; s < S; s++) {
            const int *r = rec + s * 8;
            int qf = r[0];   // full[s]: the weight issuers, the plane issuers, the scale-store warps
            for (int k = 1; k < 3 + BS_NSS; k++)
                if (k != 2) qf = max(qf, r[k]);
            if (qf >= 0) {
                for (int k = 0; k < 3 + BS_NSS; k++)
                    if (k != 2 && r[k] < qf) mbar_arrive(&full[s]);
                mbar_wait(&full[s], (uint32_t)(qf / S) & 1);
            }
            const int qs = max(r[1], r[2]);   // sf_src[s]: the plane issuers (atoms), the weight-atom warp
            if (qs >= 0) {
                if (r[1] < qs) mbar_arrive(&sf_src[s]);
                if (r[2] < qs) mbar_arrive(&sf_src[s]);
                mbar_wait(&sf_src[s], (uint32_t)(qs / S) & 1);
            }
        }
    }
}

// ------------------------------------------------------------------------------------------ T -> orig down
// A T-layout store keeps dnT_w [2688 neurons][512 B] (neuron-major: the output rows of a neuron together),
// which FP4 operands of the tensor core cannot take (they must be K-major). For a prompt the down halves of the
// experts the prompt uses are converted once into dconv, [1024 rows][1344 B] codes then [1024][168] scales
// per expert - the orig layout, as from_T_fast does for the reference's prompt path (nem_super.py:324-328) -
// and the block-scaled down GEMM reads them there. Experts with no pair are skipped.
constexpr int DCV_R = 64, DCV_C = 128;   // scales: 128 rows per CTA; codes: 64 neurons x 256 rows per CTA

// 8 x 8 nibble transpose in registers: w[i] holds nibbles (i, 0..7) at bits 4j; afterwards w[j] holds
// nibbles (0..7, j) at bits 4i. Three rounds of masked swaps (16-bit halves, bytes, nibbles).
__device__ __forceinline__ void nibble_transpose8(uint32_t (&w)[8]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t a = w[i], b = w[i + 4];
        w[i] = (a & 0x0000FFFFu) | (b << 16);
        w[i + 4] = (a >> 16) | (b & 0xFFFF0000u);
    }
#pragma unroll
    for (int i = 0; i < 8; i += (i & 1) ? 3 : 1) {   // i = 0, 1, 4, 5
        const uint32_t a = w[i], b = w[i + 2];
        w[i] = (a & 0x00FF00FFu) | ((b & 0x00FF00FFu) << 8);
        w[i + 2] = ((a >> 8) & 0x00FF00FFu) | (b & 0xFF00FF00u);
    }
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        const uint32_t a = w[i], b = w[i + 1];
        w[i] = (a & 0x0F0F0F0Fu) | ((b & 0x0F0F0F0Fu) << 4);
        w[i + 1] = ((a >> 4) & 0x0F0F0F0Fu) | (b & 0xF0F0F0F0u);
    }
}

// dnT_w [2688 neurons][512 B] -> dn_w [1024 rows][1344 B]: a CTA stages 64 neurons x 256 output rows (128 B
// per neuron) in shared memory; thread (a, b) transposes the 8 x 8 nibble block of neurons 8a.. and rows 8b..
// and writes 4 bytes to each of its 8 output rows (8 consecutive lanes fill one 32-byte sector).
__global__ void __launch_bounds__(256) pf_dnT_codes_kernel(const Params p) {
    __shared__ uint32_t tile[DCV_R][33];
    const int e = blockIdx.z, ce = p.ecomp[e];
    if (ce < 0) return;
    const int n0 = blockIdx.x * DCV_R, r0 = blockIdx.y * 256;
    const uint8_t *A = p.store + (int64_t)e * p.bstride + O_DW;   // [2688][512 B]
    uint8_t *B = p.dconv + (int64_t)ce * DC_STRIDE;                // [1024][1344 B]
    const int tid = threadIdx.x;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int idx = tid + 256 * k, row = idx >> 3, part = idx & 7;
        const uint4 v = *reinterpret_cast<const uint4 *>(A + (int64_t)(n0 + row) * (LAT / 2) + r0 / 2 + 16 * part);
        tile[row][4 * part] = v.x, tile[row][4 * part + 1] = v.y, tile[row][4 * part + 2] = v.z, tile[row][4 * part + 3] = v.w;
    }
    __syncthreads();
    const int a = tid & 7, b = tid >> 3;
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = tile[8 * a + i][b];
    nibble_transpose8(w);
#pragma unroll
    for (int j = 0; j < 8; ++j)
        *reinterpret_cast<uint32_t *>(B + (int64_t)(r0 + 8 * b + j) * KB_DN + n0 / 2 + 4 * a) = w[j];
}

// dnT_s [168 groups][1024 rows] -> [1024 rows][168 groups] for 128 rows per CTA.
__global__ void __launch_bounds__(256) pf_dnT_scales_kernel(const Params p) {
    __shared__ __align__(16) uint8_t s[G_DN][DCV_C + 4];
    const int e = blockIdx.y, ce = p.ecomp[e];
    if (ce < 0) return;
    const int r0 = blockIdx.x * DCV_C;
    const uint8_t *A = p.store + (int64_t)e * p.bstride + O_DS;   // [168][1024]
    uint8_t *B = p.dconv + (int64_t)ce * DC_STRIDE + DC_W;         // [1024][168]
    for (int i = threadIdx.x; i < G_DN * (DCV_C / 16); i += blockDim.x) {
        const int g = i >> 3, part = i & 7;
        const uint4 v = *reinterpret_cast<const uint4 *>(A + (int64_t)g * LAT + r0 + 16 * part);
        uint32_t *d = reinterpret_cast<uint32_t *>(&s[g][16 * part]);
        d[0] = v.x, d[1] = v.y, d[2] = v.z, d[3] = v.w;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < DCV_C * (G_DN / 4); i += blockDim.x) {   // 4 scale bytes per store
        const int rr = i / (G_DN / 4), g4 = (i - rr * (G_DN / 4)) * 4;
        const uint32_t v = (uint32_t)s[g4][rr] | ((uint32_t)s[g4 + 1][rr] << 8) | ((uint32_t)s[g4 + 2][rr] << 16) |
                           ((uint32_t)s[g4 + 3][rr] << 24);
        *reinterpret_cast<uint32_t *>(B + (int64_t)(r0 + rr) * G_DN + g4) = v;
    }
}

// ------------------------------------------------------------------------------------------ host
struct WsLayout {
    size_t status, tile_count, cnt, eoff, toff, ecomp, chunk_hist, tiles, pair_tok, pair_coef, pair_pos, pair_exp, tile_scale,
        hs, op, pair_tile, xq, hq, sfbx, sfbh, dconv, xtq, xtsc, xt_exp, total;
    int P, nchunks, tiles_cap;
};

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

inline WsLayout ws_layout(int T, int topk, int ne, bool layout_T) {
    WsLayout L{};
    L.P = T * topk;
    L.nchunks = (T + CHUNK_T - 1) / CHUNK_T;
    L.tiles_cap = (L.P + NT - 1) / NT + (ne < L.P ? ne : L.P);
    size_t o = 0;
    auto take = [&](size_t bytes) {
        const size_t at = o;
        o = align_up(o + bytes, 256);
        return at;
    };
    L.status = take(64);
    L.tile_count = take(4);
    L.cnt = take(sizeof(int) * ne);
    L.eoff = take(sizeof(int) * (ne + 1));
    L.toff = take(sizeof(int) * ne);
    L.ecomp = take(sizeof(int) * ne);
    L.chunk_hist = take(sizeof(int) * (size_t)L.nchunks * ne);
    L.tiles = take(sizeof(int4) * (size_t)L.tiles_cap);
    L.pair_tok = take(sizeof(int) * (size_t)L.P);
    L.pair_coef = take(sizeof(float) * (size_t)L.P);
    L.pair_pos = take(sizeof(int) * (size_t)L.P);
    L.pair_exp = take(sizeof(int) * (size_t)L.P);
    L.tile_scale = take(sizeof(int) * (size_t)L.tiles_cap * MT_UP);
    L.hs = take((size_t)L.P * INTER * 4);   // f32 h
    L.op = take((size_t)L.P * LAT * 4);
    L.pair_tile = take(sizeof(int) * (size_t)L.P);
    L.xq = take((size_t)NP * L.P * (LAT / 2));
    L.xtq = take((size_t)NP * T * (LAT / 2));
    L.xtsc = take((size_t)NP * T * G_UP);
    L.xt_exp = take(sizeof(int) * (size_t)T);
    L.hq = take((size_t)NP * L.P * KB_DN);
    L.sfbx = take((size_t)L.tiles_cap * KS_UP * NP * BS_ATOM);
    // T layout: the converted down halves of the experts with pairs (at most min(ne, P) of them)
    L.dconv = take(layout_T ? (size_t)(ne < L.P ? ne : L.P) * DC_STRIDE : 0);
    L.sfbh = take((size_t)L.tiles_cap * KS_DN * NP * BS_ATOM);
    L.total = o;
    return L;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    });
    return fn;
}

// The store as a u8 tensor [ne][BLOCK / pitch][pitch] (expert stride bstride), for TMA boxes of
// {box_x bytes, box_y rows} out of one block region.
inline bool make_store_map(CUtensorMap *m, const void *store, int64_t bstride, int ne, int pitch, int box_x,
                           int box_y, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_NONE, int64_t span = BLOCK) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)pitch, (cuuint64_t)(span / pitch), (cuuint64_t)ne};
    const cuuint64_t strides[2] = {(cuuint64_t)pitch, (cuuint64_t)bstride};
    const cuuint32_t box[3] = {(cuuint32_t)box_x, (cuuint32_t)box_y, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(store), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// NVFP4 planes [NP][P][row_bytes] u8 -> map with boxes {64 B, box_rows, NP} and 64-byte swizzle (rows past P
// read as zero).
inline bool make_plane_map(CUtensorMap *m, void *base, int64_t P, int row_bytes, int box_rows) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)row_bytes, (cuuint64_t)P, (cuuint64_t)NP};
    const cuuint64_t strides[2] = {(cuuint64_t)row_bytes, (cuuint64_t)P * row_bytes};
    const cuuint32_t box[3] = {(cuuint32_t)(BS_BK / 2), (cuuint32_t)box_rows, (cuuint32_t)NP};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

std::atomic<uint64_t> g_smem_up{0}, g_smem_dn_o{0};
std::atomic<long long> g_wait_cycles[MAX_DEVICES];   // 0: the default bound

} // namespace pf
} // namespace qmoe

using namespace qmoe;

extern "C" {

size_t qmoe_prefill_workspace_bytes(int T, int topk, int n_experts, int layout_T) {
    if (T < 1 || T > pf::MAX_T || topk < 1 || topk > pf::MAX_TOPK || n_experts < 1 || n_experts > pf::MAX_NE) return 0;
    return pf::ws_layout(T, topk, n_experts, layout_T != 0).total;
}

int qmoe_prefill_grouped(const uint8_t *store, int64_t block_stride, int n_experts, int layout_T, const int32_t *ids,
                         const float *weights, const float *s2, const void *x, int x_dtype, int T, int topk, float *out,
                         void *workspace, size_t workspace_bytes, void *stream) {
    using namespace qmoe::pf;
    if (!store || !ids || !weights || !s2 || !x || !out || !workspace) return QMOE_ERR_NULL;
    if (T < 1 || T > MAX_T || topk < 1 || topk > MAX_TOPK || n_experts < 1 || n_experts > MAX_NE)
        return QMOE_ERR_SHAPE;
    if (block_stride < BLOCK) return QMOE_ERR_SHAPE;
    if (!valid_dtype(x_dtype)) return QMOE_ERR_DTYPE;
    if ((block_stride & 15) || !aligned16(store) || !aligned16(x) || !aligned16(out) || !aligned4(ids) ||
        !aligned4(weights) || !aligned4(s2) || (reinterpret_cast<uintptr_t>(workspace) & 255u))
        return QMOE_ERR_ALIGN;
    const WsLayout L = ws_layout(T, topk, n_experts, layout_T != 0);
    if (workspace_bytes < L.total) return QMOE_ERR_WORKSPACE;
    int dev;
    DeviceInfo *di;
    if (int rc = current_device(&dev, &di)) return rc;

    uint8_t *ws = static_cast<uint8_t *>(workspace);
    Params p{};
    p.store = store;
    p.bstride = block_stride;
    p.ne = n_experts;
    p.ids = ids;
    p.wts = weights;
    p.s2 = s2;
    p.x = x;
    p.x_dtype = x_dtype;
    p.T = T;
    p.topk = topk;
    p.P = L.P;
    p.nchunks = L.nchunks;
    p.tiles_cap = L.tiles_cap;
    p.out = out;
    p.status = reinterpret_cast<int *>(ws + L.status);
    const long long wc = g_wait_cycles[dev].load(std::memory_order_relaxed);
    p.wait_cycles = wc > 0 ? wc : WAIT_CYCLES;
    p.tile_count = reinterpret_cast<int *>(ws + L.tile_count);
    p.cnt = reinterpret_cast<int *>(ws + L.cnt);
    p.eoff = reinterpret_cast<int *>(ws + L.eoff);
    p.toff = reinterpret_cast<int *>(ws + L.toff);
    p.ecomp = reinterpret_cast<int *>(ws + L.ecomp);
    p.chunk_hist = reinterpret_cast<int *>(ws + L.chunk_hist);
    p.tiles = reinterpret_cast<int4 *>(ws + L.tiles);
    p.pair_tok = reinterpret_cast<int *>(ws + L.pair_tok);
    p.pair_coef = reinterpret_cast<float *>(ws + L.pair_coef);
    p.pair_pos = reinterpret_cast<int *>(ws + L.pair_pos);
    p.pair_exp = reinterpret_cast<int *>(ws + L.pair_exp);
    p.tile_scale = reinterpret_cast<int *>(ws + L.tile_scale);
    p.hs = reinterpret_cast<float *>(ws + L.hs);
    p.dconv = ws + L.dconv;
    if (layout_T) {   // the down GEMM reads the converted halves
        p.dn_w = p.dconv;
        p.dn_sc = p.dconv + DC_W;
        p.dn_bstride = DC_STRIDE;
        p.dn_row0 = 0;
        p.dn_compact = 1;
    } else {
        p.dn_w = store;
        p.dn_sc = store + O_DS;
        p.dn_bstride = block_stride;
        p.dn_row0 = ROW1344_DW;
    }
    p.op = reinterpret_cast<float *>(ws + L.op);
    p.pair_tile = reinterpret_cast<int *>(ws + L.pair_tile);
    p.xq = ws + L.xq;
    p.xtq = ws + L.xtq;
    p.xtsc = ws + L.xtsc;
    p.xt_exp = reinterpret_cast<int *>(ws + L.xt_exp);
    p.hq = ws + L.hq;
    p.sfbx = ws + L.sfbx;
    p.sfbh = ws + L.sfbh;

    // both halves: block-scaled NVFP4 on the weights as stored (the down half of a T-layout store converted
    // first), the activations as NVFP4 planes
    PlaneMaps xm, hm;
    CUtensorMap wu, wdo;
    for (int k = 0; k < NBOX; k++) {
        if (!make_plane_map(&xm.m[k], p.xq, L.P, LAT / 2, 16 * (k + 1)) ||
            !make_plane_map(&hm.m[k], p.hq, L.P, KB_DN, 16 * (k + 1)))
            return QMOE_ERR_LAUNCH;
    }
    if (!make_store_map(&wu, store, block_stride, n_experts, KB_UP, BS_BK / 2, BM, CU_TENSOR_MAP_SWIZZLE_64B))
        return QMOE_ERR_LAUNCH;
    const int n_conv = n_experts < L.P ? n_experts : L.P;   // converted halves: one per expert with pairs
    if (layout_T ? !make_store_map(&wdo, p.dconv, DC_STRIDE, n_conv, KB_DN, BS_BK / 2, BM, CU_TENSOR_MAP_SWIZZLE_64B,
                                   DC_STRIDE)
                 : !make_store_map(&wdo, store, block_stride, n_experts, KB_DN, BS_BK / 2, BM, CU_TENSOR_MAP_SWIZZLE_64B))
        return QMOE_ERR_LAUNCH;
    auto up = pfb_gemm_kernel<PH_UP>;
    auto dn = pfb_gemm_kernel<PH_DN_O>;
    if (!ensure_smem(up, BsPlan<PH_UP>::SMEM, dev, g_smem_up) || !ensure_smem(dn, BsPlan<PH_DN_O>::SMEM, dev, g_smem_dn_o))
        return QMOE_ERR_LAUNCH;

    cudaStream_t st = as_stream(stream);
    pf_hist_kernel<<<L.nchunks, 256, 0, st>>>(p);
    pf_chunkscan_kernel<<<(n_experts + 7) / 8, 256, 0, st>>>(p);
    pf_scan_kernel<<<1, 1024, 0, st>>>(p);
    pf_place_kernel<<<L.nchunks, 32, 0, st>>>(p);
    pf_xtok_kernel<<<(T + 7) / 8, 256, 0, st>>>(p);
    pf_xplanes_kernel<<<(L.P + 7) / 8, 256, 0, st>>>(p);
    if (layout_T) {
        pf_dnT_codes_kernel<<<dim3(INTER / DCV_R, LAT / 256, n_experts), 256, 0, st>>>(p);
        pf_dnT_scales_kernel<<<dim3(LAT / DCV_C, n_experts), 256, 0, st>>>(p);
    }
    up<<<di->sms, BS_THREADS, BsPlan<PH_UP>::SMEM, st>>>(p, wu, xm);
    pf_hplanes_kernel<<<(L.P + 7) / 8, 256, 0, st>>>(p);
    dn<<<di->sms, BS_THREADS, BsPlan<PH_DN_O>::SMEM, st>>>(p, wdo, hm);
    pf_combine_kernel<<<T, 256, 0, st>>>(p);
    return launch_status();
}

int qmoe_set_wait_cycles(long long cycles) {
    int dev;
    DeviceInfo *di;
    if (int rc = current_device(&dev, &di)) return rc;
    pf::g_wait_cycles[dev].store(cycles > 0 ? cycles : 0, std::memory_order_relaxed);
    return QMOE_OK;
}

} // extern "C"
