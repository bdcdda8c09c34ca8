// Dense FP8 / NVFP4 GEMVs (dense_q.py:35-136) and the exact dequantizer `dequant_rows`
// (dense_q.py:179-188) for sm_100a. The GEMV body is gemv_kernel (gemv.cuh); this file picks its
// compile-time shape (chunks per lane, vector count) and the grid: about two CTAs per SM, each CTA a
// contiguous run of rows so that the activation vectors are staged once per CTA.
#include "common.cuh"
#include "gemv.cuh"
#include "host.h"

namespace qmoe {

template <int FMT, int CPL, int M, bool VF32>
static int launch_dense_t(const GemvArgs &g, cudaStream_t st, int dev, const DeviceInfo &di) {
    static std::atomic<uint64_t> done{0};
    auto kern = gemv_kernel<FMT, GM_DENSE, CPL, M, VF32>;
    const size_t smem = gemv_smem_bytes(VF32, M, g.K);
    if (smem > di.smem_optin) return QMOE_ERR_SHAPE;
    if (!ensure_smem(kern, smem, dev, done)) return QMOE_ERR_LAUNCH;
    const int unit = 2 * GEMV_WARPS;  // rows one pass of the CTA covers
    const int target = 2 * di.sms;
    int rows = (g.N + target - 1) / target;
    rows = (rows + unit - 1) / unit * unit;
    const int grid = (g.N + rows - 1) / rows;
    kern<<<grid, GEMV_THREADS, smem, st>>>(g, rows);
    return launch_status();
}

// fp32 activations are staged and multiplied in fp32; bf16 / f16 ones as exactly prescaled f16.
template <int FMT, int CPL, bool VF32>
static int launch_dense_v(const GemvArgs &g, cudaStream_t st, int dev, const DeviceInfo &di) {
    switch (g.M) {
    case 1: return launch_dense_t<FMT, CPL, 1, VF32>(g, st, dev, di);
    case 2: return launch_dense_t<FMT, CPL, 2, VF32>(g, st, dev, di);
    case 3: return launch_dense_t<FMT, CPL, 3, VF32>(g, st, dev, di);
    case 4: return launch_dense_t<FMT, CPL, 4, VF32>(g, st, dev, di);
    default: return QMOE_ERR_SHAPE;
    }
}

template <int FMT, int CPL>
static int launch_dense_m(const GemvArgs &g, cudaStream_t st, int dev, const DeviceInfo &di) {
    if constexpr (FMT == 2) {
        return launch_dense_v<FMT, CPL, true>(g, st, dev, di);
    } else {
        return g.x_dtype == QMOE_DT_F32 ? launch_dense_v<FMT, CPL, true>(g, st, dev, di)
                                        : launch_dense_v<FMT, CPL, false>(g, st, dev, di);
    }
}

template <int FMT>
static int launch_dense(const GemvArgs &g, cudaStream_t st, int dev, const DeviceInfo &di) {
    const int nch = (FMT == 1 ? g.K / 2 : FMT == 2 ? g.K * 2 : g.K) / 16;
    const int need = (nch + 31) / 32;
    if (need <= 2) return launch_dense_m<FMT, 2>(g, st, dev, di);
    if (need <= 4) return launch_dense_m<FMT, 4>(g, st, dev, di);
    return launch_dense_m<FMT, 8>(g, st, dev, di);
}

// dense_q.py:179-188: FP8 -> e4m3 * s; NVFP4 -> e2m1 * (e4m3 * s), in fp32, stored as OUT. One thread per byte.
template <typename OUT>
__device__ __forceinline__ OUT cvt_out(float v);
template <> __device__ __forceinline__ float cvt_out<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 cvt_out<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half cvt_out<__half>(float v) { return __float2half_rn(v); }

template <typename OUT>
__global__ void dequant_rows_kernel(int fmt, const uint8_t *__restrict__ w, const uint8_t *__restrict__ sc,
                                    const float *__restrict__ s, int64_t K, int64_t r0, int64_t r1,
                                    OUT *__restrict__ out) {
    const int64_t KB = fmt == 0 ? K : K / 2;
    const int64_t total = (r1 - r0) * KB;
    const float sv = *s;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t rr = i / KB, b = i - rr * KB, n = r0 + rr;
        const uint8_t v = w[n * KB + b];
        if (fmt == 0) {
            out[rr * K + b] = cvt_out<OUT>(__fmul_rn(e4m3_f32(v), sv));
        } else {
            const float f = __fmul_rn(e4m3_f32(sc[n * (K / 16) + (2 * b) / 16]), sv);
            out[rr * K + 2 * b] = cvt_out<OUT>(__fmul_rn(e2m1_f32(v), f));
            out[rr * K + 2 * b + 1] = cvt_out<OUT>(__fmul_rn(e2m1_f32((uint32_t)v >> 4), f));
        }
    }
}

} // namespace qmoe

using namespace qmoe;

extern "C" {

int dq_gemv_fp8(const uint8_t *w, const float *s, const void *x, int x_dtype, int M, int N, int K, float *y,
                void *stream) {
    if (!w || !s || !x || !y) return QMOE_ERR_NULL;
    if (M < 1 || M > 4 || N < 1 || K < 16 || (K % 16)) return QMOE_ERR_SHAPE;
    if (!aligned16(w)) return QMOE_ERR_ALIGN;
    if (!valid_dtype(x_dtype)) return QMOE_ERR_DTYPE;
    int dev;
    DeviceInfo *di;
    if (int e = current_device(&dev, &di)) return e;
    GemvArgs g{};
    g.w = w;
    g.s = s;
    g.x = x;
    g.x_dtype = x_dtype;
    g.y = y;
    g.M = M;
    g.N = N;
    g.K = K;
    return launch_dense<0>(g, as_stream(stream), dev, *di);
}

int dq_gemv_nvfp4(const uint8_t *w, const uint8_t *sc, const float *s2, const void *x, int x_dtype, int M, int N,
                  int K, float *y, void *stream) {
    if (!w || !sc || !s2 || !x || !y) return QMOE_ERR_NULL;
    if (M < 1 || M > 4 || N < 1 || K < 32 || (K % 32)) return QMOE_ERR_SHAPE;
    if (!aligned16(w) || (reinterpret_cast<uintptr_t>(sc) & 1u)) return QMOE_ERR_ALIGN;
    if (!valid_dtype(x_dtype)) return QMOE_ERR_DTYPE;
    int dev;
    DeviceInfo *di;
    if (int e = current_device(&dev, &di)) return e;
    GemvArgs g{};
    g.w = w;
    g.sc = sc;
    g.s = s2;
    g.x = x;
    g.x_dtype = x_dtype;
    g.y = y;
    g.M = M;
    g.N = N;
    g.K = K;
    return launch_dense<1>(g, as_stream(stream), dev, *di);
}

int dq_gemv_nvfp4_bf16(const uint8_t *w, const uint8_t *sc, const float *s2, const void *x, int x_dtype, int M, int N,
                       int K, int epilogue, const uint16_t *residual, uint16_t *y, void *stream) {
    if (!w || !sc || !s2 || !x || !y || (epilogue == 2 && !residual)) return QMOE_ERR_NULL;
    if (epilogue < 0 || epilogue > 2 || M < 1 || M > 4 || N < 1 || K < 32 || (K % 32)) return QMOE_ERR_SHAPE;
    if (!aligned16(w) || (reinterpret_cast<uintptr_t>(sc) & 1u)) return QMOE_ERR_ALIGN;
    if (!valid_dtype(x_dtype)) return QMOE_ERR_DTYPE;
    int dev;
    DeviceInfo *di;
    if (int e = current_device(&dev, &di)) return e;
    GemvArgs g{};
    g.w = w;
    g.sc = sc;
    g.s = s2;
    g.x = x;
    g.x_dtype = x_dtype;
    g.M = M;
    g.N = N;
    g.K = K;
    g.out_op = epilogue == 0 ? 3 : epilogue;   // 3: the plain bf16 cast (neither 1 nor 2 below)
    g.ybf = y;
    g.res = residual;
    return launch_dense<1>(g, as_stream(stream), dev, *di);
}

int dq_gemv_bf16(const uint16_t *w, const void *x, int x_dtype, int M, int N, int K, int epilogue,
                 const uint16_t *residual, uint16_t *y, void *stream) {
    if (!w || !x || !y || (epilogue == 2 && !residual)) return QMOE_ERR_NULL;
    if (epilogue < 0 || epilogue > 2 || M < 1 || M > 4 || N < 1 || K < 8 || (K % 8)) return QMOE_ERR_SHAPE;
    if (!aligned16(w)) return QMOE_ERR_ALIGN;
    if (!valid_dtype(x_dtype) && x_dtype != QMOE_DT_F32_AS_BF16) return QMOE_ERR_DTYPE;
    int dev;
    DeviceInfo *di;
    if (int e = current_device(&dev, &di)) return e;
    GemvArgs g{};
    g.w = reinterpret_cast<const uint8_t *>(w);
    g.x = x;
    g.x_dtype = x_dtype;
    g.M = M;
    g.N = N;
    g.K = K;
    g.out_op = epilogue == 0 ? 3 : epilogue;
    g.ybf = y;
    g.res = residual;
    return launch_dense<2>(g, as_stream(stream), dev, *di);
}

int dq_dequant_rows(int fmt, const uint8_t *w, const uint8_t *sc, const float *s, int64_t N, int64_t K, int64_t r0,
                    int64_t r1, void *out, int out_dtype, void *stream) {
    if (!w || !s || !out || (fmt == 1 && !sc)) return QMOE_ERR_NULL;
    if ((fmt != 0 && fmt != 1) || K < 16 || (K % 16) || r0 < 0 || r1 < r0 || r1 > N) return QMOE_ERR_SHAPE;
    if (!valid_dtype(out_dtype)) return QMOE_ERR_DTYPE;
    if (int e = current_device(nullptr, nullptr)) return e;
    if (r1 == r0) return QMOE_OK;
    const int64_t total = (r1 - r0) * (fmt == 0 ? K : K / 2);
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 64) blocks = 148 * 64;
    cudaStream_t st = as_stream(stream);
    if (out_dtype == QMOE_DT_BF16)
        dequant_rows_kernel<<<(unsigned)blocks, 256, 0, st>>>(fmt, w, sc, s, K, r0, r1, static_cast<__nv_bfloat16 *>(out));
    else if (out_dtype == QMOE_DT_F16)
        dequant_rows_kernel<<<(unsigned)blocks, 256, 0, st>>>(fmt, w, sc, s, K, r0, r1, static_cast<__half *>(out));
    else
        dequant_rows_kernel<<<(unsigned)blocks, 256, 0, st>>>(fmt, w, sc, s, K, r0, r1, static_cast<float *>(out));
    return launch_status();
}

} // extern "C"
