// Expert-block layout conversions and dequantization for sm_100a.
//
//   from_T (qmoe_ns.py:345-353 from_T_fast, :367-375 from_T) and to_T (repack_T.py:27-35,
//   qmoe_ns.py:356-364) are byte permutations of the down half of a block:
//     - the codes are a 4-bit matrix transpose, [2688 neuron x 1024 row] <-> [1024 row x 2688 neuron],
//       done in 64 x 128-nibble tiles through shared memory into a caller scratch buffer, then copied
//       back over the block with one strided device-to-device copy;
//     - the 172,032 scale bytes of a block ([168 x 1024] <-> [1024 x 168]) are transposed in place by
//       one CTA that holds the whole region in shared memory.
//   block_deq (qmoe_ns.py:407-412) expands one orig-layout block into fp32 matrices, bit-exact:
//   (e2m1 * e4m3) * weight_scale_2 with round-to-nearest fp32 multiplies, as deq does (qmoe_ns.py:395-404).
#include "common.cuh"
#include "host.h"

namespace qmoe {

constexpr int NT_R = 64;    // tile rows of the source nibble matrix
constexpr int NT_C = 128;   // tile columns (nibbles) of the source
constexpr int NT_THREADS = 256;
constexpr int64_t DW_BYTES = O_DS - O_DW;      // 1,376,256 code bytes of down
constexpr int64_t DS_BYTES = BLOCK - O_DS;     // 172,032 scale bytes of down

// Transpose the nibble matrix A [R][C] (C nibbles per row, two per byte, low nibble = even column)
// of block e into B [C][R] at dst + e * DW_BYTES.
__global__ void __launch_bounds__(NT_THREADS) nibble_transpose_kernel(const uint8_t *__restrict__ blks, int R, int C,
                                                                      uint8_t *__restrict__ dst) {
    __shared__ __align__(16) uint8_t tile[NT_R][NT_C / 2 + 16];
    const int64_t e = blockIdx.z;
    const int r0 = blockIdx.x * NT_R, c0 = blockIdx.y * NT_C;
    const uint8_t *A = blks + e * BLOCK + O_DW;
    uint8_t *B = dst + e * DW_BYTES;
    const int tid = threadIdx.x;
    {   // read 64 rows x 64 bytes: one 16-byte piece per thread
        const int rr = tid >> 2, part = tid & 3;
        const uint4 v = *reinterpret_cast<const uint4 *>(A + (int64_t)(r0 + rr) * (C / 2) + c0 / 2 + 16 * part);
        *reinterpret_cast<uint4 *>(&tile[rr][16 * part]) = v;
    }
    __syncthreads();
    {   // write 128 rows x 32 bytes: output row c (= source column), bytes hold source rows (2b, 2b+1)
        const int cc = tid >> 1, half = tid & 1;
        const int sh = 4 * (cc & 1), cb = cc >> 1;
        uint8_t out[16];
#pragma unroll
        for (int b = 0; b < 16; ++b) {
            const int r = 2 * (16 * half + b);
            const int lo = (tile[r][cb] >> sh) & 15, hi = (tile[r + 1][cb] >> sh) & 15;
            out[b] = (uint8_t)(lo | (hi << 4));
        }
        *reinterpret_cast<uint4 *>(B + (int64_t)(c0 + cc) * (R / 2) + r0 / 2 + 16 * half) =
            *reinterpret_cast<const uint4 *>(out);
    }
}

// In-place byte transpose of the scale region of block e: [rows][cols] -> [cols][rows].
__global__ void __launch_bounds__(1024) scale_transpose_kernel(uint8_t *__restrict__ blks, int rows, int cols) {
    extern __shared__ __align__(16) uint8_t s[];
    uint8_t *p = blks + (int64_t)blockIdx.x * BLOCK + O_DS;
    const int n16 = (int)(DS_BYTES / 16);
    for (int i = threadIdx.x; i < n16; i += blockDim.x)
        reinterpret_cast<uint4 *>(s)[i] = reinterpret_cast<const uint4 *>(p)[i];
    __syncthreads();
    // out[c][r] = in[r][c]; 4 output bytes per thread step
    const int total = rows * cols;
    for (int o = 4 * threadIdx.x; o < total; o += 4 * blockDim.x) {
        uint32_t v = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int oo = o + k, c = oo / rows, r = oo - c * rows;
            v |= (uint32_t)s[r * cols + c] << (8 * k);
        }
        *reinterpret_cast<uint32_t *>(p + o) = v;
    }
}

__global__ void block_deq_kernel(const uint8_t *__restrict__ blk, float s2u, float s2d, float *__restrict__ up,
                                 float *__restrict__ down) {
    // up codes: bytes [0, 1376256) with scale bytes at O_US (64 per row); down codes: [O_DW, O_DS)
    const int64_t n_up = (int64_t)INTER * KB_UP, n_dn = (int64_t)LAT * KB_DN;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_up + n_dn;
         i += (int64_t)gridDim.x * blockDim.x) {
        uint8_t v, sb;
        float s2;
        float *o;
        if (i < n_up) {
            const int64_t row = i / KB_UP, b = i - row * KB_UP;
            v = blk[O_UW + i];
            sb = blk[O_US + row * G_UP + b / 8];
            s2 = s2u;
            o = up + 2 * i;
        } else {
            const int64_t k = i - n_up, row = k / KB_DN, b = k - row * KB_DN;
            v = blk[O_DW + k];
            sb = blk[O_DS + row * G_DN + b / 8];
            s2 = s2d;
            o = down + 2 * k;
        }
        const float sc = e4m3_f32(sb);
        o[0] = __fmul_rn(__fmul_rn(e2m1_f32(v), sc), s2);
        o[1] = __fmul_rn(__fmul_rn(e2m1_f32(v >> 4), sc), s2);
    }
}

// deq (qmoe_ns.py:395-404) for any [N, K]: one thread per code byte.
__global__ void deq_kernel(const uint8_t *__restrict__ w, const uint8_t *__restrict__ s, float ws2, int64_t N,
                           int64_t K, float *__restrict__ out) {
    const int64_t KB = K / 2, total = N * KB;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / KB, b = i - row * KB;
        const float sc = e4m3_f32(s[row * (K / 16) + b / 8]);
        const uint32_t v = w[i];
        out[2 * i] = __fmul_rn(__fmul_rn(e2m1_f32(v), sc), ws2);
        out[2 * i + 1] = __fmul_rn(__fmul_rn(e2m1_f32(v >> 4), sc), ws2);
    }
}

static std::atomic<uint64_t> g_st_smem{0};

// Shared body of from_T / to_T. src_R x src_C is the source nibble matrix of each block's code region.
static int convert(uint8_t *blks, int N, uint8_t *scratch, int src_R, int src_C, int srows, int scols,
                   cudaStream_t st) {
    int dev;
    DeviceInfo *di;
    if (int e = current_device(&dev, &di)) return e;
    dim3 grid(src_R / NT_R, src_C / NT_C, N);
    nibble_transpose_kernel<<<grid, NT_THREADS, 0, st>>>(blks, src_R, src_C, scratch);
    if (int e = launch_status()) return e;
    if (!ensure_smem(scale_transpose_kernel, (size_t)DS_BYTES, dev, g_st_smem)) return QMOE_ERR_LAUNCH;
    scale_transpose_kernel<<<N, 1024, (size_t)DS_BYTES, st>>>(blks, srows, scols);
    if (int e = launch_status()) return e;
    if (cudaMemcpy2DAsync(blks + O_DW, (size_t)BLOCK, scratch, (size_t)DW_BYTES, (size_t)DW_BYTES, (size_t)N,
                          cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return QMOE_ERR_LAUNCH;
    return launch_status();
}

} // namespace qmoe

using namespace qmoe;

extern "C" {

int qmoe_from_T(uint8_t *blks, int N, uint8_t *scratch, void *stream) {
    if (!blks || !scratch) return QMOE_ERR_NULL;
    if (N < 0 || N > 65535) return QMOE_ERR_SHAPE;
    if (!aligned16(blks) || !aligned16(scratch)) return QMOE_ERR_ALIGN;
    if (N == 0) return QMOE_OK;
    // T codes: [2688 neuron][1024 row]; T scales: [168][1024] -> [1024][168]
    return convert(blks, N, scratch, INTER, LAT, G_DN, LAT, as_stream(stream));
}

int qmoe_to_T(uint8_t *blks, int N, uint8_t *scratch, void *stream) {
    if (!blks || !scratch) return QMOE_ERR_NULL;
    if (N < 0 || N > 65535) return QMOE_ERR_SHAPE;
    if (!aligned16(blks) || !aligned16(scratch)) return QMOE_ERR_ALIGN;
    if (N == 0) return QMOE_OK;
    // orig codes: [1024 row][2688 neuron]; orig scales: [1024][168] -> [168][1024]
    return convert(blks, N, scratch, LAT, INTER, LAT, G_DN, as_stream(stream));
}

int qmoe_deq(const uint8_t *w, const uint8_t *s, float ws2, int64_t N, int64_t K, float *out, void *stream) {
    if (!w || !s || !out) return QMOE_ERR_NULL;
    if (N < 0 || K < 16 || (K % 16)) return QMOE_ERR_SHAPE;
    if (int e = current_device(nullptr, nullptr)) return e;
    if (N == 0) return QMOE_OK;
    int64_t blocks = (N * (K / 2) + 255) / 256;
    if (blocks > 148 * 64) blocks = 148 * 64;
    deq_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(w, s, ws2, N, K, out);
    return launch_status();
}

int qmoe_block_deq(const uint8_t *blk, float s2_up, float s2_down, float *up, float *down, void *stream) {
    if (!blk || !up || !down) return QMOE_ERR_NULL;
    if (int e = current_device(nullptr, nullptr)) return e;
    block_deq_kernel<<<1184, 256, 0, as_stream(stream)>>>(blk, s2_up, s2_down, up, down);
    return launch_status();
}

} // extern "C"
