// Shared device helpers of libqmoe_b200: block-format constants, NVFP4 / FP8 decode, activation
// prescaling, and PTX wrappers for mbarriers and bulk (TMA) copies with bounded waits.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/qmoe_b200.h"

namespace qmoe {

// Expert block format (qmoe_ns.py:9-14, repack.py:3-7): up_w [2688,512] | up_s [2688,64] e4m3 |
// dn_w [1024,1344] | dn_s [1024,168] e4m3; T layout (qmoe_ns.py:137-141): dnT_w [2688,512] | dnT_s [168,1024].
constexpr int LAT = 1024;
constexpr int INTER = 2688;
constexpr int64_t BLOCK = 3096576;
constexpr int64_t O_UW = 0, O_US = 1376256, O_DW = 1548288, O_DS = 2924544;
constexpr int64_t UPB = O_DW;
constexpr int KB_UP = LAT / 2, G_UP = LAT / 16;     // 512 bytes, 64 groups per up row
constexpr int KB_DN = INTER / 2, G_DN = INTER / 16; // 1344 bytes, 168 groups per down row
static_assert(O_DS + (int64_t)LAT * G_DN == BLOCK, "block layout");

// Error codes a kernel records in its device status word (first error wins).
constexpr int DEV_ERR_TIMEOUT = QMOE_ERR_TIMEOUT;

// Bound on one spin-wait, in SM clock cycles (~2 s at 1.9 GHz).
constexpr long long WAIT_CYCLES = 4000000000LL;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- decode
// One 32-bit word = 4 bytes = 8 e2m1 codes (low nibble = even element, qmoe_ns.py:3) -> four f16x2
// {element 2k, element 2k+1}, exact (hardware cvt.rn.f16x2.e2m1x2, the instruction the reference's
// _e2m1_hw uses at qmoe_ns.py:17-21).
__device__ __forceinline__ void e2m1x8_f16x2(uint32_t w, uint32_t (&o)[4]) {
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
        : "r"(w));
}

// One e2m1 code (low 4 bits of c) -> fp32, exact, by assembling the fp32 bits: magnitudes 1..6 have
// exponent 127 + (m >> 1) and mantissa (m & 1) / 2, m = 1 is 0.5, m = 0 is (signed) zero. Used by the
// exact dequantizers, which decode one byte at a time.
__device__ __forceinline__ float e2m1_f32(uint32_t c) {
    const uint32_t m = c & 7u, s = (c & 8u) << 28;
    const uint32_t mag = m >= 2u ? ((m << 22) + (126u << 23)) : (m ? 0x3F000000u : 0u);
    return __uint_as_float(mag | s);
}

// Two e4m3 bytes (low byte = first) -> f16x2, exact (every e4m3 value is an f16 value).
__device__ __forceinline__ uint32_t e4m3x2_f16x2(uint16_t v) {
    uint32_t o;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(o) : "h"(v));
    return o;
}

// Four e4m3 bytes -> two f16x2 (bytes 0,1 and bytes 2,3).
__device__ __forceinline__ void e4m3x4_f16x2(uint32_t w, uint32_t &lo, uint32_t &hi) {
    lo = e4m3x2_f16x2(static_cast<uint16_t>(w & 0xFFFFu));
    hi = e4m3x2_f16x2(static_cast<uint16_t>(w >> 16));
}

__device__ __forceinline__ float e4m3_f32(uint8_t b) {
    uint32_t h2 = e4m3x2_f16x2(static_cast<uint16_t>(b));
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xFFFFu)));
}

__device__ __forceinline__ __half2 as_h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }
__device__ __forceinline__ uint32_t h2_as_u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

// c_lo += a.lo * b.lo and c_hi += a.hi * b.hi for two f16x2 words, in fp32 (fma.rn.f32.f16: both f16 operands
// are widened exactly, so the product is exact and the one rounding is the fp32 add).
__device__ __forceinline__ void fma2_f16_f32(uint32_t a, uint32_t b, float &c_lo, float &c_hi) {
    asm("{\n\t.reg .b16 al, ah, bl, bh;\n\t"
        "mov.b32 {al, ah}, %2;\n\t"
        "mov.b32 {bl, bh}, %3;\n\t"
        "fma.rn.f32.f16 %0, al, bl, %0;\n\t"
        "fma.rn.f32.f16 %1, ah, bh, %1;\n\t}"
        : "+f"(c_lo), "+f"(c_hi)
        : "r"(a), "r"(b));
}

// f16x2 -> (lo + hi) in fp32.
__device__ __forceinline__ float h2sum_f32(__half2 a) {
    float2 f = __half22float2(a);
    return f.x + f.y;
}

// ---------------------------------------------------------------- activations
// Activations enter as fp32 / bf16 / fp16 (QMOE_DT_*).
__device__ __forceinline__ float load_act(const void *p, int dt, int64_t i) {
    if (dt == QMOE_DT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
    if (dt == QMOE_DT_F16) return __half2float(reinterpret_cast<const __half *>(p)[i]);
    if (dt == QMOE_DT_F32_AS_BF16)
        return __bfloat162float(__float2bfloat16_rn(reinterpret_cast<const float *>(p)[i]));
    return reinterpret_cast<const float *>(p)[i];
}

// Power-of-two exponent E so that amax * 2^E lies in [2^(top-1), 2^top). Multiplying by 2^E is exact,
// and a bf16 value scaled this way converts to f16 exactly while it stays in f16's normal range.
// E is clamped to [-126, 127] so that 2^E and 2^-E are normal floats (pow2f); a vector whose amax is
// below 2^-110 is zero for every purpose here.
__device__ __forceinline__ int prescale_exp(float amax, int top) {
    if (!(amax > 0.f) || !isfinite(amax)) return 0;
    const int e = (int)((__float_as_uint(amax) >> 23) & 0xFFu) - 126;   // amax = m * 2^e, m in [0.5, 1)
    int E = top - (amax >= 1.17549435e-38f ? e : -125);
    return E < -126 ? -126 : (E > 127 ? 127 : E);
}

// 2^E as a float for -126 <= E <= 127, from its exponent bits (exact; no library call).
__device__ __forceinline__ float pow2f(int E) { return __uint_as_float((uint32_t)(127 + E) << 23); }

// ---------------------------------------------------------------- mbarrier + bulk copy (TMA engine)
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity; false after WAIT_CYCLES.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > WAIT_CYCLES) return false;
    }
    return true;
}

// Programmatic dependent launch controls (no-ops when the launch has no PDL attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// Hint: bring the 128-byte line at p into L2, kept with evict_last priority.
__device__ __forceinline__ void prefetch_l2(const void *p) {
    asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(p));
}

// Record the first device-side error in a status word.
__device__ __forceinline__ void set_error(int *status, int code) {
    if (status) atomicCAS(status, 0, code);
}

// Streaming 16-byte global load that does not allocate in L1.
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

} // namespace qmoe
