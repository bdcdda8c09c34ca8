/*
 * TEST INFRASTRUCTURE ONLY — NOT PART OF THE PRODUCT.
 *
 * CPU restatement of the reference engine's NVFP4 routed-expert and FP8/NVFP4 dense arithmetic
 * (helgard-orlm/nemotron-super-8gb: qmoe_ns.py, dense_q.py, nem_super.py). It is the parity checker
 * for the CUDA library and the timed CPU baseline of bench.py; only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg load it. The product library (libqmoe_b200.so) never links it.
 *
 * Every function cites the reference lines it restates. Values follow the reference exactly:
 *   - NVFP4 dequant is (e2m1 * e4m3_scale) * weight_scale_2 in fp32 (qmoe_ns.py:395-404);
 *   - dense NVFP4 dequant is e2m1 * (e4m3_scale * s2) in fp32 (dense_q.py:184-187; the op order differs);
 *   - FP8 dequant is e4m3 * s in fp32 (dense_q.py:182).
 * The checkers then accumulate in fp64 from those exact fp32 weights, as tests/kern_test.py:35-39 does.
 * The *_fp32 functions accumulate in fp32 and stand in for the reference's fp32 CPU expert path
 * (nem_super.py:342-346: block_deq to fp32, F.linear, relu^2, F.linear, x coef).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define LAT 1024
#define INTER 2688
#define BLOCK 3096576
#define O_UW 0
#define O_US 1376256
#define O_DW 1548288
#define O_DS 2924544
#define KB_UP 512  /* LAT/2 bytes per up row   (qmoe_ns.py:12) */
#define G_UP 64    /* LAT/16 groups per up row */
#define KB_DN 1344 /* INTER/2 bytes per down row */
#define G_DN 168   /* INTER/16 groups per down row */

/* qmoe_ns.py:391 — e2m1 code -> value; the low nibble of a byte is the even element (qmoe_ns.py:3). */
static const float E2M1[16] = {0.f, .5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f,
                               -0.f, -.5f, -1.f, -1.5f, -2.f, -3.f, -4.f, -6.f};

void orc_e2m1_table(float *out16) { memcpy(out16, E2M1, sizeof(E2M1)); }

/* torch.float8_e4m3fn decode (the `.view(torch.float8_e4m3fn).float()` of qmoe_ns.py:403 and
 * dense_q.py:182/186): 1 sign, 4 exponent (bias 7), 3 mantissa bits, no infinities, S.1111.111 = NaN. */
float orc_e4m3(uint8_t b) {
    int s = b >> 7, e = (b >> 3) & 15, m = b & 7;
    float v;
    if (e == 15 && m == 7) return NAN;
    if (e == 0)
        v = ldexpf((float)m, -9);
    else
        v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
    return s ? -v : v;
}

void orc_e4m3_table(float *out256) {
    for (int i = 0; i < 256; ++i) out256[i] = orc_e4m3((uint8_t)i);
}

/* qmoe_ns.py:395-404 `deq`: w [N, K/2] u8, s [N, K/16] e4m3 bytes, ws2 -> fp32 [N, K] = (e2m1*s)*ws2.
 * swap != 0 reproduces the reference's negative control SWAP (high nibble taken as the even element). */
void orc_deq(const uint8_t *w, const uint8_t *s, float ws2, int64_t N, int64_t K, int swap, float *out) {
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        const uint8_t *wr = w + n * (K / 2);
        const uint8_t *sr = s + n * (K / 16);
        float *o = out + n * K;
        for (int64_t b = 0; b < K / 2; ++b) {
            float sc = orc_e4m3(sr[(2 * b) / 16]);
            int lo = wr[b] & 15, hi = wr[b] >> 4;
            if (swap) { int t = lo; lo = hi; hi = t; }
            o[2 * b] = (E2M1[lo] * sc) * ws2;
            o[2 * b + 1] = (E2M1[hi] * sc) * ws2;
        }
    }
}

/* qmoe_ns.py:356-364 `to_T` (and repack_T.py:27-35 `to_T_batch`): orig block -> T block.
 *   dnT_w[n, b] = nib(dn_w, row 2b, col n) | nib(dn_w, row 2b+1, col n) << 4
 *   dnT_s[g, r] = dn_s[r, g]; the up half is copied unchanged. */
void orc_to_T(const uint8_t *blk, uint8_t *out) {
    memcpy(out, blk, O_DW);
    const uint8_t *dw = blk + O_DW, *ds = blk + O_DS;
    uint8_t *tw = out + O_DW, *ts = out + O_DS;
    for (int n = 0; n < INTER; ++n) {
        for (int b = 0; b < LAT / 2; ++b) {
            int r0 = 2 * b, r1 = 2 * b + 1;
            int v0 = (dw[r0 * KB_DN + n / 2] >> (4 * (n & 1))) & 15;
            int v1 = (dw[r1 * KB_DN + n / 2] >> (4 * (n & 1))) & 15;
            tw[n * (LAT / 2) + b] = (uint8_t)(v0 | (v1 << 4));
        }
    }
    for (int g = 0; g < G_DN; ++g)
        for (int r = 0; r < LAT; ++r) ts[g * LAT + r] = ds[r * G_DN + g];
}

/* qmoe_ns.py:367-375 `from_T`: T block -> orig block (inverse of orc_to_T). */
void orc_from_T(const uint8_t *blk, uint8_t *out) {
    memcpy(out, blk, O_DW);
    const uint8_t *tw = blk + O_DW, *ts = blk + O_DS;
    uint8_t *dw = out + O_DW, *ds = out + O_DS;
    for (int r = 0; r < LAT; ++r) {
        for (int c = 0; c < KB_DN; ++c) {
            int n0 = 2 * c, n1 = 2 * c + 1;
            int v0 = (tw[n0 * (LAT / 2) + r / 2] >> (4 * (r & 1))) & 15;
            int v1 = (tw[n1 * (LAT / 2) + r / 2] >> (4 * (r & 1))) & 15;
            dw[r * KB_DN + c] = (uint8_t)(v0 | (v1 << 4));
        }
    }
    for (int r = 0; r < LAT; ++r)
        for (int g = 0; g < G_DN; ++g) ds[r * G_DN + g] = ts[g * LAT + r];
}

/* Dequantized down weight D[r, n] of one block in either layout (values of qmoe_ns.py:411). */
static inline float down_w(const uint8_t *blk, int layoutT, float s2d, int r, int n) {
    int v;
    float sc;
    if (layoutT) {
        v = (blk[O_DW + n * (LAT / 2) + r / 2] >> (4 * (r & 1))) & 15;
        sc = orc_e4m3(blk[O_DS + (n / 16) * LAT + r]);
    } else {
        v = (blk[O_DW + r * KB_DN + n / 2] >> (4 * (n & 1))) & 15;
        sc = orc_e4m3(blk[O_DS + r * G_DN + n / 16]);
    }
    return (E2M1[v] * sc) * s2d;
}

/* One expert's up GEMV (qmoe_ns.py:24-44 `_up`, values of qmoe_ns.py:410): u[n] = sum_k U[n,k] x[k]
 * with U the fp32 dequantized up weight, accumulated in fp64. */
static void expert_up64(const uint8_t *blk, float s2u, const float *x, double *u) {
    for (int n = 0; n < INTER; ++n) {
        const uint8_t *wr = blk + O_UW + (int64_t)n * KB_UP;
        const uint8_t *sr = blk + O_US + (int64_t)n * G_UP;
        double acc = 0.0;
        for (int b = 0; b < KB_UP; ++b) {
            float sc = orc_e4m3(sr[b / 8]);
            acc += (double)((E2M1[wr[b] & 15] * sc) * s2u) * (double)x[2 * b];
            acc += (double)((E2M1[wr[b] >> 4] * sc) * s2u) * (double)x[2 * b + 1];
        }
        u[n] = acc;
    }
}

/* One expert's down GEMV over h (qmoe_ns.py:47-67 `_down`): y[r] = sum_n D[r,n] h[n] in fp64. */
static void expert_down64(const uint8_t *blk, int layoutT, float s2d, const double *h, double *y) {
    for (int r = 0; r < LAT; ++r) y[r] = 0.0;
    for (int n = 0; n < INTER; ++n) {
        if (h[n] == 0.0) continue; /* exact: a zero term adds nothing */
        for (int r = 0; r < LAT; ++r) y[r] += (double)down_w(blk, layoutT, s2d, r, n) * h[n];
    }
}

/* Routed-expert forward of one decode token, fp64 (qmoe_ns.py:70-76 `moe_decode`, checked as in
 * tests/kern_test.py:35-39): h_j = relu(U_j x)^2, y = sum_j coef_j D_j h_j, summed in slot order j.
 * blks[j] points at expert j's block (orig layout, or T layout when layoutT != 0). h_out [K,2688]
 * (nullable) receives h; yj_out [K,1024] (nullable) receives coef_j D_j h_j. */
void orc_moe_decode(const uint8_t *const *blks, int layoutT, int K, const float *s2, const float *coef,
                    const float *x, double *h_out, double *yj_out, double *y) {
    double *hh = (double *)malloc(sizeof(double) * (size_t)K * INTER);
    double *yy = (double *)malloc(sizeof(double) * (size_t)K * LAT);
#pragma omp parallel for schedule(dynamic, 1)
    for (int j = 0; j < K; ++j) {
        double *h = hh + (size_t)j * INTER;
        expert_up64(blks[j], s2[2 * j], x, h);
        for (int n = 0; n < INTER; ++n) h[n] = h[n] > 0.0 ? h[n] * h[n] : 0.0;
        double *yj = yy + (size_t)j * LAT;
        expert_down64(blks[j], layoutT, s2[2 * j + 1], h, yj);
        for (int r = 0; r < LAT; ++r) yj[r] *= (double)coef[j];
    }
    for (int r = 0; r < LAT; ++r) y[r] = 0.0;
    for (int j = 0; j < K; ++j)
        for (int r = 0; r < LAT; ++r) y[r] += yy[(size_t)j * LAT + r];
    if (h_out) memcpy(h_out, hh, sizeof(double) * (size_t)K * INTER);
    if (yj_out) memcpy(yj_out, yy, sizeof(double) * (size_t)K * LAT);
    free(hh);
    free(yy);
}

/* qmoe_ns.py:249-251: glive[j,g] = any(h[j,16g:16g+16] > 0); gcnt[j] = sum_g glive; gidx[j] =
 * stable descending sort of glive = live groups ascending, then dead groups ascending. */
void orc_live_groups(const float *h, int K, int32_t *gidx, int32_t *gcnt) {
    for (int j = 0; j < K; ++j) {
        int live[G_DN];
        int c = 0;
        for (int g = 0; g < G_DN; ++g) {
            live[g] = 0;
            for (int i = 0; i < 16; ++i)
                if (h[(size_t)j * INTER + 16 * g + i] > 0.f) live[g] = 1;
            c += live[g];
        }
        gcnt[j] = c;
        int p = 0, q = c;
        for (int g = 0; g < G_DN; ++g) {
            if (live[g])
                gidx[j * G_DN + p++] = g;
            else
                gidx[j * G_DN + q++] = g;
        }
    }
}

/* Prefill pairs (qmoe_ns.py:79-133 `moe_pairs`): pair p = (slot pslot[p], token ptok[p]);
 * out[p] = coef[p] * D h_p with h_p = relu(U X[tok])^2, fp64. blks[s] = block of slot s. */
void orc_pairs(const uint8_t *const *blks, int layoutT, int P, const int32_t *pslot, const int32_t *ptok,
               const float *s2p, const float *coefp, const float *X, double *out) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int p = 0; p < P; ++p) {
        double *h = (double *)malloc(sizeof(double) * INTER);
        const uint8_t *blk = blks[pslot[p]];
        expert_up64(blk, s2p[2 * p], X + (size_t)ptok[p] * LAT, h);
        for (int n = 0; n < INTER; ++n) h[n] = h[n] > 0.0 ? h[n] * h[n] : 0.0;
        expert_down64(blk, layoutT, s2p[2 * p + 1], h, out + (size_t)p * LAT);
        for (int r = 0; r < LAT; ++r) out[(size_t)p * LAT + r] *= (double)coefp[p];
        free(h);
    }
}

/* dense_q.py:179-188 `dequant_rows` + a fp64 matvec: y[m, n] = sum_k W[n,k] x[m,k].
 * fmt 0 = FP8 (W = e4m3(w) * s), fmt 1 = NVFP4 (W = e2m1 * (e4m3(sc) * s)). */
void orc_dense(int fmt, const uint8_t *w, const uint8_t *sc, float s, int64_t N, int64_t K, const float *x,
               int M, double *y) {
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        for (int m = 0; m < M; ++m) {
            double acc = 0.0;
            const float *xm = x + (size_t)m * K;
            if (fmt == 0) {
                const uint8_t *wr = w + n * K;
                for (int64_t k = 0; k < K; ++k) acc += (double)(orc_e4m3(wr[k]) * s) * (double)xm[k];
            } else {
                const uint8_t *wr = w + n * (K / 2);
                const uint8_t *sr = sc + n * (K / 16);
                for (int64_t b = 0; b < K / 2; ++b) {
                    float f = orc_e4m3(sr[(2 * b) / 16]) * s;
                    acc += (double)(E2M1[wr[b] & 15] * f) * (double)xm[2 * b];
                    acc += (double)(E2M1[wr[b] >> 4] * f) * (double)xm[2 * b + 1];
                }
            }
            y[(size_t)m * N + n] = acc;
        }
    }
}

/* fp32 -> bf16 bits, round to nearest even (torch's `.copy_` of fp32 into a bf16 tensor). */
static inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
    uint32_t r = 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)((u + r) >> 16);
}

/* dense_q.py:179-188 `dequant_rows` exactly: rows [r0, r1) -> bf16 bits [r1-r0, K]. */
void orc_dequant_rows_bf16(int fmt, const uint8_t *w, const uint8_t *sc, float s, int64_t K, int64_t r0,
                           int64_t r1, uint16_t *out) {
#pragma omp parallel for schedule(static)
    for (int64_t n = r0; n < r1; ++n) {
        uint16_t *o = out + (n - r0) * K;
        if (fmt == 0) {
            for (int64_t k = 0; k < K; ++k) o[k] = f32_to_bf16(orc_e4m3(w[n * K + k]) * s);
        } else {
            for (int64_t b = 0; b < K / 2; ++b) {
                float f = orc_e4m3(sc[n * (K / 16) + (2 * b) / 16]) * s;
                uint8_t v = w[n * (K / 2) + b];
                o[2 * b] = f32_to_bf16(E2M1[v & 15] * f);
                o[2 * b + 1] = f32_to_bf16(E2M1[v >> 4] * f);
            }
        }
    }
}

/* ---------------------------------------------------------------------------------------------
 * The reference's fp32 CPU expert path, used as the timed CPU baseline (nem_super.py:342-346 and
 * the BASELINE CPU recipe): per routed expert, block_deq to fp32 matrices (qmoe_ns.py:407-412),
 * u = U x (fp32), h = relu(u)^2, d = D h (fp32), y += coef * d. Experts run on `nthreads` threads,
 * each materialising its own fp32 U [2688,1024] and D [1024,2688] as block_deq does; the K results
 * are summed in slot order. blks may be in either layout (the T layout is read in place).
 * --------------------------------------------------------------------------------------------- */
void orc_cpu_layer_fp32(const uint8_t *const *blks, int layoutT, int K, const float *s2, const float *coef,
                        const float *x, int nthreads, float *y) {
    float *yy = (float *)malloc(sizeof(float) * (size_t)K * LAT);
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#endif
#pragma omp parallel
    {
        float *U = (float *)malloc(sizeof(float) * (size_t)INTER * LAT);
        float *D = (float *)malloc(sizeof(float) * (size_t)LAT * INTER);
        float *h = (float *)malloc(sizeof(float) * INTER);
#pragma omp for schedule(dynamic, 1)
        for (int j = 0; j < K; ++j) {
            const uint8_t *blk = blks[j];
            float s2u = s2[2 * j], s2d = s2[2 * j + 1];
            orc_deq(blk + O_UW, blk + O_US, s2u, INTER, LAT, 0, U);
            if (layoutT) {
                for (int r = 0; r < LAT; ++r)
                    for (int n = 0; n < INTER; ++n) D[(size_t)r * INTER + n] = down_w(blk, 1, s2d, r, n);
            } else {
                orc_deq(blk + O_DW, blk + O_DS, s2d, LAT, INTER, 0, D);
            }
            for (int n = 0; n < INTER; ++n) {
                const float *ur = U + (size_t)n * LAT;
                float acc = 0.f;
                for (int k = 0; k < LAT; ++k) acc += ur[k] * x[k];
                acc = acc > 0.f ? acc : 0.f;
                h[n] = acc * acc;
            }
            float *yj = yy + (size_t)j * LAT;
            for (int r = 0; r < LAT; ++r) {
                const float *dr = D + (size_t)r * INTER;
                float acc = 0.f;
                for (int n = 0; n < INTER; ++n) acc += dr[n] * h[n];
                yj[r] = acc * coef[j];
            }
        }
        free(U);
        free(D);
        free(h);
    }
    for (int r = 0; r < LAT; ++r) {
        float acc = 0.f;
        for (int j = 0; j < K; ++j) acc += yy[(size_t)j * LAT + r];
        y[r] = acc;
    }
    free(yy);
}

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
