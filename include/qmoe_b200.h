/*
 * libqmoe_b200 — B200 (sm_100a) kernels for the NVFP4 routed-expert forward and the FP8/NVFP4 dense
 * GEMVs of the Nemotron-3.5-Super engine (helgard-orlm/nemotron-super-8gb), behind a plain C ABI.
 *
 * Conventions shared by every entry point:
 *   - All pointers are device pointers unless stated; sizes are element counts.
 *   - `stream` is a cudaStream_t passed as void* (0 = the legacy default stream).
 *   - Launches are asynchronous on `stream`; nothing synchronises the host.
 *   - The return value is a status (QMOE_OK or one of QMOE_ERR_*) for argument checks and the
 *     launch itself. Kernels that wait on other CTAs bound every wait and record a timeout in the
 *     caller's workspace status word, read with qmoe_workspace_status().
 *   - Nothing allocates device memory. Kernels that need scratch take a caller workspace whose size
 *     comes from the matching *_workspace_bytes() function.
 *   - Expert blocks use the reference's byte format (qmoe_ns.py:9-14, repack.py:3-7):
 *       up_w [2688,512] u8 @0 | up_s [2688,64] e4m3 @1376256 | dn_w [1024,1344] u8 @1548288 |
 *       dn_s [1024,168] e4m3 @2924544, BLOCK = 3096576 bytes; two e2m1 per byte, low nibble = even
 *       element; value = e2m1 * e4m3 * weight_scale_2. The "T" layout (qmoe_ns.py:137-141) keeps the
 *       up half and stores down as dnT_w [2688 neuron, 512] @1548288 (low nibble = even row) and
 *       dnT_s [168 group, 1024 row] @2924544.
 */
#ifndef QMOE_B200_H
#define QMOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QMOE_OK 0
#define QMOE_ERR_SHAPE 1       /* a size or count is out of range */
#define QMOE_ERR_ALIGN 2       /* a pointer or stride breaks the required alignment */
#define QMOE_ERR_LAUNCH 3      /* the CUDA launch failed (cudaGetLastError) */
#define QMOE_ERR_TIMEOUT 4     /* a device-side wait gave up (recorded in the workspace status) */
#define QMOE_ERR_NULL 5        /* a required pointer is NULL */
#define QMOE_ERR_DTYPE 6       /* unknown activation dtype code */
#define QMOE_ERR_DEVICE 7      /* the current device is not an sm_100 part */
#define QMOE_ERR_WORKSPACE 8   /* workspace too small */
#define QMOE_ERR_SCRATCH_LIMIT 9 /* K too large for the static scratch of qmoe_decode_groups_static */

/* activation dtype codes */
#define QMOE_DT_F32 0
#define QMOE_DT_BF16 1
#define QMOE_DT_F16 2
#define QMOE_DT_F32_AS_BF16 3  /* dq_gemv_bf16 only: fp32 values, each rounded to bf16 as it is read */

#define QMOE_LAT 1024
#define QMOE_INTER 2688
#define QMOE_BLOCK 3096576
#define QMOE_UPB 1548288
#define QMOE_MAX_K 65535       /* experts (or pairs) per call; the model routes 22 per token */

/* Library version string and status names. */
const char *qmoe_version(void);
const char *qmoe_status_string(int status);

/* Device status word of a workspace (copies 4 bytes to the host and synchronises `stream`).
 * Returns QMOE_OK or the first device-side error code the kernels recorded; `clear` resets it. */
int qmoe_workspace_status(void *workspace, int clear, void *stream);

/* No counterpart in the reference (its host round trips are torch copies). Copies `bytes` from src to dst with a
 * kernel launched as a programmatic dependent of the preceding kernel on `stream`: for the small per-layer records
 * of a decode step whose inputs come from the host (x, routing) and whose output goes back (y), inside the kernel
 * chain rather than as copy-engine transfers between kernels. Either pointer may be pinned host memory
 * (cudaHostAlloc / torch pin_memory: device-accessible under unified addressing); regions must not overlap.
 * bytes == 0 does nothing. */
int qmoe_copy_async(void *dst, const void *src, size_t bytes, void *stream);

/* ------------------------------------------------------------------ routed experts, decode step */

/* Replaces `_up` (qmoe_ns.py:24-44) as launched by moe_decode / moe_decode_groups
 * (qmoe_ns.py:74, :248): h[j, n] = relu(s2[j,0] * sum_g up_s[n,g] * sum_{16} e2m1(up_w) * x)^2 for the
 * expert in slot sidx[j], j < K. slots: base of the slot array (nslots slots), slot_bytes its row stride
 * (BLOCK or UPB, multiple of 16). x [1024] in x_dtype; s2 [K,2] f32; h [K,2688] f32 out.
 * A slot index outside [0, nslots) reads nothing and yields NaN for that expert. */
int qmoe_decode_up(const uint8_t *slots, int64_t slot_bytes, int64_t nslots, const int32_t *sidx, int K,
                   const float *s2, const void *x, int x_dtype, float *h, void *stream);

/* Replaces the live-group glue of moe_decode_groups (qmoe_ns.py:249-251): glive[j,g] = any(h[j,16g:16g+16] > 0),
 * gcnt[j] = number of live groups, gidx[j] = live groups ascending followed by dead groups ascending
 * (= the stable descending sort of glive). h [K,2688] f32; gidx [K,168] i32; gcnt [K] i32. */
int qmoe_live_groups(const float *h, int K, int32_t *gidx, int32_t *gcnt, void *stream);

/* Replaces `_down_groups` (qmoe_ns.py:209-239) with GROUP_CFG's split (qmoe_ns.py:242):
 * part[s, j, r] = coef[j] * s2[j,1] * sum_{live group g = gidx[j,k], k = s mod KS, k < gcnt[j]}
 *                 dnT_s[g, r] * sum_{n in g, h[j,n] > 0} e2m1(dnT_w[n, r]) * h[j, n].
 * tab [K] i64: device addresses of the T-layout blocks; part [KS, K, 1024] f32 out; 1 <= KS <= 8. */
int qmoe_decode_down_groups(const int64_t *tab, const float *h, const int32_t *gidx, const int32_t *gcnt,
                            const float *s2, const float *coef, int K, int KS, float *part, void *stream);

/* Replaces `moe_decode_groups` (qmoe_ns.py:245-255), the decode-step routed-expert forward over the
 * T layout: up GEMV + ReLU^2 (reads slots_up + sidx[j]*slot_bytes), live-group compaction, and the
 * live-group down GEMV (reads the block at tab[j]), then the fixed-order sum over experts:
 *   y[r] = sum_j coef[j] * s2[j,1] * (D_j h_j)[r].
 * Outputs: h [K,2688] f32, gidx [K,168] i32, gcnt [K] i32 (as the reference leaves them), y [1024] f32;
 * part [K,1024] f32 receives the per-expert outputs coef_j*s2d_j*D_j h_j (the reference's part_buf[0,:K]).
 * Every sum is fp32; results are bit-identical from call to call. For K up to the SM count one kernel per
 * layer (each expert's neurons over a cluster of CTAs that stream their up rows and add their own live
 * neurons' down rows) and a small kernel summing the experts in slot order; above it, the up GEMV and the
 * live-group down GEMV. Both launch as programmatic dependents of the preceding work on `stream`. The
 * workspace (size from qmoe_decode_groups_workspace_bytes, zero-filled once) must not be used by another
 * call running concurrently. y may be pinned host memory (device-accessible under unified addressing): the
 * finish kernel then writes the layer's output straight back to the host. */
size_t qmoe_decode_groups_workspace_bytes(int K);
int qmoe_decode_groups(const uint8_t *slots_up, int64_t slot_bytes, int64_t nslots, const int32_t *sidx,
                       const int64_t *tab,
                       const float *s2, const float *coef, const void *x, int x_dtype, int K, float *h,
                       int32_t *gidx, int32_t *gcnt, float *part, float *y, void *workspace,
                       size_t workspace_bytes, void *stream);

/* No counterpart in the reference. The decode-step layer of qmoe_decode_groups for callers that cannot call
 * cudaMalloc: hosts whose device memory is already committed to their own fixed pool or arena (for
 * example an engine that reserves HBM for the resident expert store and its caches up front), code running
 * while a CUDA graph is captured in a mode where allocation calls are refused, and thin foreign-language
 * hosts that only pass through pointers they were given. It allocates nothing: its scratch is a
 * QMOE_STATIC_SCRATCH_BYTES array of device memory inside the library, which every GPU that loads the
 * library holds until the process exits. Limit: K <= QMOE_STATIC_MAX_K, else QMOE_ERR_SCRATCH_LIMIT before
 * any work. The first call on a device looks up the array's device address (once per device), so make
 * that first call before any stream capture. All calls share the one array: calls that overlap on the GPU
 * (other streams, other host threads) race and corrupt each other's results, so serialise them. The
 * arrival counters that must start at zero are cleared on every call and the live masks are rewritten; the
 * status word is not: it keeps the first device-side error of the calls since it was last cleared (a tab entry
 * that is null or not 16-byte aligned records QMOE_ERR_ALIGN and makes that expert's part row, and so y, NaN)
 * until qmoe_decode_groups_static_status reads and clears it.
 * Arguments and outputs as qmoe_decode_groups, without the workspace. */
#define QMOE_STATIC_SCRATCH_BYTES 32768
#define QMOE_STATIC_MAX_K 96
int qmoe_decode_groups_static(const uint8_t *slots_up, int64_t slot_bytes, int64_t nslots, const int32_t *sidx,
                              const int64_t *tab, const float *s2, const float *coef, const void *x, int x_dtype,
                              int K, float *h, int32_t *gidx, int32_t *gcnt, float *part, float *y, void *stream);

/* No counterpart in the reference. The status word of qmoe_decode_groups_static's static array on the current
 * device: waits for `stream`, returns QMOE_OK or the first error recorded since the last clear, and with
 * clear != 0 resets it. Allocates nothing. */
int qmoe_decode_groups_static_status(int clear, void *stream);

/* Replaces `moe_decode` (qmoe_ns.py:70-76), the orig-layout decode forward (full down, no skip):
 * h [K,2688] f32 out, out [K,1024] f32 out (out[j] = coef[j]*s2[j,1]*D_j h_j), y [1024] = sum_j out[j]
 * in slot order. slots/slot_bytes as in qmoe_decode_up (slot_bytes = BLOCK). */
int qmoe_decode(const uint8_t *slots, int64_t slot_bytes, int64_t nslots, const int32_t *sidx, const float *s2,
                const float *coef, const void *x, int x_dtype, int K, float *h, float *out, float *y, void *stream);

/* ------------------------------------------------------------------ routed experts, prompt path */

/* Replaces `moe_pairs` (qmoe_ns.py:127-133, kernels :79-124): P pairs p = (slot pslot[p], token ptok[p]):
 * h[p] = relu(s2p[p,0] * U_slot X[ptok[p]])^2, out[p] = coefp[p] * s2p[p,1] * D_slot h[p].
 * X [T,1024] in x_dtype (T > max ptok); h [P,2688] f32 out; out [P,1024] f32 out. Orig layout. */
int qmoe_pairs(const uint8_t *slots, int64_t slot_bytes, int64_t nslots, const int32_t *pslot, const int32_t *ptok,
               const float *s2p, const float *coefp, const void *X, int x_dtype, int T, int P, float *h, float *out,
               void *stream);

/* Replaces the prompt path of StreamExperts.forward (nem_super.py:295-348): for T tokens with top-k
 * expert ids ids [T,topk] (values in [0, n_experts)) and routing weights [T,topk] f32,
 *   out[t] = sum_k (in k order) weights[t,k] * s2[e,1] * D_e relu(s2[e,0] * U_e x[t])^2,  e = ids[t,k],
 * the moe_pairs arithmetic (qmoe_ns.py:79-133) and the per-expert fp32 path (nem_super.py:342-346) as
 * one expert-grouped GEMM on the tensor cores: block-scaled NVFP4 tcgen05 MMA on the stored weights with the
 * activations as three NVFP4 residual planes, fp32 accumulation, h kept as f32. With a T-layout store the down
 * halves of the experts the prompt uses are first converted to the orig layout inside the workspace (as the
 * reference's prompt path does with from_T_fast); both layouts give identical results. Expert e's block is at
 * store + e * block_stride (block_stride >= BLOCK, multiple of 16); layout_T selects the T layout of the
 * down half (else the orig layout). s2 [n_experts, 2] f32; x [T,1024] in x_dtype (bf16 is converted
 * exactly); out [T,1024] f32. Id -1 means "no expert" (the pair is skipped; expert-parallel blocks use it for
 * experts on other ranks); any other id outside [0, n_experts) records QMOE_ERR_SHAPE in the workspace status
 * and makes that token's output NaN. 1 <= T <= 65536, 1 <= topk <= 32, 1 <= n_experts <= 1024.
 * The workspace (qmoe_prefill_workspace_bytes(T, topk, n_experts, layout_T) bytes, 256-byte aligned) holds
 * the sorted pairs, their activation planes, the h rows and, for a T-layout store only, room for the converted
 * down halves of the experts the prompt can use (min(n_experts, T*topk) of them, 1.55 MB each); its status
 * word must start at zero. */
size_t qmoe_prefill_workspace_bytes(int T, int topk, int n_experts, int layout_T);
int qmoe_prefill_grouped(const uint8_t *store, int64_t block_stride, int n_experts, int layout_T, const int32_t *ids,
                         const float *weights, const float *s2, const void *x, int x_dtype, int T, int topk, float *out,
                         void *workspace, size_t workspace_bytes, void *stream);

/* No counterpart in the reference. Bound, in SM clock cycles, on each device-side wait of the kernels that wait
 * (the pipeline roles of qmoe_prefill_grouped's tensor-core GEMMs) on the current device, from the next call on;
 * cycles <= 0 restores the default of 4e9 cycles (about 2 s). A wait that runs out records QMOE_ERR_TIMEOUT in the
 * workspace status word and the kernel stops: every copy it started lands and every MMA it issued completes
 * (each waited for with the default bound) before it frees its tensor memory and returns; its outputs are then
 * undefined and the next call runs normally. Meant for failure handling and its tests: a short bound makes
 * ordinary calls time out. */
int qmoe_set_wait_cycles(long long cycles);

/* Replaces, for a decode step (one token), the routing of NemotronHTopkRouter.forward / route_tokens_to_experts
 * (tf:697-720, 748-751; the reference calls it at nem_super.py:366-367) after its fp32 linear, together with the
 * expert-store lookup of the routed layer: from logits [n_experts] f32 (the router's fp32 linear) and the
 * correction bias [n_experts] f32, score = sigmoid(logit), choice = score + bias, the top_k largest choices (ties
 * to the lower id; a NaN choice is never taken), weight = score * scaling (no renormalisation: norm_topk_prob
 * false, one expert group). For each chosen expert r (in order of decreasing choice): ids[r] its id,
 * sidx[r] = slot_base + id its store row, tab[r] = blocks + sidx[r] * block_stride, s2_sel[r] = s2[id] (two
 * f32), coef[r] its weight. The sets of ids and weights are those of the reference; their order is not (the
 * reference's top-k is unsorted). 1 <= top_k <= 32, top_k <= n_experts <= 1024. */
int qmoe_route_decode(const float *logits, const float *bias, int n_experts, int top_k, float scaling, int slot_base,
                      const uint8_t *blocks, int64_t block_stride, const float *s2, int64_t *ids, int32_t *sidx,
                      int64_t *tab, float *s2_sel, float *coef, void *stream);

/* ------------------------------------------------------------------ expert parallelism */

/* No counterpart in the reference (it runs every expert on one GPU). Expert e lives on rank
 * e / (n_experts / world). Dispatch pack of one rank's T tokens for a fixed-size all-to-all: for every
 * destination rank d, the tokens with at least one expert on d, in token order, fill rows 0..send_cnt[d)-1 of
 * block d. send_x [world, T, 1024] (x's dtype); send_meta [world, T, 2*topk] i32: the block-local expert ids
 * (-1 for experts on other ranks and for unused rows) then the routing weights as f32 bits; row_of [world, T]
 * i32: row of token t in block d or -1; send_cnt [world] i32. */
int qmoe_ep_dispatch_pack(const void *x, int x_dtype, const int32_t *ids, const float *weights, int T, int topk,
                          int n_experts, int world, void *send_x, int32_t *send_meta, int32_t *row_of,
                          int32_t *send_cnt, void *stream);

/* No counterpart in the reference. Combine after the return all-to-all: recv_part [world, T, 1024] f32 holds,
 * in block d, rank d's partial outputs for the rows this rank packed for d; out[t] = sum over d in rank
 * order of recv_part[d, row_of[d, t]] (rows with row_of -1 skipped). */
int qmoe_ep_combine(const float *recv_part, const int32_t *row_of, int T, int world, float *out, void *stream);

/* ------------------------------------------------------------------ layouts */

/* Replaces `from_T_fast` (qmoe_ns.py:345-353, kernel `_fromT_w` :327-342): N blocks (stride BLOCK)
 * converted from the T layout to the orig layout in place. scratch >= N * 1376256 bytes. */
int qmoe_from_T(uint8_t *blks, int N, uint8_t *scratch, void *stream);

/* Replaces `to_T_batch` (repack_T.py:27-35; qmoe_ns.py:356-364 per block): orig -> T in place.
 * scratch >= N * 1376256 bytes. */
int qmoe_to_T(uint8_t *blks, int N, uint8_t *scratch, void *stream);

/* Replaces `deq` (qmoe_ns.py:395-404): w [N, K/2] u8 codes, s [N, K/16] e4m3 -> out [N, K] fp32 =
 * (e2m1 * e4m3) * ws2, bit-exact with the reference. K a multiple of 16. */
int qmoe_deq(const uint8_t *w, const uint8_t *s, float ws2, int64_t N, int64_t K, float *out, void *stream);

/* Replaces `block_deq` (qmoe_ns.py:407-412, via deq :395-404): one orig-layout block -> up [2688,1024]
 * and down [1024,2688] fp32 = (e2m1 * e4m3) * s2. Bit-exact with the reference. */
int qmoe_block_deq(const uint8_t *blk, float s2_up, float s2_down, float *up, float *down, void *stream);

/* ------------------------------------------------------------------ dense quantized linears */

/* Replaces `_gemv_fp8` / `_gemv_fp8_m2` (dense_q.py:35-53, :83-103) as dispatched by gemv / gemv_mb
 * (dense_q.py:139-152, :199-212): y[m, n] = s * sum_k e4m3(w[n,k]) * x[m,k]. w [N,K] u8; s [1] f32
 * (device); x [M,K] in x_dtype; y [M,N] f32 out; 1 <= M <= 4; K a multiple of 16. */
int dq_gemv_fp8(const uint8_t *w, const float *s, const void *x, int x_dtype, int M, int N, int K, float *y,
                void *stream);

/* Replaces `_gemv_nvfp4` / `_gemv_nvfp4_m2` (dense_q.py:56-80, :106-136):
 * y[m, n] = s2 * sum_g e4m3(sc[n,g]) * sum_{16} e2m1(w[n,.]) * x[m,.]. w [N,K/2] u8; sc [N,K/16] e4m3;
 * s2 [1] f32 (device); 1 <= M <= 4; K a multiple of 32. */
int dq_gemv_nvfp4(const uint8_t *w, const uint8_t *sc, const float *s2, const void *x, int x_dtype, int M, int N,
                  int K, float *y, void *stream);

/* No counterpart kernel in the reference (its bf16 projections, e.g. fc1_latent_proj / fc2_latent_proj of the MoE
 * block, nem_super.py:376-377, run through torch's F.linear): y [M, N] bf16 = bf16 weights w [N, K] times x [M, K]
 * (bf16, f16 or fp32), the weights widened to fp32 exactly and every product accumulated in fp32, then rounded to
 * bf16 with the same epilogues as dq_gemv_nvfp4_bf16 (0: the result; 1: relu^2; 2: + residual). 1 <= M <= 4,
 * K % 8 == 0, w 16-byte aligned. x_dtype may also be QMOE_DT_F32_AS_BF16: fp32 x rounded to bf16 on load, the
 * same values as a bf16 cast of x before the call (the MoE block's routed output y before fc2_latent_proj). */
int dq_gemv_bf16(const uint16_t *w, const void *x, int x_dtype, int M, int N, int K, int epilogue,
                 const uint16_t *residual, uint16_t *y, void *stream);

/* The same GEMV with a bf16 result that folds in the bf16 operators that follow it in the model's shared expert
 * (tf:722-737: shared_experts(x) = down(relu(up(x))^2), added to the routed output), with torch's roundings:
 * epilogue 0: y = bf16(v) (as dense_q.qlinear returns); 1: y = bf16(relu(bf16(v))^2) (the up projection and its
 * squared ReLU); 2: y = bf16(bf16(v) + residual) (the down projection added to residual [M, N] bf16). v is
 * dq_gemv_nvfp4's fp32 result, so each epilogue equals the unfused torch sequence bit for bit. y [M, N] bf16. */
int dq_gemv_nvfp4_bf16(const uint8_t *w, const uint8_t *sc, const float *s2, const void *x, int x_dtype, int M, int N,
                       int K, int epilogue, const uint16_t *residual, uint16_t *y, void *stream);

/* Replaces `dequant_rows` (dense_q.py:179-188): rows [r0, r1) (r1 <= N) of a quantized weight -> out [r1-r0, K]
 * (FP8: e4m3 * s; NVFP4: e2m1 * (e4m3 * s2), computed in fp32 and rounded to out_dtype, a QMOE_DT_*
 * code), bit-exact with the reference. fmt 0 = FP8, 1 = NVFP4; sc ignored for FP8. */
int dq_dequant_rows(int fmt, const uint8_t *w, const uint8_t *sc, const float *s, int64_t N, int64_t K, int64_t r0,
                    int64_t r1, void *out, int out_dtype, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* QMOE_B200_H */
