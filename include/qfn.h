/*
 * qfn.h -- C ABI of the B200 (sm_100a) quantized matrix-product library.
 *
 * Scope: the quantized matrix products of a Qwen3.8-Flash-Next-style MoE
 * decoder.  Every entry point takes plain device pointers, sizes and a CUDA
 * stream handle; no C++ or torch types cross this boundary.  Every entry
 * point validates its arguments on the host and returns QFN_OK (0) or a
 * positive QFN_ERR_* code; it never traps on the device.  Kernels are queued
 * on `stream` and nothing blocks the host, so every entry point can be
 * recorded into a CUDA graph (no allocation, no host synchronisation).
 *
 * Data formats (the reference's repacked expert block, repack_experts.py:2-3,
 * 12-19 and qmoe.py:9-14):
 *   one expert block = 2,764,800 bytes:
 *     gate_w  u8[640][1280]  @ 0         two e2m1 codes per byte, low nibble = even k
 *     up_w    u8[640][1280]  @ 819200
 *     down_w  u8[2560][320]  @ 1638400
 *     gate_s  e4m3[640][160] @ 2457600   one E4M3 scale per 16 consecutive k
 *     up_s    e4m3[640][160] @ 2560000
 *     down_s  e4m3[2560][40] @ 2662400
 *   per-expert fp32 global scales s2[3] = (ws2_gate, ws2_up, ws2_down).
 *   dequantized weight W[n][k] = E2M1[nibble] * e4m3(scale[n][k/16]) * ws2.
 */
#ifndef QFN_H
#define QFN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* A cudaStream_t passed as an opaque pointer (0 = the legacy default stream). */
typedef void* qfn_stream_t;

/* Status codes. */
enum {
    QFN_OK = 0,
    QFN_ERR_INVALID_ARG = 1,   /* null pointer, bad size, bad dtype code     */
    QFN_ERR_ALIGNMENT = 2,     /* a pointer is not aligned as documented     */
    QFN_ERR_CUDA = 3,          /* a CUDA runtime call failed (see message)   */
    QFN_ERR_UNSUPPORTED = 4,   /* shape outside what the kernels implement   */
    QFN_ERR_WORKSPACE = 5,     /* workspace too small (size query returned)  */
    QFN_ERR_DEVICE = 6         /* device is not sm_100 / no device           */
};

/* Element type codes for `x` / `y` arguments. */
enum { QFN_DTYPE_F32 = 0, QFN_DTYPE_BF16 = 1 };

/* Model constants of the expert block (qmoe.py:9-14). */
#define QFN_HID 2560
#define QFN_INTER 640
#define QFN_BLOCK_BYTES 2764800
#define QFN_O_GW 0
#define QFN_O_UW 819200
#define QFN_O_DW 1638400
#define QFN_O_GS 2457600
#define QFN_O_US 2560000
#define QFN_O_DS 2662400
#define QFN_MAX_TOPK 32

/* Library version (major*10000 + minor*100 + patch). */
int qfn_version(void);

/* Static text for a status code. */
const char* qfn_strerror(int status);

/* Detail of the last failure on the calling host thread ("" if none). */
const char* qfn_last_error(void);

/*
 * qfn_deq -- replaces qmoe.deq (qmoe.py:93-102).
 *   out[n][k] = E2M1[nibble(w[n][k/2], k&1)] * e4m3(s[n][k/16]) * ws2   (fp32)
 *   w: u8[N][K/2], s: u8[N][K/16] (E4M3 bytes), out: f32[N][K], all row-major
 *   and contiguous.  K % 32 == 0.  Bit-exact with the reference.
 */
int qfn_deq(const uint8_t* w, const uint8_t* s, float ws2, float* out,
            int64_t N, int64_t K, qfn_stream_t stream);

/*
 * qfn_block_deq -- replaces qmoe.block_deq (qmoe.py:105-111).
 *   blk: one expert block (QFN_BLOCK_BYTES, 16-byte aligned) in device memory;
 *   s2: host array of 3 floats (ws2 gate, up, down).
 *   gate/up: f32[640][2560], down: f32[2560][640].
 */
int qfn_block_deq(const uint8_t* blk, const float s2[3], float* gate, float* up,
                  float* down, qfn_stream_t stream);

/*
 * qfn_moe_decode -- replaces qmoe.moe_decode (qmoe.py:77-83), the bs=1
 * NVFP4 SwiGLU expert layer fused over K experts plus the weighted combine:
 *   h[j][n]  = silu(ws2_g[j] * Wg_j[n].x) * (ws2_u[j] * Wu_j[n].x)
 *   out[r]   = sum_j coef[j] * ws2_d[j] * Wd_j[r].h[j]
 *   table:  u8[n_blocks][QFN_BLOCK_BYTES] device, 16-byte aligned.  Either
 *           the reference's slot table or the whole HBM-resident expert table.
 *   sidx:   int32[K] device, block index of expert j (0 <= sidx < n_blocks;
 *           an out-of-range index is not read: it yields NaN in `out`).
 *   s2:     f32[K][3] device; coef: f32[K] device.
 *   x:      [2560] device, 16-byte aligned, dtype QFN_DTYPE_BF16 or QFN_DTYPE_F32.
 *   h_buf:  f32[>=K][640] device scratch (the reference's h_buf).  On return
 *           it holds h, as in the reference.
 *   out:    f32[2560] device; written (not accumulated).
 *   1 <= K <= QFN_MAX_TOPK.
 *   K <= 10 on a 148-SM part with a 16-byte aligned out runs the slice path:
 *   one cooperative launch per layer without a grid-wide barrier (every CTA
 *   owns one expert's 32-48 features, computes their h on chip and
 *   multiplies them into the matching column slice of the down rows; the
 *   CTAs' partial outputs meet in out through fp32 atomic adds, so repeated
 *   calls agree to fp32 rounding of the summation order, not bit for bit).
 *   The library keeps a small per-device array of call counters for it
 *   (file-scope device memory, nothing allocated per call).  Otherwise the
 *   two-launch CUDA-core path runs (bit-reproducible).
 */
int qfn_moe_decode(const uint8_t* table, int64_t n_blocks, const int32_t* sidx,
                   const float* s2, const float* coef, const void* x, int x_dtype,
                   float* h_buf, float* out, int K, qfn_stream_t stream);

/*
 * qfn_moe_decode_variant -- qfn_moe_decode with the kernel path chosen by the
 * caller (no counterpart in the reference; for tests and measurements):
 * variant 0 = automatic (as qfn_moe_decode), 2 = CUDA-core path (two
 * launches, any K), 4 = slice path (K <= 10, a 148-SM-class device, out
 * 16-byte aligned).  Variants 1 and 3 named earlier paths that were removed
 * and return QFN_ERR_UNSUPPORTED.
 */
int qfn_moe_decode_variant(const uint8_t* table, int64_t n_blocks, const int32_t* sidx,
                           const float* s2, const float* coef, const void* x, int x_dtype,
                           float* h_buf, float* out, int K, int variant,
                           qfn_stream_t stream);

/*
 * qfn_moe_decode_noalloc -- qfn_moe_decode for callers that cannot allocate
 * device memory when they run a step (memory planned once up front, a
 * foreign-language binding without a device allocator, a loop that forbids
 * allocator calls).  No counterpart in the reference.  It takes no h_buf:
 * the h scratch is a file-scope device array of QFN_MAX_TOPK x 640 floats
 * (80 KB) that every device loading the library holds until exit.  The
 * entry point calls no allocator.  Its first call on a device (and its first
 * call after that device's primary context was reset and created again)
 * resolves the array's device address (cudaGetSymbolAddress): make that
 * first call before any stream capture.  All calls on a device share the
 * array, so calls that overlap on the GPU (different streams, no ordering
 * between them) race.  Calls in one stream are safe: every decode kernel
 * waits for the previous kernel in the stream before it writes h.  h is
 * fully rewritten by every call, so nothing needs clearing.
 * 1 <= K <= QFN_MAX_TOPK, otherwise QFN_ERR_UNSUPPORTED.  Other arguments
 * as for qfn_moe_decode.
 */
int qfn_moe_decode_noalloc(const uint8_t* table, int64_t n_blocks, const int32_t* sidx,
                           const float* s2, const float* coef, const void* x, int x_dtype,
                           float* out, int K, qfn_stream_t stream);

/*
 * qfn_device_status -- read (and with clear != 0, reset) the device status
 * words of the decode, GEMV and FP8 linear kernels of the current device,
 * OR-ed: bit 0 = a bounded wait on a shared-memory barrier ran out (the
 * outputs of that call are invalid).
 * Synchronous (a device-to-host copy).  No counterpart in the reference,
 * whose kernels have no waits.
 */
int qfn_device_status(unsigned int* status, int clear);

/*
 * qfn_moe_route -- replaces the router of QwenEngine.moe
 * (qwen_engine.py:803-806) and the decode-argument gathers that follow it
 * (qwen_engine.py:821-825), with no host synchronisation:
 *   logits[t][e] = bf16(sum_k x[t][k] * w_router[e][k])   (fp32 sums)
 *   probs = softmax(logits[t]) in fp32; ti[t] = the topk experts of highest
 *   probability (equal probabilities: lower id first); tv[t][j] =
 *   bf16(probs[ti[t][j]] / sum_j' probs[ti[t][j']]).
 *   x:        bf16[T][2560] device, 16-byte aligned (raw 16-bit words).
 *   w_router: bf16[n_experts][2560] device, 16-byte aligned.
 *   ti:       int32[T][topk] device (expert ids).   tv: bf16[T][topk] device.
 *   logits:   bf16[T][n_experts] device (output; the select step reads it).
 *   Optional outputs for the decode entry points (null to skip):
 *   sidx = sidx_base + ti (sidx_base = layer * n_experts: rows of the
 *   HBM-resident expert table); coef = tv as fp32; s2_out[t][j][3] =
 *   s2_layer[ti[t][j]][0..2] (s2_layer f32[n_experts][3], required with s2_out).
 *   1 <= T <= 4096, n_experts % 4 == 0 and <= 1024, 1 <= topk <= 32.
 *   Two launches (logits, then selection as a programmatic dependent); the
 *   router weights are read before the dependency wait, so nothing earlier
 *   in the stream may write w_router while it runs.
 */
int qfn_moe_route(const uint16_t* x, const uint16_t* w_router, int64_t T, int n_experts, int topk,
                  int64_t sidx_base, const float* s2_layer, int32_t* ti, uint16_t* tv, int32_t* sidx,
                  float* coef, float* s2_out, uint16_t* logits, qfn_stream_t stream);

/*
 * qfn_shared_expert -- replaces the shared expert of QwenEngine.moe and its
 * combine with the routed experts (qwen_engine.py:817-818, 829-831), bf16
 * weights (the engine's Lin layers outside linear_attn are bf16):
 *   sh  = sigmoid(x . w_sg) * (w_down . (silu(w_gate . x) * (w_up . x)))
 *   out = bf16(y) + sh            (y = the routed experts' fp32 output), or
 *   out = sh                      (y = NULL)
 *   each step rounded to bf16 where the reference's bf16 tensors round it;
 *   dot products accumulate in fp32.
 *   x: bf16[T][2560] device; w_gate, w_up: bf16[inter][2560]; w_down:
 *   bf16[2560][inter]; w_sg: bf16[2560] (the [1, 2560] gate row); all
 *   16-byte aligned.  y: f32[T][2560] device or NULL.
 *   h: bf16[T][inter] device scratch (holds silu(g) * u on return), 16-byte
 *   aligned; gt: bf16[T] device scratch (the gate); out: bf16[T][2560].
 *   inter % 8 == 0, 8 <= inter <= 4096; 1 <= T <= 4096.
 *   Two launches (gate/up, then down as a programmatic dependent); both read
 *   their weight rows before the dependency wait, so nothing earlier in the
 *   stream may write the weights while they run.
 */
int qfn_shared_expert(const uint16_t* x, int64_t T, const uint16_t* w_gate, const uint16_t* w_up,
                      const uint16_t* w_down, const uint16_t* w_sg, int inter, const float* y,
                      uint16_t* h, uint16_t* gt, uint16_t* out, qfn_stream_t stream);

/*
 * The two halves of qfn_shared_expert as separate launches, so that the
 * gate/up half (which does not depend on the routing) can run on another
 * stream while the router and the routed experts run, and the down half can
 * follow the routed experts and fuse the combine with their output y:
 *   qfn_shared_expert_gate_up: h = bf16(silu(w_gate . x)) * (w_up . x) rounded
 *     as above, gt = bf16(sigmoid(bf16(x . w_sg)));
 *   qfn_shared_expert_down: out = bf16(y) + bf16(gt * bf16(w_down . h)), or
 *     the shared term alone when y is NULL.
 * Same arguments, shapes, alignment and limits as qfn_shared_expert.
 * qfn_shared_expert = gate_up then down on one stream.
 */
int qfn_shared_expert_gate_up(const uint16_t* x, int64_t T, const uint16_t* w_gate, const uint16_t* w_up,
                              const uint16_t* w_sg, int inter, uint16_t* h, uint16_t* gt, qfn_stream_t stream);
int qfn_shared_expert_down(const uint16_t* w_down, int inter, int64_t T, const uint16_t* h, const uint16_t* gt,
                           const float* y, uint16_t* out, qfn_stream_t stream);

/*
 * qfn_deltanet_step -- replaces recurrent_gated_delta_rule at T == 1
 * (qwen_engine.py:158-174), the per-token state update of the DeltaNet
 * layers (QwenEngine.deltanet, qwen_engine.py:718-719):
 *   q = l2norm(q) / sqrt(dk), k = l2norm(k)     (l2norm: x * rsqrt(sum x^2 + 1e-6))
 *   S[h] = S[h] * exp(g[h]); delta = (v[h] - S[h]^T k) * beta[h]
 *   S[h] = S[h] + k delta^T;  out[h] = bf16(S[h]^T q)
 *   q, k: bf16[n_key_heads][dk]; value head h uses key head
 *         h / (n_heads / n_key_heads) (the engine's repeat_interleave);
 *   v: bf16[n_heads][dv]; g: f32[n_heads]; beta: bf16[n_heads];
 *   S: f32[n_heads][dk][dv], updated in place; out: bf16[n_heads][dv].
 *   dk in {64, 128, 256}; dv % 32 == 0, dv <= 4096.  One launch (a
 *   programmatic dependent: the state is read before the dependency wait,
 *   so no earlier kernel of the stream may still write S).
 */
int qfn_deltanet_step(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g,
                      const uint16_t* beta, float* S, uint16_t* out, int n_heads, int n_key_heads,
                      int dk, int dv, qfn_stream_t stream);

/*
 * qfn_gemv_e4m3 -- replaces fp8gemv.gemv (fp8gemv.py:20-26).
 *   y[n] = s[n] * sum_k e4m3(q[n][k]) * x[k], fp32 accumulation.
 *   q: u8[N][K] (float8_e4m3fn bytes) device, 16-byte aligned, K % 16 == 0.
 *   s: f32[N] device; x: bf16[K] device (raw 16-bit words).
 *   y: [N] device, y_dtype QFN_DTYPE_BF16 (the reference's output, rounded to
 *      nearest even) or QFN_DTYPE_F32 (the unrounded accumulator * s).
 */
int qfn_gemv_e4m3(const uint8_t* q, const float* s, const uint16_t* x, void* y,
                  int y_dtype, int64_t N, int64_t K, qfn_stream_t stream);

/*
 * qfn_e4m3_rows_to_bf16 -- replaces the weight expression of the engine's FP8
 * linear layer for T > 1 tokens (qwen_engine.py:83):
 *   (q.to(torch.bfloat16) * s).to(torch.bfloat16)
 *   w[n][k] = bf16_rn(fp32(e4m3(q[n][k])) * s[n])   (bit-identical)
 *   q: u8[N][K] (float8_e4m3fn bytes) device, 16-byte aligned, K % 16 == 0.
 *   s: f32[N] device (the [N, 1] row scales).
 *   w: bf16[N][K] device (raw 16-bit words), 16-byte aligned.
 * The caller then runs the bf16 GEMM (F.linear(x, w)) as the reference does.
 */
int qfn_e4m3_rows_to_bf16(const uint8_t* q, const float* s, uint16_t* w, int64_t N, int64_t K,
                          qfn_stream_t stream);

/*
 * qfn_linear_e4m3 -- replaces the engine's FP8 linear layer for T > 1 tokens,
 * Lin.__call__ (qwen_engine.py:79-83): F.linear(x, (q.to(bf16) * s).to(bf16)).
 *   y[t][n] = bf16_rn( sum_k x[t][k] * w[n][k] ),  fp32 accumulation,
 *   w[n][k] = bf16_rn(fp32(e4m3(q[n][k])) * s[n])  (the weights of
 *   qfn_e4m3_rows_to_bf16, formed on chip; never written to memory).
 *   q: u8[N][K] (float8_e4m3fn bytes) device, 16-byte aligned, K % 16 == 0.
 *   s: f32[N] device.  x: bf16[T][K] device, 16-byte aligned.
 *   y: bf16[T][N] device.  T, N, K < 2^30.
 * One launch (a programmatic dependent of the previous kernel in the
 * stream).  Results differ from a library GEMM only by the fp32 summation
 * order (at most one bf16 step).
 */
int qfn_linear_e4m3(const uint8_t* q, const float* s, const uint16_t* x, uint16_t* y, int64_t T,
                    int64_t N, int64_t K, qfn_stream_t stream);

/*
 * qfn_moe_prefill -- the batched-prefill expert loop of QwenEngine.moe
 * (qwen_engine.py:835-852), which the reference runs as a Python loop over
 * experts (block_deq + three fp32 torch GEMMs + index_add_ per expert):
 *   out[t] = sum_k tv[t][k] * down_e(silu(gate_e x[t]) * up_e x[t]),
 *   e = ti[t][k], expert e's block at table[(base + e) * QFN_BLOCK_BYTES].
 *   x:     bf16[T][2560] device, 16-byte aligned.
 *   ti:    [T][topk] device expert ids in [0, n_experts), int64 (torch.topk's
 *          output; ti_is_int64 = 1) or int32.  Pairs with id -1 are skipped
 *          (expert-parallel callers mark the pairs of other ranks' experts so);
 *          pairs with any other id outside the range are skipped and flagged
 *          in qfn_prefill_status (bit 2).
 *   tv:    [T][topk] device routing weights, tv_dtype BF16 or F32.
 *   s2l:   f32[n_experts][3] device (ws2 gate/up/down of the layer's experts).
 *   out:   f32[T][2560] device, 16-byte aligned; written (not accumulated).
 *   workspace: device scratch of qfn_moe_prefill_workspace(T, topk,
 *          n_experts) bytes, 256-byte aligned.
 *   1 <= topk <= QFN_MAX_TOPK, 1 <= n_experts <= 1024, base + n_experts <=
 *   n_blocks.  Eight launches on `stream` (routing sort in three passes,
 *   activation gather, tcgen05 gate/up GEMM, h packing, zeroing of out,
 *   tcgen05 down GEMM).
 *   The combine adds with fp32 atomics, so the summation order over a
 *   token's experts varies between calls (as index_add_ on CUDA).
 */
size_t qfn_moe_prefill_workspace(int64_t T, int topk, int n_experts);
int qfn_moe_prefill(const void* x, int64_t T, const void* ti, int ti_is_int64,
                    const void* tv, int tv_dtype, int topk, const uint8_t* table,
                    int64_t n_blocks, int64_t base, const float* s2l, int n_experts,
                    float* out, void* workspace, size_t workspace_bytes,
                    qfn_stream_t stream);

/*
 * qfn_set_prefill_sm_budget -- for the current device, run the persistent
 * grouped-GEMM kernels of qfn_moe_prefill on at most n_sms CTAs (0 = one per
 * SM, the default), leaving the other SMs to kernels that should run at the
 * same time: an expert-parallel caller overlapping NCCL collectives with the
 * GEMMs of another chunk of tokens.  No counterpart in the reference.
 */
int qfn_set_prefill_sm_budget(int n_sms);

/*
 * qfn_prefill_status -- read (and with clear != 0 reset) the prefill status
 * word of the current device: bit 0 = a bounded wait ran out (outputs of that
 * call invalid), bit 2 = an expert id outside [0, n_experts) was skipped.
 * No counterpart in the reference.
 */
int qfn_prefill_status(unsigned int* status, int clear);

/*
 * qfn_moe_prefill_ep -- the expert-parallel MoE layer (batched prefill or
 * batched decode) over an NCCL communicator, for callers that run NCCL
 * themselves (the torch path is ep.moe_prefill_ep_ag; the reference is
 * single-GPU).  Every rank passes its own T tokens and the same T:
 *   all-gather x and the routing over `comm`, map the ids through
 *   `local_of`, the grouped GEMM of qfn_moe_prefill over all W x T tokens and
 *   this rank's n_local experts, reduce-scatter (sum) of the fp32 partial
 *   sums: out = this rank's tokens' MoE output (as qfn_moe_prefill over all
 *   512 experts would give, up to the order of the fp32 sums).
 *   x: bf16[T][2560] device; ti, tv, topk as qfn_moe_prefill (ids are global
 *   expert ids in [0, n_experts)); table/n_blocks/base/s2l: this rank's
 *   expert table (local expert i = block base + i, ws2 s2l[i]); local_of:
 *   int32[n_experts] device, the local index of each global expert on this
 *   rank or -1; comm: an ncclComm_t of W ranks whose device is the current
 *   one; out: f32[T][2560]; workspace: qfn_moe_prefill_ep_workspace(T, topk,
 *   n_local, W) bytes, 256-byte aligned.  All work, collectives included, is
 *   queued on `stream`; libnccl.so.2 is resolved at run time.
 */
size_t qfn_moe_prefill_ep_workspace(int64_t T, int topk, int n_local, int world);
int qfn_moe_prefill_ep(const void* x, int64_t T, const void* ti, int ti_is_int64,
                       const void* tv, int tv_dtype, int topk, const uint8_t* table,
                       int64_t n_blocks, int64_t base, const float* s2l, int n_local,
                       const int32_t* local_of, int n_experts, void* comm, float* out,
                       void* workspace, size_t workspace_bytes, qfn_stream_t stream);

/*
 * NCCL bootstrap for callers without one: qfn_nccl_unique_id writes the
 * 128-byte ncclUniqueId (one rank creates it and sends it to the others by
 * any means); qfn_nccl_comm_init makes this rank's communicator on the
 * current device; qfn_nccl_comm_destroy releases it.
 */
int qfn_nccl_unique_id(void* id_out);
int qfn_nccl_comm_init(void** comm_out, int world, int rank, const void* id);
int qfn_nccl_comm_destroy(void* comm);

#ifdef __cplusplus
}
#endif

#endif /* QFN_H */
