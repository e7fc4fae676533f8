/*
 * w8a8_b200.h -- C ABI of the B200 (sm_100a) W8A8 linear hot path.
 *
 * Drop-in boundary for the int8 linear layers of the Gemma E2B NPU pipeline
 * (AyaSakura-comp/gemma-npu).  Every entry point takes plain device pointers,
 * element strides and sizes, is ordered on the given CUDA stream (NULL = the
 * legacy default stream), and returns W8_OK (0) or a W8_ERR_* status.  Nothing
 * here allocates per call, and no torch type crosses the boundary.  On a
 * non-zero status, w8_last_error() holds a one-line description.
 *
 * Device-side waits are bounded: a kernel whose pipeline stalls records
 * W8_ERR_DEVICE_TIMEOUT, which w8_device_status() reports after a sync.
 *
 * Reference interfaces replaced (file:line within the reference project):
 *   w8_mm_i8                npu_kernels.py:59-64 (mm_i8) + :40-56 (matmul_i8_k)
 *   w8_gemm_dequant_bf16    gemma_npu.py:127-150 (NPUGemm.matmul launch + _dequant)
 *   w8_quant_rows_bf16/f32  pipeline.py:49-52 (_quant), gemma_npu.py:37-42 (_quant_rows),
 *                           gemma_npu.py:68-69 (NPUGemm weight quant), :165-166 (Int8Head)
 *   w8_dequant_bf16         pipeline.py:55-57 (_deq), gemma_npu.py:45-47 (_dequant)
 *   w8_int8_linear_bf16     gemma_npu.py:155-156 (cpu_int8_linear = torch._weight_int8pack_mm)
 *   w8_lm_head_f32          gemma_npu.py:170-172 (Int8Head.forward) + pipeline.py:335-338 (softcap)
 *   w8_lm_head_argmax_f32   the same + the greedy token argmax (gemma_npu.py:291)
 *   w8_lm_head_peer_f32     the same split by rows over a node's GPUs, all-gathered over NVLink
 *   w8_lm_head_peer_argmax  its greedy token only (gemma_npu.py:291), keys exchanged over NVLink
 *   w8_gemm_gelu_up_quant   pipeline.py:102-107 (k_gelu) fused onto the gate/up GEMM of
 *                           pipeline.py:233-242 (Prefill.gemm)
 *   w8_rms_quant_bf16       pipeline.py:66-69 (k_in)
 *   w8_post_norm_quant_bf16 pipeline.py:95-99 (k_post_attn), :110-114 (k_post_ff)
 *   w8_attn_out_quant_bf16  pipeline.py:88-92 (k_attn_out)
 *   w8_ple_gate_quant_bf16  pipeline.py:117-121 (k_ple_gate)
 *   w8_ple_out_bf16         pipeline.py:124-127 (k_ple_out) [+ :66-69, the next layer's k_in]
 *   w8_qkv_norm_rope_bf16   pipeline.py:72-86 (k_qkv)
 *   w8_gemm_qkv_norm_rope   pipeline.py:233-242 (the qkv GEMM) + :72-86 (k_qkv) in one kernel
 *   w8_gemm_qkv_norm_rope_tiled  the same, cos / sin in an 8-column tiled layout
 *   w8_attention_prefill_bf16 pipeline.py:139-180 (full_attention / sliding_attention)
 *   w8_attention_prefill_quant the same followed by pipeline.py:88-92 (k_attn_out)
 */
#ifndef W8A8_B200_H
#define W8A8_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t. */
typedef struct CUstream_st* w8_stream_t;

/* Status codes. */
#define W8_OK 0
#define W8_ERR_INVALID_ARG 1    /* bad size, stride, pointer or layout code            */
#define W8_ERR_ALIGNMENT 2      /* pointer or row pitch misses the TMA/vector alignment */
#define W8_ERR_UNSUPPORTED 3    /* no sm_100 device, or a shape outside the kernels' limits */
#define W8_ERR_CUDA 4           /* a CUDA runtime/driver call failed                     */
#define W8_ERR_DEVICE_TIMEOUT 5 /* a bounded device-side wait gave up (reported by w8_device_status) */

/* Layout of the B (weight) operand of the GEMMs. */
#define W8_B_KN 0 /* B is [K, N] row-major: the reference's mm_i8 layout (npu_kernels.py:59-60) */
#define W8_B_NK 1 /* B is [N, K] row-major (K-major): the resident weight layout, shared with the GEMV */

/* ---- diagnostics ------------------------------------------------------- */
const char* w8_status_string(int status);
/* Text of the last host-side error on this thread ("" if none). */
const char* w8_last_error(void);
/* Sticky device-side status (W8_OK or W8_ERR_DEVICE_TIMEOUT) of the current device;
 * synchronises the device first.  clear != 0 resets it to W8_OK. */
int w8_device_status(int clear);
/* ABI version: (major << 16) | minor. */
int w8_abi_version(void);
/* Schedule of the last GEMM launched from the calling thread: *stream_k = 1 when its
 * tiles were split over workers (stream-K), *workers = CTA pairs or CTAs launched,
 * *tile_n = output columns per tile; returns 1 for the CTA-pair kernel, 0 for the
 * single-CTA kernel (0 everywhere before the first launch).  A diagnostic of this
 * library with no reference counterpart (the reference's grid is always (M/512, N/512),
 * npu_kernels.py:63). */
int w8_gemm_last_schedule(int* stream_k, int* workers, int* tile_n);
/* Fault injection for tests of the bounded device-side wait, with no reference
 * counterpart: while drop_signal != 0, the owner of a stream-K tile split between
 * workers stores its partial sum but never signals the other contributors, whose
 * counter wait then gives up after wait_limit_ns (0 = the default 2 s) and records
 * W8_ERR_DEVICE_TIMEOUT for w8_device_status().  The kernel still ends and the context
 * stays usable; the counters of that call are left non-zero (use a fresh workspace
 * afterwards).  Synchronises the current device.  Production code never calls it;
 * w8_inject_stream_k_stall(0, 0) restores normal operation. */
int w8_inject_stream_k_stall(int drop_signal, uint64_t wait_limit_ns);

/* ---- prefill GEMMs (tcgen05 kind::i8, int32 accumulators in TMEM) ----- */

/* C[M,N] (int32) = A[M,K] (int8) @ B (int8), exact int32 accumulation.
 * Replaces mm_i8 (npu_kernels.py:59-64) / matmul_i8_k (npu_kernels.py:40-56).
 * Unlike the reference, M and N need no padding to 512 and K none to 128:
 * K % 16 == 0; lda, ldb multiples of 16 (bytes == elements); a, b 16-byte
 * aligned (TMA).  C may have any row pitch ldc >= N (16-byte vector stores
 * when c is 16-byte aligned and ldc % 4 == 0, element stores otherwise).
 * b_layout is W8_B_KN ([K,N], ldb >= N) or W8_B_NK ([N,K], ldb >= K). */
int w8_mm_i8(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, int b_layout,
             int32_t* c, int64_t ldc, int64_t m, int64_t n, int64_t k, w8_stream_t stream);

/* w8_mm_i8 with a caller-provided workspace, which lets the kernel balance a ragged
 * last wave of tiles (stream-K: tiles split across SMs are summed exactly in int32).
 * Same result bits as w8_mm_i8.  The workspace holds one 32-bit counter per tile:
 * it must be zero-filled before its first use, it is zero again when each call
 * completes, and it must not be shared by calls that may run at the same time.
 * A workspace smaller than w8_mm_i8_workspace_bytes() (or NULL) just disables
 * stream-K.  Replaces the same reference call as w8_mm_i8 (npu_kernels.py:59-64). */
int w8_mm_i8_ws(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, int b_layout,
                int32_t* c, int64_t ldc, int64_t m, int64_t n, int64_t k, void* workspace,
                int64_t workspace_bytes, w8_stream_t stream);
/* Bytes of workspace w8_mm_i8_ws can use for an M x N x K product (4 per tile). */
int64_t w8_mm_i8_workspace_bytes(int64_t m, int64_t n, int64_t k);

/* w8_mm_i8_ws for callers that cannot allocate device memory.  It has no counterpart
 * in the reference.  Some callers may not call cudaMalloc at all on their path: a
 * plugin or operator run inside another framework's execute callback that owns the
 * whole device-memory budget, a serving loop that must not synchronise the device
 * (cudaMalloc and cudaFree can), or code with a fixed memory plan.  They pass only
 * inputs and outputs; the stream-K tile counters live in a 64 KiB static device array
 * inside this library, held by every GPU that loads it until the process exits.
 * Limit: at most 16384 tile counters, i.e. ceil(M/128) * ceil(N/256) <= 16384
 * (for example M = 4096 and N = 131072); larger products are rejected with
 * W8_ERR_INVALID_ARG.  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current), so make that first call before any
 * stream capture.  Each call clears the counters it uses (an asynchronous memset on
 * `stream`, queued after the argument checks pass) and allocates nothing.  All calls share the one array: calls that can
 * overlap on the GPU (other streams, other threads) race and must be serialised by the
 * caller.  Same constraints and result bits as w8_mm_i8. */
int w8_mm_i8_noalloc(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, int b_layout,
                     int32_t* c, int64_t ldc, int64_t m, int64_t n, int64_t k, w8_stream_t stream);

/* Y[M,N] (bf16) = bf16((float(A@B) * sx[m]) * sw[n]) with the dequant fused
 * into the GEMM epilogue.  Bit-identical to mm_i8 followed by _deq.
 * Replaces NPUGemm.matmul's launches + _dequant (gemma_npu.py:127-150).
 * Same constraints as w8_mm_i8 (y any pitch ldy >= N; vector stores when
 * y is 16-byte aligned and ldy % 8 == 0). */
int w8_gemm_dequant_bf16(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, int b_layout,
                         const float* sx, const float* sw, uint16_t* y, int64_t ldy,
                         int64_t m, int64_t n, int64_t k, w8_stream_t stream);

/* The gate/up GEMM with the glue that follows it fused (k_gelu, pipeline.py:102-107):
 *   y   = _deq(A @ W^T, sx, sw)                      [M, 2I], never written
 *   a   = bf16(gelu_tanh(y[:, :I]) * y[:, I:])       [M, I] bf16, written to `y_out`
 *   q,s = _quant(a)                                  int8 [M, I] + fp32 [M]
 * W and sw are the gate/up weight and scales PACKED by 128-row blocks: packed row
 * 256t + j (j < 128) is gate row 128t + j and packed row 256t + 128 + j is up row
 * I + 128t + j, so each 256-column GEMM tile holds matching gate and up columns.
 * inter = I must be a multiple of 128; K % 16 == 0 (K % 128 == 0 for M > 128 to use
 * CTA pairs).  y_out: 16-byte aligned, ldy*2 % 16 == 0.  q: 8-byte aligned, ldq % 8 == 0.
 * row_absmax: M floats that must be zero on entry; they are zero again on return.
 * Two launches on `stream`: the GEMM (epilogue writes a and folds max|a| per row into
 * row_absmax) and the row quant.  No counterpart in the reference beyond the glue it
 * fuses: the reference runs k_gelu on the CPU over the int32 GEMM output. */
int w8_gemm_gelu_up_quant(const int8_t* a, int64_t lda, const int8_t* w, int64_t ldw,
                          const float* sx, const float* sw, int64_t m, int64_t inter, int64_t k,
                          uint16_t* y_out, int64_t ldy, float* row_absmax, int8_t* q, int64_t ldq,
                          float* s, w8_stream_t stream);

/* The qkv GEMM with k_qkv (pipeline.py:72-86) fused into its epilogue, for head_dim 256
 * (Gemma E2B's sliding layers): out = the head-major q [heads, T, 256], k, v [kv_heads, T,
 * 256] (bf16) that w8_gemm_dequant_bf16 followed by w8_qkv_norm_rope_bf16 produce, bit for
 * bit, without the bf16 [T, N] intermediate.  w is the resident [N, K] qkv weight with
 * N = (heads + 2 kv_heads) * 256 (heads * 256 when shared: q only, a KV-shared layer);
 * head h of the output starts at out + h * ld_head, token t at + t * ld_tok.  Each 256-column
 * GEMM tile is one head: the epilogue dequantises it, takes the head's RMSNorm (q_norm /
 * k_norm weight, none for v) and rotates q and k (cos / sin [T, >= 256], pitch ldcs).
 * Replaces Prefill.gemm (pipeline.py:233-242) of the qkv group plus k_qkv. */
int w8_gemm_qkv_norm_rope(const int8_t* a, int64_t lda, const int8_t* w, int64_t ldw, const float* sx,
                          const float* sw, int64_t m, int64_t heads, int64_t kv_heads, int shared,
                          const uint16_t* cos, const uint16_t* sin, int64_t ldcs, const uint16_t* qw,
                          const uint16_t* kw, float eps, uint16_t* out, int64_t ld_head, int64_t ld_tok,
                          int64_t k, w8_stream_t stream);

/* w8_gemm_qkv_norm_rope with cos / sin in an 8-column tiled layout, the same result bits:
 * column d of token t at cos_t[(d / 8) * tile_pitch + t * 8 + d % 8] (tile_pitch >= 8 T,
 * % 8 == 0), i.e. [D / 8][T][8].  The epilogue holds one token per thread, so with [T, D]
 * tables every 16-byte load of a warp touches 32 rows; tiled, the warp's 32 tokens read
 * 512 contiguous bytes.  The tables are per prompt (positions), shared by every layer with
 * the same RoPE, so a caller lays them out once.  Same reference call as
 * w8_gemm_qkv_norm_rope. */
int w8_gemm_qkv_norm_rope_tiled(const int8_t* a, int64_t lda, const int8_t* w, int64_t ldw, const float* sx,
                                const float* sw, int64_t m, int64_t heads, int64_t kv_heads, int shared,
                                const uint16_t* cos_t, const uint16_t* sin_t, int64_t tile_pitch,
                                const uint16_t* qw, const uint16_t* kw, float eps, uint16_t* out,
                                int64_t ld_head, int64_t ld_tok, int64_t k, w8_stream_t stream);

/* ---- the RMSNorm / residual glue around the GEMMs (bf16 rows) ------------
 * One warp per row, the row held in registers: row length n <= 2048, n % 8 == 0, rows
 * and norm weights 16-byte aligned, pitches in elements % 8 == 0, q 8-byte aligned.
 * _rms (pipeline.py:43-46) is fp32 x * pow(mean(x^2) + eps, -0.5) * w with the mean
 * summed in a different order than ATen's, so a bf16 output may differ from the
 * reference by one bf16 step and an int8 code by one. */

/* k_in (pipeline.py:66-69): q, s = _quant(bf16(_rms(h, w))). */
int w8_rms_quant_bf16(const uint16_t* h, int64_t ldh, const uint16_t* w, float eps, int8_t* q,
                      int64_t ldq, float* s, int64_t t, int64_t n, w8_stream_t stream);

/* After the o or down GEMM with the dequant fused (y = w8_gemm_dequant_bf16 output):
 *   h = bf16(res + bf16(_rms(y, w1)))                          written to h
 *   w2 != NULL: q, s = _quant(bf16(_rms(h, w2)))   (k_post_attn, pipeline.py:95-99)
 *   w2 == NULL: q, s = _quant(h)                   (k_post_ff, pipeline.py:110-114)
 * h may alias res (in-place residual update); it must not alias y. */
int w8_post_norm_quant_bf16(const uint16_t* y, int64_t ldy, const uint16_t* res, int64_t ldr,
                            const uint16_t* w1, const uint16_t* w2, float eps, uint16_t* h,
                            int64_t ldh, int8_t* q, int64_t ldq, float* s, int64_t t, int64_t n,
                            w8_stream_t stream);

/* k_ple_gate (pipeline.py:117-121) after the PLE gate GEMM with the dequant fused
 * (y = _deq(acc), bf16 [T, n]) and this layer's per-layer input ple (bf16 [T, n], row pitch
 * ldp): q, s = _quant(bf16(bf16(gelu_tanh(y)) * ple)), q [T, n] int8, s [T] fp32.
 * n % 8 == 0, n <= 2048.  gelu's 1 + tanh comes from exp2 / reciprocal approximations
 * (relative error a few 2^-23): a bf16 value may move by one step, an int8 code by one. */
int w8_ple_gate_quant_bf16(const uint16_t* y, int64_t ldy, const uint16_t* ple, int64_t ldp, int8_t* q,
                           int64_t ldq, float* s, int64_t t, int64_t n, w8_stream_t stream);

/* k_ple_out (pipeline.py:124-127) after the PLE projection GEMM with the dequant fused
 * (y = _deq(acc), bf16 [T, n]): h = bf16(bf16(res + bf16(_rms(y, w_post))) * scalar), scalar
 * the layer's bf16 layer_scalar as a float.  With w_next != NULL the next layer's k_in
 * (pipeline.py:66-69) follows in the same row pass: q, s = _quant(bf16(_rms(h, w_next)));
 * with w_next == NULL, q and s must be NULL.  h may alias res.  Same tolerance as
 * w8_post_norm_quant_bf16. */
int w8_ple_out_bf16(const uint16_t* y, int64_t ldy, const uint16_t* res, int64_t ldr, const uint16_t* w_post,
                    float scalar, const uint16_t* w_next, float eps, uint16_t* h, int64_t ldh, int8_t* q,
                    int64_t ldq, float* s, int64_t t, int64_t n, w8_stream_t stream);

/* k_attn_out (pipeline.py:88-92): the attention output o [H, T, D] (bf16; element
 * (h, t, d) at o[h * ld_head + t * ld_tok + d]) quantised per token over its H * D
 * values (H * D <= 4096): q [T, H * D] int8, s [T] fp32.  Bit-exact (no reduction but the
 * absmax). */
int w8_attn_out_quant_bf16(const uint16_t* o, int64_t ld_head, int64_t ld_tok, int8_t* q,
                           int64_t ldq, float* s, int64_t t, int64_t heads, int64_t head_dim,
                           w8_stream_t stream);

/* k_qkv (pipeline.py:72-86) after the qkv GEMM with the dequant fused: y = _deq(acc) bf16
 * [T, (H + 2 KV) * D] (q heads, k heads, v heads), or [T, H * D] when shared != 0 (a
 * KV-shared layer, whose k and v are the reference's q).  Per (token, head): q heads
 * bf16(_rms(x, qw)) then RoPE with cos/sin bf16 [T, D] (pitch ldcs), k heads the same
 * with kw, v heads bf16(_rms(x, None)).  out[head * ld_head + t * ld_tok + d], head in
 * the order q, k, v: with ld_head = T * D and ld_tok = D, out is [H + 2 KV, T, D] and
 * its q / k / v slices are the reference's transposed [heads, T, D] tensors.
 * head_dim 64, 128, 256 or 512.  Same tolerance as the other norm glue. */
int w8_qkv_norm_rope_bf16(const uint16_t* y, int64_t ldy, const uint16_t* cos, const uint16_t* sin,
                          int64_t ldcs, const uint16_t* qw, const uint16_t* kw, float eps,
                          uint16_t* out, int64_t ld_head, int64_t ld_tok, int64_t t, int64_t heads,
                          int64_t kv_heads, int64_t head_dim, int shared, w8_stream_t stream);

/* Prefill attention of one prompt from position 0 (pipeline.py:139-180: full_attention,
 * and sliding_attention with window > 0): o[h] = softmax(q[h] k[h / G]^T, causal, and
 * key > query - window when window > 0) v[h / G], scale 1.0, G = heads / kv_heads.  bf16
 * q [heads, T, D], k, v [kv_heads, T, D], o [heads, T, D], element (h, t, d) at
 * x[h * x_head + t * x_tok + d] (the k_qkv glue's head-major output); fp32 softmax and
 * accumulation, P rounded to bf16 for the second product.  head_dim 256 or 512; 16-byte
 * aligned with pitches % 8 == 0.  Replaces local_attn.py / the CPU sdpa calls: within
 * max-rel 1e-2 of them.  Runs on tcgen05 (TMEM accumulators, TMA-fed). */
int w8_attention_prefill_bf16(const uint16_t* q, int64_t q_head, int64_t q_tok, const uint16_t* k,
                              int64_t k_head, int64_t k_tok, const uint16_t* v, int64_t v_head,
                              int64_t v_tok, uint16_t* o, int64_t o_head, int64_t o_tok, int64_t t,
                              int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t window,
                              w8_stream_t stream);
/* Attention followed by k_attn_out (pipeline.py:88-92) in one kernel: instead of o, the
 * per-token _quant of its rows, xq [T, heads * head_dim] int8 (pitch ldq) and xs [T] fp32,
 * bit-identical to w8_attention_prefill_bf16 then w8_attn_out_quant_bf16.  Takes head_dim
 * 256, kv_heads 1 and heads a power of two <= 16 (every head of a token in one CTA: the
 * Gemma E2B sliding layers); other shapes return W8_ERR_UNSUPPORTED.  xq 16-byte aligned,
 * ldq % 16 == 0. */
int w8_attention_prefill_quant(const uint16_t* q, int64_t q_head, int64_t q_tok, const uint16_t* k,
                               int64_t k_head, int64_t k_tok, const uint16_t* v, int64_t v_head,
                               int64_t v_tok, int64_t t, int64_t heads, int64_t kv_heads,
                               int64_t head_dim, int64_t window, int8_t* xq, int64_t ldq, float* xs,
                               w8_stream_t stream);
/* The same contract on warp-level mma.sync tiles (no TMA, no TMEM): a second, independent
 * schedule, kept as a cross-check of the tcgen05 one. */
int w8_attention_prefill_mma_bf16(const uint16_t* q, int64_t q_head, int64_t q_tok, const uint16_t* k,
                                  int64_t k_head, int64_t k_tok, const uint16_t* v, int64_t v_head,
                                  int64_t v_tok, uint16_t* o, int64_t o_head, int64_t o_tok, int64_t t,
                                  int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t window,
                                  w8_stream_t stream);

/* ---- quantisation ------------------------------------------------------ */

/* Per-row symmetric int8: s[r] = max(absmax(x[r,:]), 1e-8) / 127 (fp32, IEEE divide),
 * q[r,k] = clamp(round_half_even(x[r,k] / s[r]), -127, 127).
 * Replaces _quant (pipeline.py:49-52) and _quant_rows (gemma_npu.py:37-42); on a
 * weight [N,K] it is the per-output-channel quant of NPUGemm (gemma_npu.py:68-69). */
int w8_quant_rows_bf16(const uint16_t* x, int64_t ldx, int8_t* q, int64_t ldq, float* s,
                       int64_t m, int64_t k, w8_stream_t stream);
int w8_quant_rows_f32(const float* x, int64_t ldx, int8_t* q, int64_t ldq, float* s,
                      int64_t m, int64_t k, w8_stream_t stream);

/* Y[M,N] (bf16) = bf16((float(acc) * sx[m]) * sw[n]).
 * Replaces _deq (pipeline.py:55-57) / _dequant (gemma_npu.py:45-47). */
int w8_dequant_bf16(const int32_t* acc, int64_t ldacc, const float* sx, const float* sw,
                    uint16_t* y, int64_t ldy, int64_t m, int64_t n, w8_stream_t stream);

/* ---- decode: weight-only int8 GEMV / LM head -------------------------- */

/* These kernels start loading w before they wait for the previous kernel on the stream
 * (only x is taken to depend on it).  w must therefore not be written by the kernel
 * just before them on the stream when that kernel is one of this library's GEMM, GEMV,
 * glue or attention kernels, which let their successor start early; w8_quant_rows_*
 * and kernels from outside the library do not. */

/* y[t,n] (bf16) = bf16(float(s[n]) * sum_k float(x[t,k]) * w[n,k]) within max-rel 1e-2:
 * x as 16-bit fixed point over each 16-element piece's range, exact int32 dot products.
 * x bf16 [T,K], w int8 [N,K] row-major, s bf16 [N].  K % 16 == 0, ldw % 16 == 0,
 * ldx % 8 == 0, 16-byte aligned x and w.
 * Replaces cpu_int8_linear (gemma_npu.py:155-156), i.e. torch._weight_int8pack_mm. */
int w8_int8_linear_bf16(const uint16_t* x, int64_t ldx, const int8_t* w, int64_t ldw,
                        const uint16_t* s, uint16_t* y, int64_t ldy, int64_t t, int64_t n,
                        int64_t k, w8_stream_t stream);

/* LM head for one token: logits[n] (fp32) = cap * tanh(float(bf16(y[n])) / cap) with
 * y as w8_int8_linear_bf16 computes it for t = 1 (cap <= 0: logits = float(y)).
 * w is [N,K] with row pitch K; for a column-sharded head pass the shard's rows.
 * Replaces Int8Head.forward (gemma_npu.py:170-172) + final_logit_softcapping
 * (pipeline.py:335-338). */
int w8_lm_head_f32(const uint16_t* x, const int8_t* w, const uint16_t* s, float cap,
                   float* logits, int64_t n, int64_t k, w8_stream_t stream);

/* w8_lm_head_f32 plus the greedy token (gemma_npu.py:291, logits.argmax()): *best gets
 * (key << 32) | (0xFFFFFFFF - row) of the largest logit, key being its fp32 bits made
 * monotone, so the token is 0xFFFFFFFF - (*best & 0xFFFFFFFF) and ties resolve to the
 * lowest row as torch.argmax does.  `best` (8-byte aligned) is cleared on the stream
 * first; each warp folds its rows into it with one 64-bit atomicMax. */
int w8_lm_head_argmax_f32(const uint16_t* x, const int8_t* w, const uint16_t* s, float cap,
                          float* logits, int64_t n, int64_t k, uint64_t* best, w8_stream_t stream);

/* ---- column-sharded LM head with the all-gather over NVLink peer memory ---- */

/* Bytes of the gathered-logits buffer every rank holds for w8_lm_head_peer_f32:
 * the fp32 logits [vocab, padded to 64] plus 256 bytes of flags and keys. */
int64_t w8_lm_head_peer_bytes(int64_t vocab);
/* A zero-filled device buffer other processes of the node can map: *ptr gets it and
 * `handle` (64 bytes, a cudaIpcMemHandle_t) the handle to send to them.  Free with
 * w8_peer_free. */
int w8_peer_alloc(int64_t bytes, void** ptr, void* handle);
/* Map another process's buffer from its 64-byte handle (peer access is enabled as
 * needed); unmap with w8_peer_close. */
int w8_peer_open(const void* handle, void** ptr);
int w8_peer_close(void* ptr);
int w8_peer_free(void* ptr);

/* The LM head of a node's G ranks (one process per GPU), column-sharded, with its
 * all-gather fused in: Int8Head.forward (gemma_npu.py:170-172) + the softcap
 * (pipeline.py:335-338) + the greedy token (gemma_npu.py:291), replacing the GEMV
 * followed by an NCCL all-gather.  Rank `rank` holds rows [row0, row0 + n) of the
 * [vocab, k] int8 head weight (w [n, k], pitch k, bf16 scales s [n]); every rank passes
 * the same G buffers of w8_lm_head_peer_bytes(vocab) bytes (bufs[r] = rank r's buffer:
 * its own from w8_peer_alloc, the others mapped with w8_peer_open), in rank order.  Each
 * logit (bit-identical to w8_lm_head_f32 of the whole head) is stored into every rank's
 * buffer as it is computed; when the call completes on the stream, this rank's buffer
 * holds all vocab logits (fp32, from its start) and *best (if not NULL) the greedy key
 * over all ranks, in w8_lm_head_argmax_f32's format.  Every rank makes the same calls in
 * the same order; a rank writes into a peer only after that peer has started the same
 * call, so each rank must consume one call's logits before it makes the next call on the
 * same stream.  Waits are bounded: a rank that never arrives makes the others return
 * with W8_ERR_DEVICE_TIMEOUT in w8_device_status(), after which the buffers must be
 * reallocated.  At most 8 ranks; k % 16 == 0, k <= 16384. */
int w8_lm_head_peer_f32(const uint16_t* x, const int8_t* w, const uint16_t* s, float cap, int64_t n, int64_t k,
                        int64_t row0, int64_t vocab, int world, int rank, void* const* bufs, uint64_t* best,
                        w8_stream_t stream);

/* The greedy token of the same sharded head without gathering the logits
 * (gemma_npu.py:291, logits.argmax()): each rank's kernel computes its shard's logits into
 * its own buffer only (the other ranks' parts of it are left as they were), and only the
 * 8-byte greedy keys travel, so a decode step pays one flag round trip over NVLink instead
 * of a 1 MB all-gather.  *best gets the winning key as w8_lm_head_argmax_f32 packs it
 * (global row ids).  Calls of either entry point share one sequence of epochs: every rank
 * makes the same calls, of the same kind, in the same order. */
int w8_lm_head_peer_argmax(const uint16_t* x, const int8_t* w, const uint16_t* s, float cap, int64_t n,
                           int64_t k, int64_t row0, int64_t vocab, int world, int rank, void* const* bufs,
                           uint64_t* best, w8_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* W8A8_B200_H */
