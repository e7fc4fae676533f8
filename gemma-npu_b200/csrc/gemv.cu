// Weight-only int8 GEMV for decode and the LM head (sm_100a).
//
// Reference behaviour replaced: cpu_int8_linear (gemma_npu.py:155-156), i.e.
// torch._weight_int8pack_mm(x_bf16 [T,K], w int8 [N,K], s bf16 [N]) -> bf16 [T,N]:
//     y[t,n] = bf16(float(s[n]) * sum_k float(x[t,k]) * float(w[n,k]))
// and, for the LM head, Int8Head.forward (gemma_npu.py:170-172) followed by the final
// logit softcap of the prefill (pipeline.py:335-338): cap * tanh(float(y) / cap).
//
// The kernel is HBM-bound: every weight byte is read once with 16-byte non-allocating
// loads, coalesced across the warp.  The activation row is held in registers as 16-bit
// fixed point, each 16-element piece over its own range, x_q = rint(x * 32766 / max|x|),
// split into a signed high byte and an unsigned low byte (x_q = 256 hi + lo): lane l of
// the warp owning K-slice `sl` multiplies the 16 consecutive k of chunk c,
// k = ((sl*J + c)*32 + l)*16 .. +15, of every weight row it visits.  Every 4 weight bytes
// take two dp4a instructions into exact int32 sums, so the kernel issues about a quarter
// of the instructions of an fp32 dot product and is left bound by HBM; each piece's sum is
// scaled once, y = bf16(s * sum_pieces (256 sum_hi + sum_lo) * max|x_piece| / 32766).  The
// fixed point costs at most max|x_piece| / 65532 per element, far inside the GEMV's
// max-rel 1e-2 bound.  S warps ("a team") split K; the team's partial sums meet in shared
// memory, and lane r of the team's first warp finishes row r (scale, bf16, softcap, store).
// Weight loads of the first row batch are issued before waiting for the previous kernel
// of the stream (programmatic dependent launch): only the activation row depends on it.
#include "common.cuh"
#include "gemv_rows.cuh"

namespace w8 {

template <int J, int S, int R, bool LOGITS>
__global__ void __launch_bounds__(kGemvThreads)
    int8_gemv_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                         const int8_t* __restrict__ w, int64_t ldw, const __nv_bfloat16* __restrict__ s,
                         void* __restrict__ y, int64_t ldy, int t_count, int n, int k, float cap,
                         unsigned long long* __restrict__ best) {
  static_assert(kGemvWarps % S == 0, "S must divide the CTA's warps");
  unsigned long long mine = 0ull;  // best argmax_key this thread wrote (LM head, t_count == 1)
  constexpr int kTeams = kGemvWarps / S;
  __shared__ float red[kTeams][S][R];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int team = warp / S;
  const int sl = warp % S;
  pdl_launch_dependents();

  const int stride = gridDim.x * kTeams * R;
  const int first = (blockIdx.x * kTeams + team) * R;
  // One row per team per step (short matrices): the next step's weights are loaded while
  // this step computes, so a CTA with several steps waits for one DRAM round trip, not
  // one per step.  With R > 1 the doubled registers would cost residency instead.
  constexpr bool kPrefetch = R == 1;
  uint4 wv[R][J], wn[R][J];
  auto load_w = [&](uint4 (&dst)[R][J], int n0) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int c = 0; c < J; ++c) {
        const int k0 = ((sl * J + c) * 32 + lane) * 16;
        const int row = n0 + r;
        dst[r][c] = (row < n && k0 < k) ? ldg_stream(w + static_cast<int64_t>(row) * ldw + k0)
                                        : make_uint4(0u, 0u, 0u, 0u);
      }
  };
  // The weights do not depend on the previous kernel: start streaming them before
  // waiting for it (only the activation row does).  The wait sits in its own basic block
  // (t_count >= 1 on every launch): with the loads and the wait in one block the code
  // generator was free to issue the loads after the wait, and a dependent decode chain
  // of 140 layer GEMVs ran 550 us per token instead of 451 us.
  load_w(wv, first);
  if (t_count > 0) pdl_wait();

  for (int t = 0; t < t_count; ++t) {
    const __nv_bfloat16* xt = x + static_cast<int64_t>(t) * ldx;
    // This lane's 16-element pieces of the row, each as 16-bit fixed point over its own
    // range: no reduction across lanes or warps before the dot products.
    uint32_t xh[J][4], xl[J][4];
    float dq[J];
#pragma unroll
    for (int c = 0; c < J; ++c) {
      const int k0 = ((sl * J + c) * 32 + lane) * 16;
      uint32_t words[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
      if (k0 < k) {
        const uint4* p = reinterpret_cast<const uint4*>(xt + k0);
        const uint4 a = __ldg(p), b = __ldg(p + 1);
        words[0] = a.x, words[1] = a.y, words[2] = a.z, words[3] = a.w;
        words[4] = b.x, words[5] = b.y, words[6] = b.z, words[7] = b.w;
      }
      dq[c] = piece_codes(words, xh[c], xl[c]);
    }

    for (int n0 = first; n0 < n; n0 += stride) {
      bool fetched = false;
      if constexpr (kPrefetch) {
        // wv holds row n0 (loaded by the previous step, or before the wait); fetch the
        // row of the next step (the next activation row starts again at `first`).
        int nx = n0 + stride;
        if (nx >= n && t + 1 < t_count) nx = first;
        if (nx < n) {
          load_w(wn, nx);
          fetched = true;
        }
      } else {
        if (t > 0 || n0 != first) load_w(wv, n0);
      }
      float acc[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        // Each piece's exact int32 sum times its scale, then one fp32 warp reduction.
        float v = 0.f;
#pragma unroll
        for (int c = 0; c < J; ++c) {
          int hi = 0, lo = 0;
          dot16_q(wv[r][c], xh[c], xl[c], hi, lo);
          v = fmaf(static_cast<float>(256 * hi + lo), dq[c], v);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        acc[r] = v;
      }

      // Lane r finishes row n0 + r (scale, bf16 rounding, softcap, store), in parallel.
      if constexpr (S == 1) {
        float v = acc[0];
#pragma unroll
        for (int r = 1; r < R; ++r) v = lane == r ? acc[r] : v;  // every lane holds every sum
        if (lane < R && n0 + lane < n) {
          const float f = write_out<LOGITS>(y, static_cast<int64_t>(t) * ldy + n0 + lane, v, s[n0 + lane], cap);
          if (LOGITS && best != nullptr) mine = max(mine, argmax_key(f, n0 + lane));
        }
      } else {
        if (lane == 0) {
#pragma unroll
          for (int r = 0; r < R; ++r) red[team][sl][r] = acc[r];
        }
        // Team barrier: the S warps of this team only.
        asm volatile("bar.sync %0, %1;" ::"r"(1 + team), "r"(S * 32) : "memory");
        if (sl == 0 && lane < R && n0 + lane < n) {
          float v = red[team][0][lane];
#pragma unroll
          for (int q = 1; q < S; ++q) v += red[team][q][lane];
          const float f = write_out<LOGITS>(y, static_cast<int64_t>(t) * ldy + n0 + lane, v, s[n0 + lane], cap);
          if (LOGITS && best != nullptr) mine = max(mine, argmax_key(f, n0 + lane));
        }
        asm volatile("bar.sync %0, %1;" ::"r"(1 + team), "r"(S * 32) : "memory");
      }
      if constexpr (kPrefetch) {
        if (fetched) {
#pragma unroll
          for (int r = 0; r < R; ++r)
#pragma unroll
            for (int c = 0; c < J; ++c) wv[r][c] = wn[r][c];
        }
      }
    }
  }
  if constexpr (LOGITS) {
    if (best != nullptr) {  // one atomic per warp: the greedy token of the whole head
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mine = max(mine, __shfl_xor_sync(0xffffffffu, mine, o));
      if (lane == 0 && mine != 0ull) atomicMax(best, mine);
    }
  }
}

}  // namespace w8

namespace w8host {

int require_sm100(int* device);

template <int J, int S, int R, bool LOGITS>
static int launch_gemv(const __nv_bfloat16* x, int64_t ldx, const int8_t* w, int64_t ldw,
                       const __nv_bfloat16* s, void* y, int64_t ldy, int t, int n, int k, float cap,
                       cudaStream_t stream, unsigned long long* best) {
  auto kern = w8::int8_gemv_kernel<J, S, R, LOGITS>;
  int sms = 0;
  int st = num_sms(&sms);
  if (st != W8_OK) return st;
  // The (unused) dynamic shared memory caps residency at two CTAs per SM: with three or
  // four, a chain of dependent GEMVs ran slower (qkv 2560 x 1536: 3.07 against 3.74 us;
  // the 140-GEMV decode chain 497 against 524 us).  The LM head, a long stream of its own,
  // takes three (65.8 -> 63.5 us).
  constexpr int smem = LOGITS ? w8::kGemvSmemCapHead : w8::kGemvSmemCap;
  int device = 0;
  W8_CUDA_TRY(cudaGetDevice(&device));
  static bool done[64] = {};
  if (device < 0 || device >= 64) return W8_ERR_UNSUPPORTED;
  if (!done[device]) {
    W8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    done[device] = true;
  }
  int per_sm = 0;
  W8_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, w8::kGemvThreads, smem));
  if (per_sm < 1) per_sm = 1;
  constexpr int rows_per_cta = (w8::kGemvWarps / S) * R;
  const int64_t need = (static_cast<int64_t>(n) + rows_per_cta - 1) / rows_per_cta;
  const int64_t cap_blocks = static_cast<int64_t>(sms) * per_sm;
  const int grid = static_cast<int>(need < cap_blocks ? need : cap_blocks);
  // Programmatic stream serialization: the kernel may start streaming its weights while
  // the previous kernel on the stream drains (it waits before reading x).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(w8::kGemvThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, x, ldx, w, ldw, s, y, ldy, t, n, k, cap, best));
}

template <bool LOGITS>
static int gemv_dispatch(const uint16_t* xh, int64_t ldx, const int8_t* w, int64_t ldw,
                         const uint16_t* sh, void* y, int64_t ldy, int64_t t, int64_t n, int64_t k,
                         float cap, cudaStream_t stream,
                         unsigned long long* best = nullptr) {
  W8_CHECK_ARG(t >= 0 && n >= 0 && k >= 0, "negative size");
  W8_CHECK_ARG(t < (1ll << 31) && n < (1ll << 31) && k < (1ll << 31), "size beyond int32 range");
  if (t == 0 || n == 0) return W8_OK;
  W8_CHECK_ARG(xh != nullptr && w != nullptr && sh != nullptr && y != nullptr, "null pointer");
  W8_CHECK_ARG(k % 16 == 0, "k = %lld must be a multiple of 16", (long long)k);
  W8_CHECK_ARG(k <= 16384, "k = %lld exceeds the GEMV limit of 16384", (long long)k);
  W8_CHECK_ARG(ldw >= k && ldx >= k && ldy >= n, "row pitch too small");
  W8_CHECK_ALIGN(aligned(w, 16) && ldw % 16 == 0, "w must be 16-byte aligned with ldw %% 16 == 0");
  W8_CHECK_ALIGN(aligned(xh, 16) && ldx % 8 == 0, "x must be 16-byte aligned with ldx %% 8 == 0");
  int device = 0;
  const int st = require_sm100(&device);
  if (st != W8_OK) return st;
  if (k == 0) {
    W8_CUDA_TRY(cudaMemset2DAsync(y, ldy * (LOGITS ? 4 : 2), 0, n * (LOGITS ? 4 : 2), t, stream));
    return W8_OK;
  }
  const auto* x = reinterpret_cast<const __nv_bfloat16*>(xh);
  const auto* s = reinterpret_cast<const __nv_bfloat16*>(sh);
  const int ti = static_cast<int>(t), ni = static_cast<int>(n), ki = static_cast<int>(k);
  int sms = 0;
  const int st2 = num_sms(&sms);
  if (st2 != W8_OK) return st2;
  // Smallest (S, J) whose slice covers K: x stays within 64 fp32 registers per lane.
  // R rows per team per step: the smallest R whose CTAs (two per SM; one per SM when K >
  // 1536) cover the matrix in one wave, so that no CTA waits for a second DRAM round trip
  // of weights; a matrix no R covers in one wave (the LM head) takes R = 4 (J <= 3) or 2
  // (J = 4), which keep the most weight bytes in flight per warp that the registers allow.
  // The long-K GEMVs of a decode step (o 1536 x 2048, down 1536 x 6144) take one CTA per
  // SM: they then leave SM slots free, and the next GEMV of the dependent chain starts its
  // weight loads there while they run (140 layer GEMVs: 451 -> 427 us).  One row per team (R = 1)
  // also prefetches a second step's rows (measured in a dependent chain: down 1536 x 6144
  // 5.2 -> 4.2 us and 8960 x 1536 5.5 -> 4.4 us with R = 4 at one or more CTAs per SM,
  // against R = 1 at two).
#define W8_GEMV_R(J, S, R) launch_gemv<J, S, R, LOGITS>(x, ldx, w, ldw, s, y, ldy, ti, ni, ki, cap, stream, best)
#define W8_GEMV(J, S, RMAX)                                                                  \
  {                                                                                          \
    const int64_t teams = ((J) * (S) > 3 ? 1ll : 2ll) * sms * (w8::kGemvWarps / (S));         \
    if (n <= teams * 1) return W8_GEMV_R(J, S, 1);                                           \
    if (n <= teams * 2) return W8_GEMV_R(J, S, 2);                                           \
    if constexpr ((RMAX) == 4) {                                                             \
      if (n <= teams * 4) return W8_GEMV_R(J, S, 4);                                         \
      if (n <= teams * 6) return W8_GEMV_R(J, S, 6);                                         \
    }                                                                                        \
    return W8_GEMV_R(J, S, RMAX);                                                            \
  }
  if (k <= 512) W8_GEMV(1, 1, 4);
  if (k <= 1024) W8_GEMV(2, 1, 4);
  if (k <= 1536) W8_GEMV(3, 1, 4);
  if (k <= 2048) W8_GEMV(4, 1, 2);
  if (k <= 3072) W8_GEMV(3, 2, 4);
  if (k <= 4096) W8_GEMV(4, 2, 2);
  if (k <= 6144) W8_GEMV(3, 4, 4);
  if (k <= 8192) W8_GEMV(4, 4, 2);
  if (k <= 12288) W8_GEMV(3, 8, 4);
  W8_GEMV(4, 8, 2);
#undef W8_GEMV_R
#undef W8_GEMV
}

}  // namespace w8host

extern "C" int w8_int8_linear_bf16(const uint16_t* x, int64_t ldx, const int8_t* w, int64_t ldw,
                                   const uint16_t* s, uint16_t* y, int64_t ldy, int64_t t,
                                   int64_t n, int64_t k, w8_stream_t stream) {
  return w8host::gemv_dispatch<false>(x, ldx, w, ldw, s, y, ldy, t, n, k, 0.f,
                                      reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int w8_lm_head_f32(const uint16_t* x, const int8_t* w, const uint16_t* s, float cap,
                              float* logits, int64_t n, int64_t k, w8_stream_t stream) {
  return w8host::gemv_dispatch<true>(x, k, w, k, s, logits, n, 1, n, k, cap,
                                     reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int w8_lm_head_argmax_f32(const uint16_t* x, const int8_t* w, const uint16_t* s, float cap,
                                     float* logits, int64_t n, int64_t k, uint64_t* best,
                                     w8_stream_t stream) {
  W8_CHECK_ARG(best != nullptr, "null argmax output");
  W8_CHECK_ALIGN(reinterpret_cast<uintptr_t>(best) % 8 == 0, "argmax output must be 8-byte aligned");
  W8_CHECK_ARG(n > 0 && n < (1ll << 32) - 1, "n = %lld out of range for the argmax", (long long)n);
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  W8_CUDA_TRY(cudaMemsetAsync(best, 0, sizeof(uint64_t), st));
  return w8host::gemv_dispatch<true>(x, k, w, k, s, logits, n, 1, n, k, cap, st,
                                     reinterpret_cast<unsigned long long*>(best));
}

