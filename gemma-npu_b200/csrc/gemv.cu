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
#include <mutex>

#include "common.cuh"

namespace w8 {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kGemvSmemCap = 96 * 1024;  // dynamic shared memory per CTA: at most 2 CTAs per SM

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Output of one row: bf16 of the scaled sum, optionally softcapped to fp32; returns the
// value written (as fp32).
template <bool LOGITS>
__device__ __forceinline__ float write_out(void* y, int64_t idx, float acc, __nv_bfloat16 s,
                                           float cap) {
  const __nv_bfloat16 v = __float2bfloat16_rn(__fmul_rn(acc, __bfloat162float(s)));
  if constexpr (LOGITS) {
    float f = __bfloat162float(v);
    if (cap > 0.f) f = __fmul_rn(tanhf(__fdiv_rn(f, cap)), cap);
    static_cast<float*>(y)[idx] = f;
    return f;
  } else {
    static_cast<__nv_bfloat16*>(y)[idx] = v;
    return __bfloat162float(v);
  }
}

// Greedy-decode key of a logit: unsigned order = (value, then lower row first), the
// tie rule of torch.argmax.  The fp32 bits are made monotone (negatives inverted).
__device__ __forceinline__ unsigned long long argmax_key(float f, int row) {
  uint32_t u = __float_as_uint(f);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<unsigned long long>(u) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(row));
}

// J: 16-byte chunks per lane per row; S: warps splitting K; R: rows per team per step.
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// (hi, lo) += the 16 signed weight bytes of w times the lane's 16 x codes.
__device__ __forceinline__ void dot16_q(const uint4& w, const uint32_t (&xh)[4], const uint32_t (&xl)[4], int& hi,
                                        int& lo) {
  hi = dp4a_ss(w.x, xh[0], hi);
  lo = dp4a_su(w.x, xl[0], lo);
  hi = dp4a_ss(w.y, xh[1], hi);
  lo = dp4a_su(w.y, xl[1], lo);
  hi = dp4a_ss(w.z, xh[2], hi);
  lo = dp4a_su(w.z, xl[2], lo);
  hi = dp4a_ss(w.w, xh[3], hi);
  lo = dp4a_su(w.w, xl[3], lo);
}

// One 16-element piece of the activation row (8 words of bf16 pairs) as 16-bit fixed
// point over its own range: fma(x, qs, 1.5 * 2^23) rounds x * qs to the nearest integer
// (one rounding), whose two's complement low 16 bits are the float's low 16 bits; byte
// permutes gather the low bytes (unsigned lo) and the high bytes (signed hi) of four codes
// per word.  Returns the piece's scale max|x| / 32766.
__device__ __forceinline__ float piece_codes(const uint32_t (&words)[8], uint32_t (&xh)[4], uint32_t (&xl)[4]) {
  constexpr float kMagic = 12582912.f;
  __nv_bfloat162 m2 = __habs2(*reinterpret_cast<const __nv_bfloat162*>(&words[0]));
#pragma unroll
  for (int i = 1; i < 8; ++i) m2 = __hmax2(m2, __habs2(*reinterpret_cast<const __nv_bfloat162*>(&words[i])));
  const float am = fmaxf(__low2float(m2), __high2float(m2));
  // 32766 (not 32767) keeps every code inside int16 under the approximate division.
  const float qs = am > 0.f ? __fdividef(32766.f, am) : 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t w0 = words[2 * q], w1 = words[2 * q + 1];
    const uint32_t u0 = __float_as_uint(fmaf(__uint_as_float(w0 << 16), qs, kMagic));
    const uint32_t u1 = __float_as_uint(fmaf(__uint_as_float(w0 & 0xFFFF0000u), qs, kMagic));
    const uint32_t u2 = __float_as_uint(fmaf(__uint_as_float(w1 << 16), qs, kMagic));
    const uint32_t u3 = __float_as_uint(fmaf(__uint_as_float(w1 & 0xFFFF0000u), qs, kMagic));
    xl[q] = __byte_perm(__byte_perm(u0, u1, 0x0040), __byte_perm(u2, u3, 0x0040), 0x5410);
    xh[q] = __byte_perm(__byte_perm(u0, u1, 0x0051), __byte_perm(u2, u3, 0x0051), 0x5410);
  }
  return am * (1.f / 32766.f);
}

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
  // waiting for it (only the activation row does).
  load_w(wv, first);
  pdl_wait();

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

// =====================================================================================
// Decode GEMV chain: a whole decode step's GEMVs in one persistent launch.
//
// A chain of dependent GEMVs (step i + 1 may read step i's output as its activation row)
// is bound, one kernel per GEMV, by each kernel's start-up and drain plus one DRAM round
// trip: 3-19 MB GEMVs ran at 0.2-0.5 of the HBM bandwidth.  Here one CTA per SM runs the
// whole chain.  Its producer warp streams the CTA's share of every step's weight rows --
// which depend on nothing -- through a deep shared-memory ring with 1-D bulk copies,
// running ahead across step boundaries; only the activation row of a step waits, on a
// grid-wide counter that every CTA bumps when its rows of the previous step are stored.
// So the weights keep streaming while the consumers wait for the dependence.
//
// Per step, CTA b owns the contiguous weight rows [n b / G, n (b + 1) / G) (G CTAs): a
// contiguous byte range of the [N, K] row-major weight, copied in chunks of whole rows.
// Each consumer warp finishes whole rows with the arithmetic of int8_gemv_kernel at the
// same (J, S) K-split -- the same pieces, the same dp4a sums and the same fp32 order --
// so every output is bit-identical to the standalone GEMV of that step.
//
// All CTAs are co-resident (cooperative launch, one CTA per SM), every wait is bounded,
// and a CTA that gives up raises a grid-wide abort word so the others stop too; the last
// CTA to leave resets the counters, so the workspace is all-zero after every launch.
// =====================================================================================
constexpr int kChainMaxSteps = 192;
constexpr int kChainConsumerWarps = 8;
constexpr int kChainThreads = 32 * (1 + kChainConsumerWarps);
constexpr int kChainStageBytes = 24 * 1024;
constexpr int kChainStages = 9;
constexpr int kChainMaxK = 12288;
constexpr int kChainRingOff = 0;
constexpr int kChainRedOff = kChainStages * kChainStageBytes;
constexpr int kChainBarOff = kChainRedOff + kChainConsumerWarps * 4;
constexpr int kChainSmem = kChainBarOff + 2 * kChainStages * 8 + 16;
static_assert(kChainSmem <= 232448, "decode chain shared memory exceeds one CTA's budget");
static_assert(kChainStageBytes >= 2 * kChainMaxK, "a stage must hold at least two rows");

__device__ int g_chain_status = 0;  // sticky device status of the chain kernel

struct ChainStep {
  const __nv_bfloat16* x;
  const int8_t* w;
  const __nv_bfloat16* s;
  void* y;
  unsigned long long* best;  // greedy key of a logits step (zeroed by the host), or null
  int n, k;
  float cap;
  int logits;  // 0: bf16 y [n]; 1: fp32 logits [n] with the softcap (cap > 0)
  int J, S;    // the standalone kernel's K split for this K
};

struct ChainParams {
  int count;
  int independent;  // 1: no step reads an earlier step's output, so no step waits for the one before
  uint32_t* ctr;    // workspace: ctr[i] steps done per CTA; ctr[count] CTAs gone; ctr[count + 1] abort
  ChainStep step[kChainMaxSteps];
};

// This CTA's share of a step's activation row, pulled into L2 ahead of its use: the row
// is read by every CTA right after the step's dependence resolves, and an L2 hit there
// keeps that read out of the HBM queue the weight stream fills.  A row that the previous
// step is still writing may be fetched stale: the writes then update the L2 lines.
__device__ __forceinline__ void chain_prefetch_x(const ChainStep& st, int b, int G) {
  const int lines = (st.k * 2 + 127) / 128;
  for (int l = b; l < lines; l += G) prefetch_l2(reinterpret_cast<const uint8_t*>(st.x) + l * 128);
}

// Barrier of the consumer warps that also ORs a flag over them: every consumer learns
// whether any of them gave up, so they all leave the step loop together (a warp that
// left alone would leave the others waiting at the next barrier for good).
__device__ __forceinline__ bool chain_consumer_sync_or(bool flag) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, 1, %2, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(flag ? 1u : 0u), "n"(kChainConsumerWarps * 32)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until every CTA has finished step `i` (its counter reaches `target`);
// false if the grid's abort word is raised or the wait times out (then it raises it).
__device__ __forceinline__ bool chain_wait_step(const uint32_t* ctr, uint32_t target, uint32_t* abort_word) {
  const unsigned long long t0 = globaltimer();
#pragma unroll 1
  for (uint32_t spin = 0;; ++spin) {
    if (ld_acquire_gpu(ctr) >= target) return true;
    if (ld_volatile_u32(abort_word) != 0u) return false;
    if (spin > 4096) __nanosleep(64);  // a long wait: back off
    if (globaltimer() - t0 > kWaitTimeoutNs) {
      atomicExch(&g_chain_status, W8_ERR_DEVICE_TIMEOUT);
      atomicExch(abort_word, 1u);
      return false;
    }
  }
}

__global__ void __launch_bounds__(kChainThreads, 1) gemv_chain_kernel(const __grid_constant__ ChainParams p) {
  extern __shared__ __align__(16) uint8_t chain_smem[];
  const uint32_t base = smem_u32(chain_smem);
  const uint32_t bar0 = base + kChainBarOff;
  auto full_bar = [&](int st) { return bar0 + 8u * st; };
  auto empty_bar = [&](int st) { return bar0 + 8u * (kChainStages + st); };
  volatile int* abort_smem = reinterpret_cast<volatile int*>(chain_smem + kChainBarOff + 2 * kChainStages * 8);
  uint32_t* const abort_word = p.ctr + p.count + 1;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int b = blockIdx.x;

  if (threadIdx.x == 0) {
    for (int st = 0; st < kChainStages; ++st) {
      mbar_init(full_bar(st), 1);
      mbar_init(empty_bar(st), kChainConsumerWarps);
    }
    *abort_smem = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer: this CTA's weight rows of every step, in order
      int stage = 0;
      uint32_t phase = 0, issued = 0, last_phase = 0;
      bool ok = true;
      const uint64_t evict_first = l2_policy_evict_first();  // weights are read once
      for (int i = 0; ok && i < p.count; ++i) {
        const ChainStep st = p.step[i];
        const int r0 = static_cast<int>(static_cast<int64_t>(st.n) * b / G);
        const int r1 = static_cast<int>(static_cast<int64_t>(st.n) * (b + 1) / G);
        const int rpc = kChainStageBytes / st.k;  // whole rows per chunk
        for (int c0 = r0; c0 < r1; c0 += rpc) {
          const int c1 = min(c0 + rpc, r1);
          if (!mbar_wait_bounded(empty_bar(stage), phase ^ 1u, abort_smem, &g_chain_status)) {
            ok = false;
            break;
          }
          const uint32_t bytes = static_cast<uint32_t>(c1 - c0) * static_cast<uint32_t>(st.k);
          mbar_arrive_expect_tx(full_bar(stage), bytes);
          bulk_load_1d_hint(base + kChainRingOff + stage * kChainStageBytes, st.w + static_cast<int64_t>(c0) * st.k,
                            bytes, full_bar(stage), evict_first);
          issued |= 1u << stage;
          last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == kChainStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        atomicExch(abort_word, 1u);
        *abort_smem = 1;
      }
      // Copies still in flight land before the CTA may exit (consumed ones already have).
      for (int st = 0; st < kChainStages; ++st)
        if (issued & (1u << st)) mbar_wait_bounded(full_bar(st), (last_phase >> st) & 1u, nullptr, &g_chain_status);
    }
  } else {
    // ---------------- consumers: 8 warps in teams of S (the step's K split), as in
    // int8_gemv_kernel: warp sl of a team owns K-slice sl, its lanes hold their pieces of
    // the activation row as fixed point in registers, and team t finishes rows t,
    // t + teams, ... of every chunk.
    const int cw = warp - 1;
    const int ctid = threadIdx.x - 32;
    float* red = reinterpret_cast<float*>(chain_smem + kChainRedOff);  // [8] team partial sums
    int stage = 0;
    uint32_t phase = 0;
    if (ctid == 0) chain_prefetch_x(p.step[0], b, G);
    for (int i = 0; i < p.count; ++i) {
      // The step's fields in registers: read through a reference into the kernel's
      // parameters, each use in the row loop would be a load of its own.
      const ChainStep st = p.step[i];
      const int k = st.k, J = st.J, S = st.S;
      const int teams = kChainConsumerWarps / S, team = cw / S, sl = cw % S;
      if (ctid == 0 && i + 1 < p.count) chain_prefetch_x(p.step[i + 1], b, G);
      if (i > 0 && !p.independent) {
        const bool gave_up = ctid == 0 && !chain_wait_step(p.ctr + (i - 1), static_cast<uint32_t>(G), abort_word);
        if (chain_consumer_sync_or(gave_up)) {
          if (ctid == 0) *abort_smem = 1;  // the producer stops too
          break;
        }
      }
      // This lane's J pieces of the activation row.  x may be the previous step's output,
      // written by other SMs: read it from L2 (ld.global.cg).
      uint32_t xh[4][4], xl[4][4];
      float dq[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t words[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
        const int k0 = ((sl * J + c) * 32 + lane) * 16;
        if (c < J && k0 < k) {
          const uint4* src = reinterpret_cast<const uint4*>(st.x + k0);
          const uint4 a = __ldcg(src), e = __ldcg(src + 1);
          words[0] = a.x, words[1] = a.y, words[2] = a.z, words[3] = a.w;
          words[4] = e.x, words[5] = e.y, words[6] = e.z, words[7] = e.w;
        }
        dq[c] = piece_codes(words, xh[c], xl[c]);
      }

      const int r0 = static_cast<int>(static_cast<int64_t>(st.n) * b / G);
      const int r1 = static_cast<int>(static_cast<int64_t>(st.n) * (b + 1) / G);
      const int rpc = kChainStageBytes / k;
      unsigned long long mine = 0ull;
      // A warp whose wait gave up keeps walking the chunks (and every team barrier) without
      // touching their data, so the barriers stay matched; the step's closing barrier then
      // tells every consumer.
      bool failed = false;
      for (int c0 = r0; c0 < r1; c0 += rpc) {
        const int c1 = min(c0 + rpc, r1);
        // Every lane waits on the stage's barrier itself: each reader of the copied rows
        // observes their completion.
        const bool got = !failed && mbar_wait_bounded(full_bar(stage), phase, abort_smem, &g_chain_status);
        if (!__all_sync(0xffffffffu, got)) failed = true;
        const uint8_t* ring = chain_smem + kChainRingOff + stage * kChainStageBytes;
        // The channel scales of this team's rows in the chunk, fetched up front (lane j holds
        // the scale of the team's j-th row of each group of 32): a load per row at its store
        // would hold the whole warp for a memory round trip on every row.
        uint32_t s_mine = 0u;
        for (int r = team, j = 0; r < c1 - c0; r += teams, ++j) {
          if ((j & 31) == 0) {
            const int rr = r + lane * teams;
            s_mine = (!failed && rr < c1 - c0) ? static_cast<uint32_t>(__ldg(
                                                    reinterpret_cast<const unsigned short*>(st.s) + c0 + rr))
                                               : 0u;
          }
          const uint32_t s_bits = __shfl_sync(0xffffffffu, s_mine, j & 31);
          const uint8_t* wrow = ring + static_cast<int64_t>(r) * k;
          float v = 0.f;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            if (c >= J || failed) break;
            const int k0 = ((sl * J + c) * 32 + lane) * 16;
            int hi = 0, lo = 0;
            if (k0 < k) dot16_q(*reinterpret_cast<const uint4*>(wrow + k0), xh[c], xl[c], hi, lo);
            v = fmaf(static_cast<float>(256 * hi + lo), dq[c], v);
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          const int row = c0 + r;
          float total = v;
          if (S > 1) {  // the team's K-slices meet in shared memory, in slice order
            if (lane == 0) red[cw] = v;
            asm volatile("bar.sync %0, %1;" ::"r"(2 + team), "r"(S * 32) : "memory");
            if (sl == 0 && lane == 0) {
              total = red[team * S];
              for (int q = 1; q < S; ++q) total += red[team * S + q];
            }
            asm volatile("bar.sync %0, %1;" ::"r"(2 + team), "r"(S * 32) : "memory");
          }
          if (sl == 0 && lane == 0 && !failed) {
            const __nv_bfloat16 sc = __ushort_as_bfloat16(static_cast<unsigned short>(s_bits));
            if (st.logits) {
              const float f = write_out<true>(st.y, row, total, sc, st.cap);
              if (st.best != nullptr) mine = max(mine, argmax_key(f, row));
            } else {
              write_out<false>(st.y, row, total, sc, 0.f);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar(stage));
        if (++stage == kChainStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (lane == 0 && !failed && st.logits && st.best != nullptr && mine != 0ull) atomicMax(st.best, mine);
      // Every consumer warp's outputs of this step are stored; one release publishes them.
      if (chain_consumer_sync_or(failed)) {
        if (ctid == 0) {
          *abort_smem = 1;
          atomicExch(abort_word, 1u);
        }
        break;
      }
      if (ctid == 0 && !p.independent)
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.ctr + i) : "memory");
    }
  }

  __syncthreads();
  if (threadIdx.x == 0) {
    // The last CTA to leave resets every counter (and the abort word) for the next launch;
    // no CTA reads a counter after it has arrived here.
    __threadfence();
    if (atomicAdd(p.ctr + p.count, 1u) == static_cast<uint32_t>(G) - 1u) {
      for (int i = 0; i < p.count + 2; ++i) atomicExch(p.ctr + i, 0u);
      __threadfence();
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
  // four, a chain of dependent GEMVs ran slower (qkv 2560 x 1536: 3.07 against 3.74 us).
  int device = 0;
  W8_CUDA_TRY(cudaGetDevice(&device));
  static bool done[64] = {};
  if (device < 0 || device >= 64) return W8_ERR_UNSUPPORTED;
  if (!done[device]) {
    W8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, w8::kGemvSmemCap));
    done[device] = true;
  }
  int per_sm = 0;
  W8_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, w8::kGemvThreads, w8::kGemvSmemCap));
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
  cfg.dynamicSmemBytes = w8::kGemvSmemCap;
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
  // R rows per team per step: the large R keeps more weight bytes in flight per warp;
  // a matrix too short to give one CTA per SM at that R takes one row per team (measured
  // in a dependent chain: down 1536 x 6144 5.2 -> 4.2 us and 8960 x 1536 5.5 -> 4.4 us with
  // R = 4 at one or more CTAs per SM, against R = 1 at two).
#define W8_GEMV(J, S, R)                                                                      \
  return n < sms * (w8::kGemvWarps / (S)) * (R)                                                \
             ? launch_gemv<J, S, 1, LOGITS>(x, ldx, w, ldw, s, y, ldy, ti, ni, ki, cap, stream, best) \
             : launch_gemv<J, S, R, LOGITS>(x, ldx, w, ldw, s, y, ldy, ti, ni, ki, cap, stream, best)
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

// ---------------------------------------------------------------- decode GEMV chain (host)
namespace w8host {

// The standalone kernel's (J, S) K split for a given K (gemv_dispatch's table).
static void gemv_split(int k, int* J, int* S) {
  static const int kTable[][3] = {{512, 1, 1},  {1024, 2, 1}, {1536, 3, 1}, {2048, 4, 1},  {3072, 3, 2},
                                  {4096, 4, 2}, {6144, 3, 4}, {8192, 4, 4}, {12288, 3, 8}, {16384, 4, 8}};
  for (const auto& e : kTable)
    if (k <= e[0]) {
      *J = e[1];
      *S = e[2];
      return;
    }
  *J = 4;
  *S = 8;
}

static int chain_params(const w8_gemv_step* steps, int count, w8::ChainParams* p) {
  W8_CHECK_ARG(count >= 0 && count <= w8::kChainMaxSteps, "chain of %d steps (1..%d supported)", count,
               w8::kChainMaxSteps);
  W8_CHECK_ARG(count == 0 || steps != nullptr, "null step table");
  p->count = count;
  for (int i = 0; i < count; ++i) {
    const w8_gemv_step& s = steps[i];
    W8_CHECK_ARG(s.n > 0 && s.n < (1ll << 31), "step %d: n = %lld out of range", i, (long long)s.n);
    W8_CHECK_ARG(s.k > 0 && s.k % 16 == 0 && s.k <= w8::kChainMaxK,
                 "step %d: k = %lld must be a positive multiple of 16 up to %d", i, (long long)s.k, w8::kChainMaxK);
    W8_CHECK_ARG(s.x != nullptr && s.w != nullptr && s.s != nullptr && s.y != nullptr, "step %d: null pointer", i);
    W8_CHECK_ALIGN(aligned(s.x, 16) && aligned(s.w, 16), "step %d: x and w must be 16-byte aligned", i);
    W8_CHECK_ALIGN(aligned(s.y, s.logits ? 4 : 2) && aligned(s.s, 2), "step %d: y or s misaligned", i);
    W8_CHECK_ARG(s.logits || s.best == nullptr, "step %d: a greedy key needs a logits step", i);
    W8_CHECK_ALIGN(s.best == nullptr || aligned(s.best, 8), "step %d: best must be 8-byte aligned", i);
    W8_CHECK_ARG(!s.logits || s.n < (1ll << 32) - 1, "step %d: n out of range for the argmax", i);
    w8::ChainStep& d = p->step[i];
    d.x = reinterpret_cast<const __nv_bfloat16*>(s.x);
    d.w = s.w;
    d.s = reinterpret_cast<const __nv_bfloat16*>(s.s);
    d.y = s.y;
    d.best = reinterpret_cast<unsigned long long*>(s.best);
    d.n = static_cast<int>(s.n);
    d.k = static_cast<int>(s.k);
    d.cap = s.logits ? s.cap : 0.f;
    d.logits = s.logits ? 1 : 0;
    gemv_split(d.k, &d.J, &d.S);
  }
  return W8_OK;
}

int chain_device_status(int clear, int* out) {
  int v = 0;
  W8_CUDA_TRY(cudaDeviceSynchronize());
  W8_CUDA_TRY(cudaMemcpyFromSymbol(&v, w8::g_chain_status, sizeof(int)));
  if (clear) {
    const int zero = 0;
    W8_CUDA_TRY(cudaMemcpyToSymbol(w8::g_chain_status, &zero, sizeof(int)));
  }
  *out = v;
  return W8_OK;
}

}  // namespace w8host

extern "C" int64_t w8_gemv_chain_workspace_bytes(int count) { return count < 0 ? 0 : 4ll * (count + 2); }

extern "C" int w8_gemv_chain(const w8_gemv_step* steps, int count, int independent, void* workspace,
                             int64_t workspace_bytes, w8_stream_t stream) {
  static w8::ChainParams params;  // large: built here, copied into the launch
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  int st = w8host::chain_params(steps, count, &params);
  if (st != W8_OK) return st;
  params.independent = independent ? 1 : 0;
  if (count == 0) return W8_OK;
  W8_CHECK_ARG(workspace != nullptr && workspace_bytes >= w8_gemv_chain_workspace_bytes(count),
               "workspace of %lld bytes < %lld", (long long)workspace_bytes,
               (long long)w8_gemv_chain_workspace_bytes(count));
  W8_CHECK_ALIGN(w8host::aligned(workspace, 4), "workspace must be 4-byte aligned");
  params.ctr = static_cast<uint32_t*>(workspace);
  int device = 0;
  st = w8host::require_sm100(&device);
  if (st != W8_OK) return st;
  int sms = 0;
  st = w8host::num_sms(&sms);
  if (st != W8_OK) return st;
  static bool done[64] = {};
  if (!done[device]) {
    W8_CUDA_TRY(cudaFuncSetAttribute(w8::gemv_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     w8::kChainSmem));
    done[device] = true;
  }
  int per_sm = 0;
  W8_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, w8::gemv_chain_kernel, w8::kChainThreads,
                                                            w8::kChainSmem));
  if (per_sm < 1) {
    w8host::set_error("w8_gemv_chain: the kernel does not fit on an SM");
    return W8_ERR_UNSUPPORTED;
  }
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  for (int i = 0; i < count; ++i)
    if (params.step[i].best != nullptr) W8_CUDA_TRY(cudaMemsetAsync(params.step[i].best, 0, 8, s));
  // One CTA per SM, all co-resident (cooperative launch): the CTAs wait on one another.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms, 1, 1);
  cfg.blockDim = dim3(w8::kChainThreads, 1, 1);
  cfg.dynamicSmemBytes = w8::kChainSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeCooperative;
  attr.val.cooperative = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return w8host::cuda_status(cudaLaunchKernelEx(&cfg, w8::gemv_chain_kernel, params));
}
