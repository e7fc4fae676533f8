// The RMSNorm / residual / quant glue between the W8A8 GEMMs (pipeline.py:66-99, 110-114),
// on the GPU.  The reference runs these as torch.compile'd CPU functions on the int32
// GEMM output; here the GEMM's epilogue already dequantises to bf16
// (w8_gemm_dequant_bf16, = _deq), and one warp per row finishes the glue:
//
//   k_in        q, s = _quant(bf16(_rms(h, w)))                                (:66-69)
//   k_post_attn h = bf16(res + bf16(_rms(y, w1)));  q, s = _quant(bf16(_rms(h, w2)))  (:95-99)
//   k_post_ff   h = bf16(res + bf16(_rms(y, w1)));  q, s = _quant(h)           (:110-114)
//   k_attn_out  q, s = _quant(o.transpose(0, 1).reshape(T, H * D))            (:88-92)
//   k_ple_gate  q, s = _quant(bf16(bf16(gelu_tanh(y)) * ple))                  (:117-121)
//   k_ple_out   h = bf16(bf16(h + bf16(_rms(y, w1))) * scalar)                  (:124-127)
//               [+ the next layer's k_in: q, s = _quant(bf16(_rms(h, w2)))]
//
// _rms (pipeline.py:43-46) in fp32: x * pow(mean(x^2) + eps, -0.5), then * w; mean is the
// fp32 sum / N and pow(., -0.5) a correctly rounded reciprocal square root.  The sum is a
// lane-then-warp tree (ATen's CPU order differs), so the last bit of the mean may differ
// from the reference: a bf16 output can move by one bf16 step, an int8 code by one.
//
// One warp per row, the row in registers (N <= 2048, N % 8 == 0, 16-byte rows; H * D <= 4096
// for k_attn_out), eight rows per 256-thread CTA; the norm weights staged in shared memory.
#include "common.cuh"
#include "rowquant.cuh"

namespace w8 {

constexpr int kGlueWarps = 8;
constexpr int kGlueMaxVecs = 8;  // 16-byte vectors per lane: N <= 32 * 8 * 8 = 2048
constexpr int kGlueMaxVecsAttn = 16;  // k_attn_out rows: H * D <= 4096 (head_dim 512 layers)

enum GlueMode : int { kGlueIn = 0, kGluePost1 = 1, kGluePost2 = 2, kGlueAttnOut = 3, kGluePleGate = 4 };

struct GlueArgs {
  const __nv_bfloat16* x;  // k_in: h; post: y = _deq(acc); attn_out: o [H, T, D]
  int64_t ldx;             // row (token) pitch of x in elements
  int64_t ld_head;         // attn_out: pitch between heads of o, in elements
  int head_dim;            // attn_out: D
  const __nv_bfloat16* res;  // post: the residual stream; PLE gate: this layer's per-layer input
  int64_t ldr;
  const __nv_bfloat16* w1;
  const __nv_bfloat16* w2;
  float eps;
  float scalar;            // post: the layer scalar applied to h (1: none)
  __nv_bfloat16* h;        // post: the new residual stream
  int64_t ldh;
  int8_t* q;               // Post1: may be null (no quant of h)
  int64_t ldq;
  float* s;
  int t, n;
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Eight bf16 values packed in 16 bytes <-> fp32 (exact both ways for bf16-representable
// values; pack rounds to nearest even).  Every value the glue keeps between steps is a
// bf16, so a lane holds its share of the row packed: 4 registers per 8 values.
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = __uint_as_float(w[j] << 16);
    f[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
  }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
    w[j] = *reinterpret_cast<uint32_t*>(&b);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ uint4 ld16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

// pow(mean(x^2) + eps, -0.5) of this warp's row, held packed in v[].
template <int NV>
__device__ __forceinline__ float rms_factor(const uint4 (&v)[NV], int nv, int lane, int n, float eps) {
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i)
    if (lane + 32 * i < nv) {
      float f[8];
      unpack8(v[i], f);
      // fma(x, x, ss) = ss + x * x, one rounding fewer: the square of a bf16 is exact in
      // fp32 (below 2^-63 it can round, but then eps decides the factor anyway).
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = __fmaf_rn(f[e], f[e], ss);
    }
  const float ms = __fdiv_rn(warp_sum(ss), static_cast<float>(n));
  return __frsqrt_rn(__fadd_rn(ms, eps));
}

__device__ __forceinline__ float rbf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// One row of the glue (the warp's registers hold the row between the steps).
// NV: 16-byte vectors per lane the row may need (row length <= 256 NV).
template <int MODE, int NV>
__device__ __forceinline__ void glue_row(const GlueArgs& a, int row, int lane, int nv, const uint4* w1s,
                                         const uint4* w2s) {
  constexpr int kMax = NV;
  uint4 v[kMax];
#pragma unroll
  for (int i = 0; i < kMax; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nv) {
      if constexpr (MODE == kGlueAttnOut) {
        const int c = vi * 8, head = c / a.head_dim;
        v[i] = ld16(a.x + head * a.ld_head + static_cast<int64_t>(row) * a.ldx + (c - head * a.head_dim));
      } else {
        v[i] = ld16(a.x + static_cast<int64_t>(row) * a.ldx + vi * 8);
      }
    }
  }
  if constexpr (MODE == kGluePleGate) {
#pragma unroll
    for (int i = 0; i < kMax; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nv) {
        // bf16(gelu_tanh(x) * ple): the product of two bf16 values is one packed bf16 multiply.
        const uint4 p = ld16(a.res + static_cast<int64_t>(row) * a.ldr + vi * 8);
        v[i] = make_uint4(bf16x2_mul(gelu_tanh_bf16x2(v[i].x), p.x), bf16x2_mul(gelu_tanh_bf16x2(v[i].y), p.y),
                          bf16x2_mul(gelu_tanh_bf16x2(v[i].z), p.z), bf16x2_mul(gelu_tanh_bf16x2(v[i].w), p.w));
      }
    }
  } else if constexpr (MODE != kGlueAttnOut) {
    uint4 res[MODE == kGlueIn ? 1 : NV];
    if constexpr (MODE != kGlueIn) {
#pragma unroll
      for (int i = 0; i < kMax; ++i)
        if (lane + 32 * i < nv) res[i] = ld16(a.res + static_cast<int64_t>(row) * a.ldr + (lane + 32 * i) * 8);
    }
    const float r1 = rms_factor<NV>(v, nv, lane, a.n, a.eps);
    const uint64_t r1_2 = f2_pack(r1, r1), sc2 = f2_pack(a.scalar, a.scalar);
#pragma unroll
    for (int i = 0; i < kMax; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nv) {
        // Two elements per packed f32x2 step, in the scalar operation order.
        uint32_t xw[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
        const uint4 wv = w1s[vi];
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t rw[4] = {0u, 0u, 0u, 0u};
        if constexpr (MODE != kGlueIn) rw[0] = res[i].x, rw[1] = res[i].y, rw[2] = res[i].z, rw[3] = res[i].w;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t t = bf16x2_from_f2(f2_mul(f2_mul(f2_from_bf16x2(xw[j]), r1_2), f2_from_bf16x2(ww[j])));
          if constexpr (MODE == kGlueIn) {
            xw[j] = t;
          } else {
            uint32_t h = bf16x2_add(rw[j], t);  // bf16(res + t)
            if (a.scalar != 1.f) h = bf16x2_from_f2(f2_mul(f2_from_bf16x2(h), sc2));
            xw[j] = h;
          }
        }
        v[i] = make_uint4(xw[0], xw[1], xw[2], xw[3]);
        if constexpr (MODE != kGlueIn)
          *reinterpret_cast<uint4*>(a.h + static_cast<int64_t>(row) * a.ldh + vi * 8) = v[i];
      }
    }
    if constexpr (MODE == kGluePost2) {
      const float r2 = rms_factor<NV>(v, nv, lane, a.n, a.eps);
      const uint64_t r2_2 = f2_pack(r2, r2);
#pragma unroll
      for (int i = 0; i < kMax; ++i) {
        const int vi = lane + 32 * i;
        if (vi < nv) {
          uint32_t xw[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
          const uint4 wv = w2s[vi];
          const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
          for (int j = 0; j < 4; ++j)
            xw[j] = bf16x2_from_f2(f2_mul(f2_mul(f2_from_bf16x2(xw[j]), r2_2), f2_from_bf16x2(ww[j])));
          v[i] = make_uint4(xw[0], xw[1], xw[2], xw[3]);
        }
      }
    }
  }
  if (MODE == kGluePost1 && a.q == nullptr) return;  // k_ple_out alone: h only
  // _quant of the row.
  uint32_t m2 = 0u;  // two bf16 lanes of max |x|
#pragma unroll
  for (int i = 0; i < kMax; ++i)
    if (lane + 32 * i < nv) m2 = bf16x2_absmax8(v[i], m2);
  const float amax = warp_max(bf16x2_max_lanes(m2));
  const float sc = __fdiv_rn(fmaxf(amax, 1e-8f), 127.f);
  const float rc = __frcp_rn(sc);
  if (lane == 0) a.s[row] = sc;
#pragma unroll
  for (int i = 0; i < kMax; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nv)
      *reinterpret_cast<uint2*>(a.q + static_cast<int64_t>(row) * a.ldq + vi * 8) = quant8_bf16_codes(v[i], sc, rc);
  }
}

// Rows of at most 1536 values (the hidden size) keep 4 CTAs (32 warps) per SM resident, so a
// 3658-token prompt needs no second pass over rows.
template <int MODE, int NV>
__global__ void __launch_bounds__(32 * kGlueWarps, NV <= 6 ? 4 : 3) glue_rows_kernel(const GlueArgs a) {
  pdl_launch_dependents();
  // The norm weights are the same for every row: staged once per CTA in shared memory,
  // before waiting for the previous kernel of the stream (they do not depend on it).
  __shared__ uint4 w1s[(MODE == kGlueAttnOut || MODE == kGluePleGate) ? 1 : 32 * NV];
  __shared__ uint4 w2s[MODE == kGluePost2 ? 32 * NV : 1];
  const int nv = a.n / 8;
  if constexpr (MODE != kGlueAttnOut && MODE != kGluePleGate) {
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
      w1s[i] = ld16(a.w1 + i * 8);
      if constexpr (MODE == kGluePost2) w2s[i] = ld16(a.w2 + i * 8);
    }
    __syncthreads();
  }
  pdl_wait();  // the rows come from the previous kernel
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int row = blockIdx.x * kGlueWarps + warp; row < a.t; row += gridDim.x * kGlueWarps)
    glue_row<MODE, NV>(a, row, lane, nv, w1s, w2s);
}

// k_qkv (pipeline.py:72-86) after the qkv GEMM with the dequant fused (y = _deq(acc),
// bf16 [T, (H + 2 KV) * D], or [T, H * D] for a KV-shared layer): one warp per
// (token, head).  q and k heads: bf16(_rms(x, w)) then RoPE, each bf16 op rounded as
// eager torch does: out = bf16(bf16(x * cos) + bf16(rotate_half(x) * sin)); v heads:
// bf16(_rms(x, None)).  Output head-major: out[head * ld_head + t * ld_tok + d], the
// layout of the reference's .transpose(0, 1) results.  D is 64, 128, 256 or 512, so a
// lane's rotate_half partner is in its own registers (D = 512) or in lane ^ (D / 16).
struct QkvArgs {
  const __nv_bfloat16* y;
  int64_t ldy;
  const __nv_bfloat16* cos;
  const __nv_bfloat16* sin;
  int64_t ldcs;
  const __nv_bfloat16* qw;
  const __nv_bfloat16* kw;
  float eps;
  __nv_bfloat16* out;
  int64_t ld_head, ld_tok;
  int t, heads, kv_heads, d, shared;
};

__global__ void __launch_bounds__(32 * kGlueWarps) qkv_rows_kernel(const QkvArgs a) {
  pdl_launch_dependents();
  pdl_wait();  // y comes from the previous kernel
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_tok = a.shared ? a.heads : a.heads + 2 * a.kv_heads;
  const int64_t job = static_cast<int64_t>(blockIdx.x) * kGlueWarps + warp;
  if (job >= static_cast<int64_t>(a.t) * per_tok) return;
  const int tok = static_cast<int>(job / per_tok);
  const int head = static_cast<int>(job - static_cast<int64_t>(tok) * per_tok);
  const bool is_v = head >= a.heads + a.kv_heads;
  const __nv_bfloat16* w = head < a.heads ? a.qw : (is_v ? nullptr : a.kw);
  const int nv = a.d / 8;                 // vectors of the head
  const int slots = nv > 32 ? 2 : 1;      // vectors per lane
  const bool active = lane < nv;          // D = 64 / 128 use 8 / 16 lanes
  const __nv_bfloat16* yr = a.y + static_cast<int64_t>(tok) * a.ldy + static_cast<int64_t>(head) * a.d;
  uint4 v[2];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 2; ++j)
    if (j < slots && active) {
      v[j] = ld16(yr + (lane + 32 * j) * 8);
      float f[8];
      unpack8(v[j], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = __fmaf_rn(f[e], f[e], ss);  // = ss + x * x, as in rms_factor
    }
  const float r = __frsqrt_rn(__fadd_rn(__fdiv_rn(warp_sum(ss), static_cast<float>(a.d)), a.eps));
  // bf16(_rms(x, w)) of this lane's vectors.
#pragma unroll
  for (int j = 0; j < 2; ++j)
    if (j < slots && active) {
      const int c = (lane + 32 * j) * 8;
      // Two elements per packed f32x2 step (the same IEEE operations as one at a time).
      const uint64_t r2 = f2_pack(r, r);
      uint32_t xw[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
      if (w != nullptr) {
        const uint4 gv = ld16(w + c);
        const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
          xw[q] = bf16x2_from_f2(f2_mul(f2_mul(f2_from_bf16x2(xw[q]), r2), f2_from_bf16x2(gw[q])));
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) xw[q] = bf16x2_from_f2(f2_mul(f2_from_bf16x2(xw[q]), r2));
      }
      v[j] = make_uint4(xw[0], xw[1], xw[2], xw[3]);
    }
  if (!is_v) {
    // rotate_half partner of vector vi is vi + nv/2 (first half) or vi - nv/2.
    uint4 p[2];
    if (slots == 2) {
      p[0] = v[1];
      p[1] = v[0];
    } else {
      const int src = lane ^ (nv / 2);
      p[0].x = __shfl_sync(0xffffffffu, v[0].x, src);
      p[0].y = __shfl_sync(0xffffffffu, v[0].y, src);
      p[0].z = __shfl_sync(0xffffffffu, v[0].z, src);
      p[0].w = __shfl_sync(0xffffffffu, v[0].w, src);
    }
    const __nv_bfloat16* cr = a.cos + static_cast<int64_t>(tok) * a.ldcs;
    const __nv_bfloat16* sr = a.sin + static_cast<int64_t>(tok) * a.ldcs;
#pragma unroll
    for (int j = 0; j < 2; ++j)
      if (j < slots && active) {
        const int vi = lane + 32 * j;
        const int c = vi * 8;
        const bool first = vi < nv / 2;
        // bf16(bf16(x * cos) + bf16(rotate_half(x) * sin)) on packed bf16 pairs (each step
        // rounded once, as eager torch's bf16 ops); the first half's partner is negated by
        // its sign bits (exact, as -x).
        const uint4 cv = ld16(cr + c), sv = ld16(sr + c);
        const uint32_t xw[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
        const uint32_t pw[4] = {p[j].x, p[j].y, p[j].z, p[j].w};
        const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w};
        const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
        const uint32_t flip = first ? 0x80008000u : 0u;
        uint32_t ow[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          ow[q] = bf16x2_add(bf16x2_mul(xw[q], cw[q]), bf16x2_mul(pw[q] ^ flip, sw[q]));
        v[j] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
      }
  }
  __nv_bfloat16* orow = a.out + static_cast<int64_t>(head) * a.ld_head + static_cast<int64_t>(tok) * a.ld_tok;
#pragma unroll
  for (int j = 0; j < 2; ++j)
    if (j < slots && active) *reinterpret_cast<uint4*>(orow + (lane + 32 * j) * 8) = v[j];
}

// k_qkv at head_dim 256 with two (token, head) jobs per warp: both jobs' rows are in flight
// together and their reductions interleave, where one job per warp left each warp a short
// dependent chain (load, reduce, load, RoPE, store) and the launch 7.7 waves of them at
// M = 3658.  Every element takes the operations of qkv_rows_kernel in the same order, so
// the output bits are the same.
__global__ void __launch_bounds__(32 * kGlueWarps) qkv_rows256x2_kernel(const QkvArgs a) {
  pdl_launch_dependents();
  pdl_wait();  // y comes from the previous kernel
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_tok = a.shared ? a.heads : a.heads + 2 * a.kv_heads;
  const int64_t njobs = static_cast<int64_t>(a.t) * per_tok;
  const int64_t job0 = (static_cast<int64_t>(blockIdx.x) * kGlueWarps + warp) * 2;
  if (job0 >= njobs) return;
  uint4 v[2];
  int tok[2], head[2];
  bool valid[2];
  float ss[2];
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int64_t job = job0 + q;
    valid[q] = job < njobs;
    tok[q] = valid[q] ? static_cast<int>(job / per_tok) : 0;
    head[q] = valid[q] ? static_cast<int>(job - static_cast<int64_t>(tok[q]) * per_tok) : 0;
    v[q] = valid[q] ? ld16(a.y + static_cast<int64_t>(tok[q]) * a.ldy + static_cast<int64_t>(head[q]) * 256 + lane * 8)
                    : make_uint4(0u, 0u, 0u, 0u);
    float f[8];
    unpack8(v[q], f);
    ss[q] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss[q] = __fmaf_rn(f[e], f[e], ss[q]);  // = ss + x * x, as in rms_factor
  }
  float r[2];
#pragma unroll
  for (int q = 0; q < 2; ++q) r[q] = __frsqrt_rn(__fadd_rn(__fdiv_rn(warp_sum(ss[q]), 256.f), a.eps));
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const bool is_v = head[q] >= a.heads + a.kv_heads;
    const __nv_bfloat16* w = head[q] < a.heads ? a.qw : (is_v ? nullptr : a.kw);
    const uint64_t r2 = f2_pack(r[q], r[q]);
    uint32_t xw[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
    if (w != nullptr) {
      const uint4 gv = ld16(w + lane * 8);
      const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
        xw[i] = bf16x2_from_f2(f2_mul(f2_mul(f2_from_bf16x2(xw[i]), r2), f2_from_bf16x2(gw[i])));
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) xw[i] = bf16x2_from_f2(f2_mul(f2_from_bf16x2(xw[i]), r2));
    }
    v[q] = make_uint4(xw[0], xw[1], xw[2], xw[3]);
  }
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const bool is_v = head[q] >= a.heads + a.kv_heads;
    // rotate_half partner: lane ^ 16 (32 vectors of 8 columns); every lane takes part in
    // the shuffles, a v head's lanes discard the result.
    uint4 p;
    p.x = __shfl_sync(0xffffffffu, v[q].x, lane ^ 16);
    p.y = __shfl_sync(0xffffffffu, v[q].y, lane ^ 16);
    p.z = __shfl_sync(0xffffffffu, v[q].z, lane ^ 16);
    p.w = __shfl_sync(0xffffffffu, v[q].w, lane ^ 16);
    if (!is_v && valid[q]) {
      const int c = lane * 8;
      const uint4 cv = ld16(a.cos + static_cast<int64_t>(tok[q]) * a.ldcs + c);
      const uint4 sv = ld16(a.sin + static_cast<int64_t>(tok[q]) * a.ldcs + c);
      const uint32_t xw[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
      const uint32_t pw[4] = {p.x, p.y, p.z, p.w};
      const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w};
      const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
      const uint32_t flip = lane < 16 ? 0x80008000u : 0u;
      uint32_t ow[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) ow[i] = bf16x2_add(bf16x2_mul(xw[i], cw[i]), bf16x2_mul(pw[i] ^ flip, sw[i]));
      v[q] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
    if (valid[q])
      *reinterpret_cast<uint4*>(a.out + static_cast<int64_t>(head[q]) * a.ld_head +
                                static_cast<int64_t>(tok[q]) * a.ld_tok + lane * 8) = v[q];
  }
}

}  // namespace w8

namespace w8host {

int require_sm100(int* device);

// Launch with programmatic stream serialization: the kernel may start (and stage its
// constant operands) while the previous kernel of the stream drains; it waits for that
// kernel (griddepcontrol.wait) before reading its output.
template <typename Kernel, typename Args>
static int launch_pdl_glue(Kernel kern, unsigned grid, const Args& a, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(32 * w8::kGlueWarps, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, a));
}

// One warp per row, at most as many CTAs as fit on the GPU at once (each warp then loops
// over rows a grid's worth of warps apart).
template <typename Kernel>
static int glue_go(Kernel kern, const w8::GlueArgs& a, cudaStream_t stream) {
  int sms = 0, per_sm = 0;
  int st = num_sms(&sms);
  if (st != W8_OK) return st;
  W8_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 32 * w8::kGlueWarps, 0));
  const int64_t need = (static_cast<int64_t>(a.t) + w8::kGlueWarps - 1) / w8::kGlueWarps;
  const int64_t cap = static_cast<int64_t>(sms) * (per_sm > 0 ? per_sm : 1);
  const unsigned grid = static_cast<unsigned>(need < cap ? need : cap);
  return launch_pdl_glue(kern, grid, a, stream);
}

static int glue_launch(int mode, const w8::GlueArgs& a, cudaStream_t stream) {
  W8_CHECK_ARG(a.t >= 0 && a.n >= 0, "negative size");
  if (a.t == 0) return W8_OK;
  const int max_n = 32 * 8 * (mode == w8::kGlueAttnOut ? w8::kGlueMaxVecsAttn : w8::kGlueMaxVecs);
  W8_CHECK_ARG(a.n > 0 && a.n % 8 == 0 && a.n <= max_n, "row length %d must be a multiple of 8 and at most %d", a.n,
               max_n);
  const bool no_quant = mode == w8::kGluePost1 && a.q == nullptr && a.s == nullptr;
  W8_CHECK_ARG(a.x != nullptr && (no_quant || (a.q != nullptr && a.s != nullptr)), "null pointer");
  W8_CHECK_ALIGN(aligned(a.x, 16) && a.ldx % 8 == 0, "x must be 16-byte aligned with a pitch %% 8 == 0");
  W8_CHECK_ALIGN(no_quant || (aligned(a.q, 8) && a.ldq % 8 == 0 && a.ldq >= a.n),
                 "q must be 8-byte aligned, ldq %% 8 == 0, ldq >= n");
  if (mode == w8::kGluePleGate) {
    W8_CHECK_ARG(a.res != nullptr, "null per-layer input");
    W8_CHECK_ALIGN(aligned(a.res, 16) && a.ldr % 8 == 0, "per-layer input rows must be 16-byte aligned, pitch %% 8 == 0");
    W8_CHECK_ARG(a.ldr >= a.n && a.ldx >= a.n, "row pitch smaller than n");
  } else if (mode != w8::kGlueAttnOut) {
    W8_CHECK_ARG(a.w1 != nullptr, "null norm weight");
    W8_CHECK_ALIGN(aligned(a.w1, 16), "norm weights must be 16-byte aligned");
    W8_CHECK_ARG(a.ldx >= a.n, "row pitch smaller than n");
  }
  if (mode == w8::kGluePost1 || mode == w8::kGluePost2) {
    W8_CHECK_ARG(a.res != nullptr && a.h != nullptr, "null residual pointer");
    W8_CHECK_ALIGN(aligned(a.res, 16) && a.ldr % 8 == 0 && aligned(a.h, 16) && a.ldh % 8 == 0,
                   "residual rows must be 16-byte aligned with pitches %% 8 == 0");
    W8_CHECK_ARG(a.ldr >= a.n && a.ldh >= a.n, "residual pitch smaller than n");
  }
  if (mode == w8::kGluePost2) {
    W8_CHECK_ARG(a.w2 != nullptr, "null second norm weight");
    W8_CHECK_ALIGN(aligned(a.w2, 16), "norm weights must be 16-byte aligned");
  }
  if (mode == w8::kGlueAttnOut) {
    W8_CHECK_ARG(a.head_dim > 0 && a.head_dim % 8 == 0 && a.n % a.head_dim == 0,
                 "head_dim %d must be a multiple of 8 dividing H * D", a.head_dim);
    W8_CHECK_ALIGN(a.ld_head % 8 == 0, "head pitch must be a multiple of 8 elements");
    W8_CHECK_ARG(a.ldx >= a.head_dim, "token pitch smaller than head_dim");
  }
  int device = 0;
  const int st = require_sm100(&device);
  if (st != W8_OK) return st;
  switch (mode) {
    case w8::kGlueIn:
      return a.n <= 1536 ? glue_go(w8::glue_rows_kernel<w8::kGlueIn, 6>, a, stream)
                         : glue_go(w8::glue_rows_kernel<w8::kGlueIn, w8::kGlueMaxVecs>, a, stream);
    case w8::kGluePost1:
      return a.n <= 1536 ? glue_go(w8::glue_rows_kernel<w8::kGluePost1, 6>, a, stream)
                         : glue_go(w8::glue_rows_kernel<w8::kGluePost1, w8::kGlueMaxVecs>, a, stream);
    case w8::kGluePost2:
      return a.n <= 1536 ? glue_go(w8::glue_rows_kernel<w8::kGluePost2, 6>, a, stream)
                         : glue_go(w8::glue_rows_kernel<w8::kGluePost2, w8::kGlueMaxVecs>, a, stream);
    case w8::kGluePleGate:
      return a.n <= 1536 ? glue_go(w8::glue_rows_kernel<w8::kGluePleGate, 6>, a, stream)
                         : glue_go(w8::glue_rows_kernel<w8::kGluePleGate, w8::kGlueMaxVecs>, a, stream);
    default:
      return a.n <= 32 * 8 * w8::kGlueMaxVecs
                 ? glue_go(w8::glue_rows_kernel<w8::kGlueAttnOut, w8::kGlueMaxVecs>, a, stream)
                 : glue_go(w8::glue_rows_kernel<w8::kGlueAttnOut, w8::kGlueMaxVecsAttn>, a, stream);
  }
}

static w8::GlueArgs glue_args(int64_t t, int64_t n) {
  w8::GlueArgs a = {};
  a.t = static_cast<int>(t);
  a.n = static_cast<int>(n);
  a.scalar = 1.f;
  return a;
}

}  // namespace w8host

extern "C" int w8_rms_quant_bf16(const uint16_t* h, int64_t ldh, const uint16_t* w, float eps, int8_t* q,
                                 int64_t ldq, float* s, int64_t t, int64_t n, w8_stream_t stream) {
  W8_CHECK_ARG(t >= 0 && n >= 0 && t < (1ll << 31) && n < (1ll << 31), "bad size");
  w8::GlueArgs a = w8host::glue_args(t, n);
  a.x = reinterpret_cast<const __nv_bfloat16*>(h);
  a.ldx = ldh;
  a.w1 = reinterpret_cast<const __nv_bfloat16*>(w);
  a.eps = eps;
  a.q = q;
  a.ldq = ldq;
  a.s = s;
  return w8host::glue_launch(w8::kGlueIn, a, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int w8_post_norm_quant_bf16(const uint16_t* y, int64_t ldy, const uint16_t* res, int64_t ldr,
                                       const uint16_t* w1, const uint16_t* w2, float eps, uint16_t* h,
                                       int64_t ldh, int8_t* q, int64_t ldq, float* s, int64_t t, int64_t n,
                                       w8_stream_t stream) {
  W8_CHECK_ARG(t >= 0 && n >= 0 && t < (1ll << 31) && n < (1ll << 31), "bad size");
  w8::GlueArgs a = w8host::glue_args(t, n);
  a.x = reinterpret_cast<const __nv_bfloat16*>(y);
  a.ldx = ldy;
  a.res = reinterpret_cast<const __nv_bfloat16*>(res);
  a.ldr = ldr;
  a.w1 = reinterpret_cast<const __nv_bfloat16*>(w1);
  a.w2 = reinterpret_cast<const __nv_bfloat16*>(w2);
  a.eps = eps;
  a.h = reinterpret_cast<__nv_bfloat16*>(h);
  a.ldh = ldh;
  a.q = q;
  a.ldq = ldq;
  a.s = s;
  return w8host::glue_launch(w2 != nullptr ? w8::kGluePost2 : w8::kGluePost1, a,
                             reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int w8_ple_gate_quant_bf16(const uint16_t* y, int64_t ldy, const uint16_t* ple, int64_t ldp, int8_t* q,
                                      int64_t ldq, float* s, int64_t t, int64_t n, w8_stream_t stream) {
  W8_CHECK_ARG(t >= 0 && n >= 0 && t < (1ll << 31) && n < (1ll << 31), "bad size");
  w8::GlueArgs a = w8host::glue_args(t, n);
  a.x = reinterpret_cast<const __nv_bfloat16*>(y);
  a.ldx = ldy;
  a.res = reinterpret_cast<const __nv_bfloat16*>(ple);
  a.ldr = ldp;
  a.q = q;
  a.ldq = ldq;
  a.s = s;
  return w8host::glue_launch(w8::kGluePleGate, a, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int w8_ple_out_bf16(const uint16_t* y, int64_t ldy, const uint16_t* res, int64_t ldr,
                               const uint16_t* w_post, float scalar, const uint16_t* w_next, float eps, uint16_t* h,
                               int64_t ldh, int8_t* q, int64_t ldq, float* s, int64_t t, int64_t n,
                               w8_stream_t stream) {
  W8_CHECK_ARG(t >= 0 && n >= 0 && t < (1ll << 31) && n < (1ll << 31), "bad size");
  W8_CHECK_ARG(w_next != nullptr || (q == nullptr && s == nullptr),
               "q / s are written only with the next layer's norm weight");
  w8::GlueArgs a = w8host::glue_args(t, n);
  a.x = reinterpret_cast<const __nv_bfloat16*>(y);
  a.ldx = ldy;
  a.res = reinterpret_cast<const __nv_bfloat16*>(res);
  a.ldr = ldr;
  a.w1 = reinterpret_cast<const __nv_bfloat16*>(w_post);
  a.w2 = reinterpret_cast<const __nv_bfloat16*>(w_next);
  a.eps = eps;
  a.scalar = scalar;
  a.h = reinterpret_cast<__nv_bfloat16*>(h);
  a.ldh = ldh;
  a.q = q;
  a.ldq = ldq;
  a.s = s;
  return w8host::glue_launch(w_next != nullptr ? w8::kGluePost2 : w8::kGluePost1, a,
                             reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int w8_attn_out_quant_bf16(const uint16_t* o, int64_t ld_head, int64_t ld_tok, int8_t* q,
                                      int64_t ldq, float* s, int64_t t, int64_t heads, int64_t head_dim,
                                      w8_stream_t stream) {
  W8_CHECK_ARG(t >= 0 && heads >= 0 && head_dim >= 0 && t < (1ll << 31) && heads * head_dim < (1ll << 31),
               "bad size");
  w8::GlueArgs a = w8host::glue_args(t, heads * head_dim);
  a.x = reinterpret_cast<const __nv_bfloat16*>(o);
  a.ldx = ld_tok;
  a.ld_head = ld_head;
  a.head_dim = static_cast<int>(head_dim);
  a.q = q;
  a.ldq = ldq;
  a.s = s;
  return w8host::glue_launch(w8::kGlueAttnOut, a, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int w8_qkv_norm_rope_bf16(const uint16_t* y, int64_t ldy, const uint16_t* cos, const uint16_t* sin,
                                     int64_t ldcs, const uint16_t* qw, const uint16_t* kw, float eps,
                                     uint16_t* out, int64_t ld_head, int64_t ld_tok, int64_t t, int64_t heads,
                                     int64_t kv_heads, int64_t head_dim, int shared, w8_stream_t stream) {
  using namespace w8host;
  W8_CHECK_ARG(t >= 0 && heads >= 0 && kv_heads >= 0 && t < (1ll << 31), "bad size");
  W8_CHECK_ARG(head_dim == 64 || head_dim == 128 || head_dim == 256 || head_dim == 512,
               "head_dim = %lld must be 64, 128, 256 or 512", (long long)head_dim);
  const int64_t per_tok = shared ? heads : heads + 2 * kv_heads;
  if (t == 0 || per_tok == 0) return W8_OK;
  W8_CHECK_ARG(y != nullptr && cos != nullptr && sin != nullptr && qw != nullptr && out != nullptr,
               "null pointer");
  W8_CHECK_ARG(shared || kv_heads == 0 || kw != nullptr, "null k_norm weight");
  W8_CHECK_ARG(ldy >= per_tok * head_dim && ldcs >= head_dim && ld_tok >= head_dim, "pitch too small");
  W8_CHECK_ALIGN(aligned(y, 16) && ldy % 8 == 0 && aligned(cos, 16) && aligned(sin, 16) && ldcs % 8 == 0 &&
                     aligned(qw, 16) && (kw == nullptr || aligned(kw, 16)) && aligned(out, 16) &&
                     ld_head % 8 == 0 && ld_tok % 8 == 0,
                 "rows, weights and cos/sin must be 16-byte aligned with pitches %% 8 == 0");
  int device = 0;
  const int st = require_sm100(&device);
  if (st != W8_OK) return st;
  w8::QkvArgs a = {};
  a.y = reinterpret_cast<const __nv_bfloat16*>(y);
  a.ldy = ldy;
  a.cos = reinterpret_cast<const __nv_bfloat16*>(cos);
  a.sin = reinterpret_cast<const __nv_bfloat16*>(sin);
  a.ldcs = ldcs;
  a.qw = reinterpret_cast<const __nv_bfloat16*>(qw);
  a.kw = reinterpret_cast<const __nv_bfloat16*>(kw);
  a.eps = eps;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.ld_head = ld_head;
  a.ld_tok = ld_tok;
  a.t = static_cast<int>(t);
  a.heads = static_cast<int>(heads);
  a.kv_heads = static_cast<int>(kv_heads);
  a.d = static_cast<int>(head_dim);
  a.shared = shared != 0;
  const int64_t jobs = t * per_tok;
  if (head_dim == 256) {  // two (token, head) jobs per warp
    const unsigned grid2 = static_cast<unsigned>((jobs + 2 * w8::kGlueWarps - 1) / (2 * w8::kGlueWarps));
    return launch_pdl_glue(w8::qkv_rows256x2_kernel, grid2, a, reinterpret_cast<cudaStream_t>(stream));
  }
  const unsigned grid = static_cast<unsigned>((jobs + w8::kGlueWarps - 1) / w8::kGlueWarps);
  return launch_pdl_glue(w8::qkv_rows_kernel, grid, a, reinterpret_cast<cudaStream_t>(stream));
}
