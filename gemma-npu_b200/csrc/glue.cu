// The RMSNorm / residual / quant glue between the W8A8 GEMMs (pipeline.py:66-99, 110-114),
// on the GPU.  The reference runs these as torch.compile'd CPU functions on the int32
// GEMM output; here the GEMM's epilogue already dequantises to bf16
// (w8_gemm_dequant_bf16, = _deq), and one warp per row finishes the glue:
//
//   k_in        q, s = _quant(bf16(_rms(h, w)))                                (:66-69)
//   k_post_attn h = bf16(res + bf16(_rms(y, w1)));  q, s = _quant(bf16(_rms(h, w2)))  (:95-99)
//   k_post_ff   h = bf16(res + bf16(_rms(y, w1)));  q, s = _quant(h)           (:110-114)
//   k_attn_out  q, s = _quant(o.transpose(0, 1).reshape(T, H * D))            (:88-92)
//
// _rms (pipeline.py:43-46) in fp32: x * pow(mean(x^2) + eps, -0.5), then * w; mean is the
// fp32 sum / N and pow(., -0.5) a correctly rounded reciprocal square root.  The sum is a
// lane-then-warp tree (ATen's CPU order differs), so the last bit of the mean may differ
// from the reference: a bf16 output can move by one bf16 step, an int8 code by one.
//
// One warp per row, the row in registers (N <= 2048, N % 8 == 0, 16-byte rows), eight
// rows per 256-thread CTA: no shared memory and no block barrier.
#include "common.cuh"
#include "rowquant.cuh"

namespace w8 {

constexpr int kGlueWarps = 8;
constexpr int kGlueMaxVecs = 8;  // 16-byte vectors per lane: N <= 32 * 8 * 8 = 2048

enum GlueMode : int { kGlueIn = 0, kGluePost1 = 1, kGluePost2 = 2, kGlueAttnOut = 3 };

struct GlueArgs {
  const __nv_bfloat16* x;  // k_in: h; post: y = _deq(acc); attn_out: o [H, T, D]
  int64_t ldx;             // row (token) pitch of x in elements
  int64_t ld_head;         // attn_out: pitch between heads of o, in elements
  int head_dim;            // attn_out: D
  const __nv_bfloat16* res;
  int64_t ldr;
  const __nv_bfloat16* w1;
  const __nv_bfloat16* w2;
  float eps;
  __nv_bfloat16* h;        // post: the new residual stream
  int64_t ldh;
  int8_t* q;
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
__device__ __forceinline__ float rms_factor(const uint4 (&v)[kGlueMaxVecs], int nv, int lane, int n, float eps) {
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kGlueMaxVecs; ++i)
    if (lane + 32 * i < nv) {
      float f[8];
      unpack8(v[i], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = __fadd_rn(ss, __fmul_rn(f[e], f[e]));
    }
  const float ms = __fdiv_rn(warp_sum(ss), static_cast<float>(n));
  return __frsqrt_rn(__fadd_rn(ms, eps));
}

__device__ __forceinline__ float rbf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

template <int MODE>
__global__ void __launch_bounds__(32 * kGlueWarps) glue_rows_kernel(const GlueArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kGlueWarps + warp;
  if (row >= a.t) return;
  const int nv = a.n / 8;
  uint4 v[kGlueMaxVecs];
#pragma unroll
  for (int i = 0; i < kGlueMaxVecs; ++i) {
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
  if constexpr (MODE != kGlueAttnOut) {
    uint4 res[MODE == kGlueIn ? 1 : kGlueMaxVecs];
    if constexpr (MODE != kGlueIn) {
#pragma unroll
      for (int i = 0; i < kGlueMaxVecs; ++i)
        if (lane + 32 * i < nv) res[i] = ld16(a.res + static_cast<int64_t>(row) * a.ldr + (lane + 32 * i) * 8);
    }
    const float r1 = rms_factor(v, nv, lane, a.n, a.eps);
#pragma unroll
    for (int i = 0; i < kGlueMaxVecs; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nv) {
        float x[8], w[8];
        unpack8(v[i], x);
        unpack8(ld16(a.w1 + vi * 8), w);
        float rr[8];
        if constexpr (MODE != kGlueIn) unpack8(res[i], rr);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float t = rbf16(__fmul_rn(__fmul_rn(x[e], r1), w[e]));
          x[e] = MODE == kGlueIn ? t : rbf16(__fadd_rn(rr[e], t));
        }
        v[i] = pack8(x);
        if constexpr (MODE != kGlueIn)
          *reinterpret_cast<uint4*>(a.h + static_cast<int64_t>(row) * a.ldh + vi * 8) = v[i];
      }
    }
    if constexpr (MODE == kGluePost2) {
      const float r2 = rms_factor(v, nv, lane, a.n, a.eps);
#pragma unroll
      for (int i = 0; i < kGlueMaxVecs; ++i) {
        const int vi = lane + 32 * i;
        if (vi < nv) {
          float x[8], w[8];
          unpack8(v[i], x);
          unpack8(ld16(a.w2 + vi * 8), w);
#pragma unroll
          for (int e = 0; e < 8; ++e) x[e] = rbf16(__fmul_rn(__fmul_rn(x[e], r2), w[e]));
          v[i] = pack8(x);
        }
      }
    }
  }
  // _quant of the row.
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kGlueMaxVecs; ++i)
    if (lane + 32 * i < nv) {
      float x[8];
      unpack8(v[i], x);
#pragma unroll
      for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(x[e]));
    }
  amax = warp_max(amax);
  const float sc = __fdiv_rn(fmaxf(amax, 1e-8f), 127.f);
  const float rc = __frcp_rn(sc);
  if (lane == 0) a.s[row] = sc;
#pragma unroll
  for (int i = 0; i < kGlueMaxVecs; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nv) {
      float x[8];
      unpack8(v[i], x);
      int8_t out[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) out[e] = quant_one(x[e], sc, rc);
      store_q<8>(a.q + static_cast<int64_t>(row) * a.ldq + vi * 8, out);
    }
  }
}

}  // namespace w8

namespace w8host {

int require_sm100(int* device);

static int glue_launch(int mode, const w8::GlueArgs& a, cudaStream_t stream) {
  W8_CHECK_ARG(a.t >= 0 && a.n >= 0, "negative size");
  if (a.t == 0) return W8_OK;
  W8_CHECK_ARG(a.n > 0 && a.n % 8 == 0 && a.n <= 32 * 8 * w8::kGlueMaxVecs,
               "row length %d must be a multiple of 8 and at most %d", a.n, 32 * 8 * w8::kGlueMaxVecs);
  W8_CHECK_ARG(a.x != nullptr && a.q != nullptr && a.s != nullptr, "null pointer");
  W8_CHECK_ALIGN(aligned(a.x, 16) && a.ldx % 8 == 0, "x must be 16-byte aligned with a pitch %% 8 == 0");
  W8_CHECK_ALIGN(aligned(a.q, 8) && a.ldq % 8 == 0 && a.ldq >= a.n, "q must be 8-byte aligned, ldq %% 8 == 0, ldq >= n");
  if (mode != w8::kGlueAttnOut) {
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
  const unsigned grid = static_cast<unsigned>((a.t + w8::kGlueWarps - 1) / w8::kGlueWarps);
  const unsigned threads = 32 * w8::kGlueWarps;
  switch (mode) {
    case w8::kGlueIn: w8::glue_rows_kernel<w8::kGlueIn><<<grid, threads, 0, stream>>>(a); break;
    case w8::kGluePost1: w8::glue_rows_kernel<w8::kGluePost1><<<grid, threads, 0, stream>>>(a); break;
    case w8::kGluePost2: w8::glue_rows_kernel<w8::kGluePost2><<<grid, threads, 0, stream>>>(a); break;
    default: w8::glue_rows_kernel<w8::kGlueAttnOut><<<grid, threads, 0, stream>>>(a); break;
  }
  return cuda_status(cudaGetLastError());
}

static w8::GlueArgs glue_args(int64_t t, int64_t n) {
  w8::GlueArgs a = {};
  a.t = static_cast<int>(t);
  a.n = static_cast<int>(n);
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
