// Row arithmetic shared by the weight-only int8 GEMV kernels (gemv.cu) and the
// column-sharded LM head with its peer-memory all-gather (lm_head_peer.cu): 16-byte
// non-allocating weight loads, the 16-bit fixed-point activation pieces, the dp4a dot
// products and the output rounding / softcap / greedy key of one row.
#pragma once

#include "common.cuh"

namespace w8 {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kGemvSmemCap = 96 * 1024;      // dynamic shared memory per CTA: at most 2 CTAs per SM
constexpr int kGemvSmemCapHead = 72 * 1024;  // the LM head: at most 3 CTAs per SM

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

}  // namespace w8
