// Row-quant building blocks shared by the quant kernels and the glue kernels: bf16/fp32
// element access, 16-byte vectors, the correctly rounded division by a row scale and the
// int8 code of _quant (pipeline.py:49-52).
#pragma once

#include "common.cuh"

namespace w8 {

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

// x / s correctly rounded, from r = RN(1/s) (one IEEE reciprocal per row): the product
// t = RN(x * r) is within one ulp of x / s, the residual x - s * t is exact in one FMA,
// and one more FMA t + r * residual rounds to RN(x / s) (P. Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1),
// 1990; no over- or underflow here: s >= 1e-8 / 127 and |x / s| <= 127).
__device__ __forceinline__ float div_rn_by(float x, float s, float r) {
  const float t = __fmul_rn(x, r);
  return __fmaf_rn(__fmaf_rn(-s, t, x), r, t);
}

__device__ __forceinline__ int8_t quant_one(float v, float s, float r) {
  float q = rintf(div_rn_by(v, s, r));
  q = fminf(fmaxf(q, -127.f), 127.f);
  return static_cast<int8_t>(static_cast<int>(q));
}

// quant_one of the eight bf16 values of a 16-byte vector, packed little-endian in two
// words.  The division steps run two values at a time on packed f32x2 instructions (the
// same IEEE operations), and rint(q) is taken from RN(q + 1.5 * 2^23): |x| <= absmax and
// s = RN(max(absmax, 1e-8) / 127) bound |q| by 127 plus one ulp, so the sum lies in
// [2^23, 2^24), where the fp32 grid is the integers; its rounding is rint's (nearest, ties
// to even), the clamp to +-127 never binds, and the low byte of its bits is the code in
// two's complement.  Byte permutes gather the four low bytes of a word.
__device__ __forceinline__ uint2 quant8_bf16_codes(const uint4& v, float s, float r) {
  const uint64_t r2 = f2_pack(r, r), ns2 = f2_pack(-s, -s);
  const uint64_t magic2 = f2_pack(12582912.f, 12582912.f);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t b[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint64_t x2 = f2_from_bf16x2(w[j]);
    const uint64_t t2 = f2_mul(x2, r2);
    float lo, hi;
    f2_unpack(f2_add(f2_fma(f2_fma(ns2, t2, x2), r2, t2), magic2), lo, hi);
    b[2 * j] = __float_as_uint(lo);
    b[2 * j + 1] = __float_as_uint(hi);
  }
  return make_uint2(__byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410),
                    __byte_perm(__byte_perm(b[4], b[5], 0x0040), __byte_perm(b[6], b[7], 0x0040), 0x5410));
}

// max |x| over eight packed bf16 values folded into `m2` (two bf16 lanes, sign bits
// cleared); fmaxf(lo, hi) of the result is the fp32 absmax.  The bf16 max is exact.
__device__ __forceinline__ uint32_t bf16x2_absmax8(const uint4& v, uint32_t m2) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) asm("max.bf16x2 %0, %0, %1;" : "+r"(m2) : "r"(w[j] & 0x7FFF7FFFu));
  return m2;
}
__device__ __forceinline__ float bf16x2_max_lanes(uint32_t m2) {
  return fmaxf(__uint_as_float(m2 << 16), __uint_as_float(m2 & 0xFFFF0000u));
}

// VEC elements of T per 16-byte vector (VEC == 1: unaligned scalar path).
template <typename T, int VEC>
struct alignas(VEC * sizeof(T) >= 16 ? 16 : alignof(T)) Vec {
  T v[VEC];
};

template <typename T, int VEC>
__device__ __forceinline__ Vec<T, VEC> load_vec(const T* p) {
  Vec<T, VEC> r;
  if constexpr (VEC * sizeof(T) == 16) {
    *reinterpret_cast<uint4*>(r.v) = __ldg(reinterpret_cast<const uint4*>(p));
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) r.v[i] = p[i];
  }
  return r;
}

__device__ __forceinline__ uint32_t pack4(const int8_t* q) {
  return static_cast<uint32_t>(static_cast<uint8_t>(q[0])) |
         (static_cast<uint32_t>(static_cast<uint8_t>(q[1])) << 8) |
         (static_cast<uint32_t>(static_cast<uint8_t>(q[2])) << 16) |
         (static_cast<uint32_t>(static_cast<uint8_t>(q[3])) << 24);
}

template <int VEC>
__device__ __forceinline__ void store_q(int8_t* p, const int8_t (&q)[VEC]) {
  if constexpr (VEC == 8) {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack4(q), pack4(q + 4));
  } else if constexpr (VEC == 4) {
    *reinterpret_cast<uint32_t*>(p) = pack4(q);
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) p[i] = q[i];
  }
}

}  // namespace w8
