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

// quant_one on the eight bf16 values of a 16-byte vector, two at a time: the division
// steps on packed f32x2 instructions (the same IEEE operations, so the same codes).
__device__ __forceinline__ void quant8_bf16(const uint4& v, float s, float r, int8_t (&out)[8]) {
  const uint64_t r2 = f2_pack(r, r), ns2 = f2_pack(-s, -s);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint64_t x2 = f2_from_bf16x2(w[j]);
    const uint64_t t2 = f2_mul(x2, r2);
    float q0, q1;
    f2_unpack(f2_fma(f2_fma(ns2, t2, x2), r2, t2), q0, q1);
    out[2 * j] = static_cast<int8_t>(static_cast<int>(fminf(fmaxf(rintf(q0), -127.f), 127.f)));
    out[2 * j + 1] = static_cast<int8_t>(static_cast<int>(fminf(fmaxf(rintf(q1), -127.f), 127.f)));
  }
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
