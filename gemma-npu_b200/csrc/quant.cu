// Per-row symmetric int8 quantisation and int32 -> bf16 dequantisation.
//
// quant: reference _quant (pipeline.py:49-52) / _quant_rows (gemma_npu.py:37-42) and the
// per-output-channel weight quant of NPUGemm (gemma_npu.py:68-69) and Int8Head
// (gemma_npu.py:165-166):
//     s = max(absmax(row), 1e-8) / 127          (fp32, IEEE divide)
//     q = clamp(round_half_even(x / s), -127, 127)
// Both divisions are correctly rounded (__fdiv_rn) and the rounding is rintf, so the
// output is bit-identical to torch's CPU result on the same fp32/bf16 input.
//
// dequant: reference _deq (pipeline.py:55-57) / _dequant (gemma_npu.py:45-47):
//     y = bf16((float(acc) * sx[row]) * sw[col])
//
// Both are HBM-bound streaming kernels: one CTA per row for quant (the row stays in
// registers between the absmax pass and the quantise pass), a grid-stride 16-byte
// vectorised loop for dequant.
#include "common.cuh"
#include <type_traits>

#include "rowquant.cuh"

namespace w8 {

constexpr int kQuantThreads = 128;
constexpr int kQuantMaxVecs = 8;  // vectors per thread kept in registers

template <typename T, int VEC>
__global__ void __launch_bounds__(kQuantThreads)
    quant_rows_kernel(const T* __restrict__ x, int64_t ldx, int8_t* __restrict__ q, int64_t ldq,
                      float* __restrict__ s, int m, int k) {
  __shared__ float red[kQuantThreads / 32];
  const int row = blockIdx.x;
  if (row >= m) return;
  const T* xr = x + static_cast<int64_t>(row) * ldx;
  int8_t* qr = q + static_cast<int64_t>(row) * ldq;
  const int nvec = k / VEC;

  constexpr bool kBf16x8 = std::is_same<T, __nv_bfloat16>::value && VEC == 8;
  Vec<T, VEC> held[kQuantMaxVecs];
  float amax = 0.f;
  uint32_t m2 = 0u;  // bf16 rows: two bf16 lanes of max |x|
#pragma unroll
  for (int i = 0; i < kQuantMaxVecs; ++i) {
    const int vi = threadIdx.x + i * kQuantThreads;
    if (vi < nvec) {
      held[i] = load_vec<T, VEC>(xr + static_cast<int64_t>(vi) * VEC);
      if constexpr (kBf16x8) {
        m2 = bf16x2_absmax8(*reinterpret_cast<const uint4*>(held[i].v), m2);
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) amax = fmaxf(amax, fabsf(to_f32(held[i].v[e])));
      }
    }
  }
  // Rows longer than the register window: stream the rest (read again in pass 2).
  for (int vi = threadIdx.x + kQuantMaxVecs * kQuantThreads; vi < nvec; vi += kQuantThreads) {
    const Vec<T, VEC> v = load_vec<T, VEC>(xr + static_cast<int64_t>(vi) * VEC);
    if constexpr (kBf16x8) {
      m2 = bf16x2_absmax8(*reinterpret_cast<const uint4*>(v.v), m2);
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) amax = fmaxf(amax, fabsf(to_f32(v.v[e])));
    }
  }
  if constexpr (kBf16x8) amax = bf16x2_max_lanes(m2);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int w = 1; w < kQuantThreads / 32; ++w) amax = fmaxf(amax, red[w]);
  const float sc = __fdiv_rn(fmaxf(amax, 1e-8f), 127.f);
  const float rc = __frcp_rn(sc);
  if (threadIdx.x == 0) s[row] = sc;

#pragma unroll
  for (int i = 0; i < kQuantMaxVecs; ++i) {
    const int vi = threadIdx.x + i * kQuantThreads;
    if (vi < nvec) {
      if constexpr (kBf16x8) {
        *reinterpret_cast<uint2*>(qr + static_cast<int64_t>(vi) * VEC) =
            quant8_bf16_codes(*reinterpret_cast<const uint4*>(held[i].v), sc, rc);
      } else {
        int8_t out[VEC];
#pragma unroll
        for (int e = 0; e < VEC; ++e) out[e] = quant_one(to_f32(held[i].v[e]), sc, rc);
        store_q<VEC>(qr + static_cast<int64_t>(vi) * VEC, out);
      }
    }
  }
  for (int vi = threadIdx.x + kQuantMaxVecs * kQuantThreads; vi < nvec; vi += kQuantThreads) {
    const Vec<T, VEC> v = load_vec<T, VEC>(xr + static_cast<int64_t>(vi) * VEC);
    if constexpr (kBf16x8) {
      *reinterpret_cast<uint2*>(qr + static_cast<int64_t>(vi) * VEC) =
          quant8_bf16_codes(*reinterpret_cast<const uint4*>(v.v), sc, rc);
    } else {
      int8_t out[VEC];
#pragma unroll
      for (int e = 0; e < VEC; ++e) out[e] = quant_one(to_f32(v.v[e]), sc, rc);
      store_q<VEC>(qr + static_cast<int64_t>(vi) * VEC, out);
    }
  }
}

// y = bf16((float(acc) * sx[row]) * sw[col]); 4 columns per thread step when aligned.
template <int VEC>
__global__ void __launch_bounds__(256)
    dequant_kernel(const int32_t* __restrict__ acc, int64_t ldacc, const float* __restrict__ sx,
                   const float* __restrict__ sw, __nv_bfloat16* __restrict__ y, int64_t ldy, int m,
                   int n) {
  const int64_t nv = n / VEC;
  const int64_t total = static_cast<int64_t>(m) * nv;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(i / nv);
    const int col = static_cast<int>(i - static_cast<int64_t>(row) * nv) * VEC;
    const float sr = __ldg(sx + row);
    const int32_t* a = acc + static_cast<int64_t>(row) * ldacc + col;
    __nv_bfloat16* o = y + static_cast<int64_t>(row) * ldy + col;
    if constexpr (VEC == 4) {
      const int4 v = __ldg(reinterpret_cast<const int4*>(a));
      const float4 w = __ldg(reinterpret_cast<const float4*>(sw + col));
      __nv_bfloat162 p0 = __floats2bfloat162_rn(__fmul_rn(__fmul_rn(__int2float_rn(v.x), sr), w.x),
                                                __fmul_rn(__fmul_rn(__int2float_rn(v.y), sr), w.y));
      __nv_bfloat162 p1 = __floats2bfloat162_rn(__fmul_rn(__fmul_rn(__int2float_rn(v.z), sr), w.z),
                                                __fmul_rn(__fmul_rn(__int2float_rn(v.w), sr), w.w));
      uint2 pk;
      pk.x = *reinterpret_cast<uint32_t*>(&p0);
      pk.y = *reinterpret_cast<uint32_t*>(&p1);
      *reinterpret_cast<uint2*>(o) = pk;
    } else {
      o[0] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(__int2float_rn(__ldg(a)), sr), __ldg(sw + col)));
    }
  }
}

// The quant half of the gate/up glue (pipeline.py:107, _quant of k_gelu's bf16 output)
// when the row absmax is already known: the fused GEMM epilogue folded it into
// absmax[row] (fp32 bits, atomicMax).  s = max(absmax, 1e-8) / 127 and q exactly as in
// quant_rows_kernel; absmax[row] is reset to zero for the next call.  One CTA per row,
// 8 bf16 per thread step (16-byte loads, 8-byte stores); the row's loads are issued
// before the absmax word is read, so the two latencies overlap.
__global__ void __launch_bounds__(kQuantThreads)
    quant_absmax_kernel(const __nv_bfloat16* __restrict__ y, int64_t ldy, float* __restrict__ absmax,
                        int8_t* __restrict__ q, int64_t ldq, float* __restrict__ s, int k) {
  const int row = blockIdx.x;
  const __nv_bfloat16* yr = y + static_cast<int64_t>(row) * ldy;
  int8_t* qr = q + static_cast<int64_t>(row) * ldq;
  const int nvec = k / 8;
  Vec<__nv_bfloat16, 8> held[kQuantMaxVecs];
#pragma unroll
  for (int i = 0; i < kQuantMaxVecs; ++i) {
    const int vi = threadIdx.x + i * kQuantThreads;
    if (vi < nvec) held[i] = load_vec<__nv_bfloat16, 8>(yr + vi * 8);
  }
  const float sc = __fdiv_rn(fmaxf(absmax[row], 1e-8f), 127.f);
  const float rc = __frcp_rn(sc);
  __syncthreads();  // every thread has read absmax[row]
  if (threadIdx.x == 0) {
    s[row] = sc;
    absmax[row] = 0.f;
  }
#pragma unroll
  for (int i = 0; i < kQuantMaxVecs; ++i) {
    const int vi = threadIdx.x + i * kQuantThreads;
    if (vi < nvec) {
      *reinterpret_cast<uint2*>(qr + vi * 8) = quant8_bf16_codes(*reinterpret_cast<const uint4*>(held[i].v), sc, rc);
    }
  }
  // Rows longer than the register window: the rest streams through.
  for (int vi = threadIdx.x + kQuantMaxVecs * kQuantThreads; vi < nvec; vi += kQuantThreads) {
    const Vec<__nv_bfloat16, 8> v = load_vec<__nv_bfloat16, 8>(yr + vi * 8);
    *reinterpret_cast<uint2*>(qr + vi * 8) = quant8_bf16_codes(*reinterpret_cast<const uint4*>(v.v), sc, rc);
  }
}

}  // namespace w8

namespace w8host {

int quant_rows_absmax_bf16(const uint16_t* y, int64_t ldy, float* absmax, int8_t* q, int64_t ldq, float* s,
                           int64_t m, int64_t k, cudaStream_t stream) {
  W8_CHECK_ARG(m >= 0 && k >= 0 && m < (1ll << 31) && k < (1ll << 31), "bad size");
  if (m == 0) return W8_OK;
  W8_CHECK_ARG(y != nullptr && absmax != nullptr && q != nullptr && s != nullptr, "null pointer");
  W8_CHECK_ARG(ldy >= k && ldq >= k, "row pitch smaller than k");
  W8_CHECK_ARG(k % 8 == 0, "k = %lld must be a multiple of 8", (long long)k);
  W8_CHECK_ALIGN(aligned(y, 16) && (ldy * 2) % 16 == 0, "y must be 16-byte aligned with a 16-byte row pitch");
  W8_CHECK_ALIGN(aligned(q, 8) && ldq % 8 == 0, "q must be 8-byte aligned with ldq %% 8 == 0");
  w8::quant_absmax_kernel<<<static_cast<unsigned>(m), w8::kQuantThreads, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(y), ldy, absmax, q, ldq, s, static_cast<int>(k));
  return cuda_status(cudaGetLastError());
}

int require_sm100(int* device);

template <typename T>
static int quant_rows(const T* x, int64_t ldx, int8_t* q, int64_t ldq, float* s, int64_t m,
                      int64_t k, cudaStream_t stream) {
  W8_CHECK_ARG(m >= 0 && k >= 0, "negative size");
  W8_CHECK_ARG(m < (1ll << 31) && k < (1ll << 31), "size beyond int32 range");
  if (m == 0) return W8_OK;
  W8_CHECK_ARG(x != nullptr && q != nullptr && s != nullptr, "null pointer");
  W8_CHECK_ARG(ldx >= k && ldq >= k, "row pitch smaller than k");
  int device = 0;
  const int st = require_sm100(&device);
  if (st != W8_OK) return st;
  constexpr int VEC = 16 / static_cast<int>(sizeof(T));
  const bool vec_ok = aligned(x, 16) && (ldx * sizeof(T)) % 16 == 0 && k % VEC == 0 &&
                      aligned(q, VEC) && ldq % VEC == 0;
  const dim3 grid(static_cast<unsigned>(m));
  if (vec_ok)
    w8::quant_rows_kernel<T, VEC><<<grid, w8::kQuantThreads, 0, stream>>>(
        x, ldx, q, ldq, s, static_cast<int>(m), static_cast<int>(k));
  else
    w8::quant_rows_kernel<T, 1><<<grid, w8::kQuantThreads, 0, stream>>>(
        x, ldx, q, ldq, s, static_cast<int>(m), static_cast<int>(k));
  return cuda_status(cudaGetLastError());
}

}  // namespace w8host

extern "C" int w8_quant_rows_bf16(const uint16_t* x, int64_t ldx, int8_t* q, int64_t ldq, float* s,
                                  int64_t m, int64_t k, w8_stream_t stream) {
  return w8host::quant_rows(reinterpret_cast<const __nv_bfloat16*>(x), ldx, q, ldq, s, m, k,
                            reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int w8_quant_rows_f32(const float* x, int64_t ldx, int8_t* q, int64_t ldq, float* s,
                                 int64_t m, int64_t k, w8_stream_t stream) {
  return w8host::quant_rows(x, ldx, q, ldq, s, m, k, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int w8_dequant_bf16(const int32_t* acc, int64_t ldacc, const float* sx, const float* sw,
                               uint16_t* y, int64_t ldy, int64_t m, int64_t n, w8_stream_t stream) {
  W8_CHECK_ARG(m >= 0 && n >= 0, "negative size");
  W8_CHECK_ARG(m < (1ll << 31) && n < (1ll << 31), "size beyond int32 range");
  if (m == 0 || n == 0) return W8_OK;
  W8_CHECK_ARG(acc != nullptr && sx != nullptr && sw != nullptr && y != nullptr, "null pointer");
  W8_CHECK_ARG(ldacc >= n && ldy >= n, "row pitch smaller than n");
  int device = 0;
  const int st = w8host::require_sm100(&device);
  if (st != W8_OK) return st;
  int sms = 0;
  const int st2 = w8host::num_sms(&sms);
  if (st2 != W8_OK) return st2;
  const bool vec_ok = w8host::aligned(acc, 16) && ldacc % 4 == 0 && w8host::aligned(sw, 16) &&
                      w8host::aligned(y, 8) && ldy % 4 == 0 && n % 4 == 0;
  const int64_t work = m * (vec_ok ? n / 4 : n);
  int64_t blocks = (work + 255) / 256;
  if (blocks > static_cast<int64_t>(sms) * 16) blocks = static_cast<int64_t>(sms) * 16;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  auto* out = reinterpret_cast<__nv_bfloat16*>(y);
  if (vec_ok)
    w8::dequant_kernel<4><<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        acc, ldacc, sx, sw, out, ldy, static_cast<int>(m), static_cast<int>(n));
  else
    w8::dequant_kernel<1><<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        acc, ldacc, sx, sw, out, ldy, static_cast<int>(m), static_cast<int>(n));
  return w8host::cuda_status(cudaGetLastError());
}
