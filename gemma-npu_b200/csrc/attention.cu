// Prefill attention of one prompt (pipeline.py:139-180: full_attention and
// sliding_attention with q_start = 0), bf16 in and out, fp32 softmax and accumulation.
//
//   o[h, i, :] = sum_j p_ij v[h / G, j, :],  p_i = softmax_j(q[h, i, :] . k[h / G, j, :])
//
// over the keys j <= i, and with a window W > 0 only i - j < W (sliding_attention's mask);
// scale 1.0 (Gemma's q_norm / k_norm take its place), G = H / KV query heads per KV head.
// q, k, v, o are head-major [heads, T, D] as the k_qkv glue writes them.
//
// Flash-attention schedule with warp-level bf16 tensor-core MMAs (mma.sync m16n8k16):
// a CTA of 4 warps owns 64 queries of one head and 256 output columns; each warp owns 16
// query rows.  Per 64-key tile: S = Q K^T (fragments from swizzled shared memory with
// ldmatrix), online softmax in registers (log2 domain, exp2), O += P V with P reused from
// the S accumulators as the A operand.  Key tiles outside the causal / window range are
// skipped; the boundary tiles are masked.  D = 512 (full-attention layers) runs two
// groups of 4 warps, one per 256-column half of O, sharing one S through shared memory.
#include "common.cuh"

namespace w8 {

constexpr int kAttnWarps = 4;
constexpr int kAttnBM = 16 * kAttnWarps;  // queries per CTA
constexpr int kAttnBN = 64;               // keys per tile
constexpr int kAttnDO = 256;              // output columns per CTA

struct AttnArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  __nv_bfloat16* o;
  int64_t q_head, q_tok, k_head, k_tok, v_head, v_tok, o_head, o_tok;  // pitches in elements
  int t, heads, kv_heads, window;
};

// Row r of a [rows, D] bf16 tile at `base`: 16-byte chunk c stored at chunk c ^ (r & 7).
template <int D>
__device__ __forceinline__ uint32_t tile_addr(uint32_t base, int r, int chunk) {
  return base + r * (D * 2) + ((chunk ^ (r & 7)) << 4);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// rows x D bf16 from global (row pitch `pitch`, rows >= `valid_rows` zero-filled) into a
// swizzled tile; columns [c0, c0 + D) of the source.
template <int D, int ROWS, int PARTS>
__device__ __forceinline__ void load_tile(uint32_t base, const __nv_bfloat16* src, int64_t pitch, int valid_rows,
                                          int c0) {
  constexpr int kChunks = ROWS * D / 8;
  for (int i = threadIdx.x; i < kChunks; i += 32 * kAttnWarps * PARTS) {
    const int r = i / (D / 8), c = i % (D / 8);
    const bool ok = r < valid_rows;
    const __nv_bfloat16* p = src + (ok ? static_cast<int64_t>(r) * pitch : 0) + c0 + c * 8;
    cp_async16(tile_addr<D>(base, r, c), p, ok);
  }
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}
__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// PARTS = D / 256 warp groups of 4 warps; group gi owns output columns [256 gi, 256 gi + 256)
// of the CTA's 64 queries.  Group 0 computes S and the softmax; with two groups it hands P
// (bf16) and the per-row rescale factors over through shared memory, so S is computed
// once for D = 512.
template <int D>
__global__ void __launch_bounds__(32 * kAttnWarps * (D / kAttnDO)) attention_kernel(const AttnArgs a) {
  constexpr int PARTS = D / kAttnDO;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sq = smem_u32(smem);
  const uint32_t sk = sq + kAttnBM * D * 2;
  const uint32_t sv = sk + kAttnBN * D * 2;
  const uint32_t sp = sv + kAttnBN * D * 2;  // P [64 queries x 64 keys] bf16 (PARTS > 1)
  float* stat = reinterpret_cast<float*>(smem + (kAttnBM + 2 * kAttnBN) * D * 2 + kAttnBM * kAttnBN * 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wg = warp / kAttnWarps, wr = warp % kAttnWarps;  // warp group, warp within it
  // Heaviest query tiles (most keys under the causal mask) are scheduled first.
  const int q0 = (gridDim.x - 1 - blockIdx.x) * kAttnBM;
  const int head = blockIdx.y;
  const int c0 = wg * kAttnDO;  // this group's output columns
  const int kvh = head / (a.heads / a.kv_heads);
  const __nv_bfloat16* qh = a.q + head * a.q_head + static_cast<int64_t>(q0) * a.q_tok;
  const __nv_bfloat16* kh = a.k + kvh * a.k_head;
  const __nv_bfloat16* vh = a.v + kvh * a.v_head;

  load_tile<D, kAttnBM, PARTS>(sq, qh, a.q_tok, a.t - q0, 0);

  const int g = lane >> 2, qd = lane & 3;  // mma fragment row group / column pair
  const int lr_a = wr * 16 + g, lr_b = lr_a + 8;  // rows within the CTA's 64
  const int row_a = q0 + lr_a, row_b = q0 + lr_b;
  float o[kAttnDO / 8][4];
#pragma unroll
  for (int j = 0; j < kAttnDO / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  constexpr float kLog2e = 1.4426950408889634f;

  const int last_key = min(q0 + kAttnBM, a.t) - 1;
  const int first_key = a.window > 0 ? max(0, q0 - a.window + 1) : 0;
  for (int kt = first_key / kAttnBN; kt * kAttnBN <= last_key; ++kt) {
    const int k0 = kt * kAttnBN;
    __syncthreads();  // the previous tile's K / V / P are consumed
    load_tile<D, kAttnBN, PARTS>(sk, kh + static_cast<int64_t>(k0) * a.k_tok, a.k_tok, a.t - k0, 0);
    load_tile<D, kAttnBN, PARTS>(sv, vh + static_cast<int64_t>(k0) * a.v_tok, a.v_tok, a.t - k0, 0);
    cp_async_wait_all();
    __syncthreads();

    uint32_t p[kAttnBN / 8][2];
    float corr_a = 1.f, corr_b = 1.f;
    if (wg == 0) {
      // S = Q K^T for this warp's 16 rows x 64 keys.
      float s[kAttnBN / 8][4];
#pragma unroll
      for (int j = 0; j < kAttnBN / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll 4
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t af[4];
        ldsm_x4(tile_addr<D>(sq, wr * 16 + (lane & 7) + 8 * ((lane >> 3) & 1), 2 * kk + (lane >> 4)), af);
#pragma unroll
        for (int jj = 0; jj < kAttnBN / 16; ++jj) {
          uint32_t bf[4];
          ldsm_x4(tile_addr<D>(sk, jj * 16 + (lane & 7) + 8 * (lane >> 4), 2 * kk + ((lane >> 3) & 1)), bf);
          mma_bf16(s[2 * jj], af, bf[0], bf[1]);
          mma_bf16(s[2 * jj + 1], af, bf[2], bf[3]);
        }
      }
      // Mask (causal, window, keys past T), then the online softmax in the log2 domain.
      float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
      for (int j = 0; j < kAttnBN / 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = k0 + j * 8 + 2 * qd + (e & 1);
          const int row = e < 2 ? row_a : row_b;
          float v = s[j][e] * kLog2e;
          if (key > row || key >= a.t || (a.window > 0 && row - key >= a.window)) v = -INFINITY;
          s[j][e] = v;
          if (e < 2) mx_a = fmaxf(mx_a, v); else mx_b = fmaxf(mx_b, v);
        }
#pragma unroll
      for (int sh = 1; sh <= 2; sh <<= 1) {
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, sh));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, sh));
      }
      const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
      const float ref_a = mn_a == -INFINITY ? 0.f : mn_a, ref_b = mn_b == -INFINITY ? 0.f : mn_b;
      corr_a = exp2_approx(m_a - ref_a);
      corr_b = exp2_approx(m_b - ref_b);
      m_a = mn_a;
      m_b = mn_b;
      float sum_a = 0.f, sum_b = 0.f;
#pragma unroll
      for (int j = 0; j < kAttnBN / 8; ++j) {
        const float p0 = exp2_approx(s[j][0] - ref_a), p1 = exp2_approx(s[j][1] - ref_a);
        const float p2 = exp2_approx(s[j][2] - ref_b), p3 = exp2_approx(s[j][3] - ref_b);
        sum_a += p0 + p1;
        sum_b += p2 + p3;
        p[j][0] = pack_bf16(p0, p1);
        p[j][1] = pack_bf16(p2, p3);
      }
      l_a = l_a * corr_a + sum_a;
      l_b = l_b * corr_b + sum_b;
      if constexpr (PARTS > 1) {
        // Hand P and the rescale factors to the other group(s): P[row][key] in a
        // swizzled [64 x 64] bf16 tile (the A operand layout ldmatrix reads below).
#pragma unroll
        for (int j = 0; j < kAttnBN / 8; ++j) {
          const uint32_t col_bytes = (j * 8 + 2 * qd) * 2;
          asm volatile("st.shared.b32 [%0], %1;" ::"r"(tile_addr<kAttnBN>(sp, lr_a, j) + (col_bytes & 15)),
                       "r"(p[j][0]));
          asm volatile("st.shared.b32 [%0], %1;" ::"r"(tile_addr<kAttnBN>(sp, lr_b, j) + (col_bytes & 15)),
                       "r"(p[j][1]));
        }
        if (qd == 0) {
          stat[lr_a] = corr_a;
          stat[lr_b] = corr_b;
        }
      }
    }
    if constexpr (PARTS > 1) {
      __syncthreads();  // P and the factors are in shared memory
      if (wg != 0) {
        corr_a = stat[lr_a];
        corr_b = stat[lr_b];
      }
    }
#pragma unroll
    for (int j = 0; j < kAttnDO / 8; ++j) {
      o[j][0] *= corr_a;
      o[j][1] *= corr_a;
      o[j][2] *= corr_b;
      o[j][3] *= corr_b;
    }
    // O += P V over this group's 256 columns.
#pragma unroll
    for (int kk = 0; kk < kAttnBN / 16; ++kk) {
      uint32_t af[4];
      if constexpr (PARTS == 1) {
        af[0] = p[2 * kk][0];
        af[1] = p[2 * kk][1];
        af[2] = p[2 * kk + 1][0];
        af[3] = p[2 * kk + 1][1];
      } else {
        ldsm_x4(tile_addr<kAttnBN>(sp, wr * 16 + (lane & 7) + 8 * ((lane >> 3) & 1), 2 * kk + (lane >> 4)), af);
      }
#pragma unroll
      for (int jj = 0; jj < kAttnDO / 16; ++jj) {
        uint32_t bf[4];
        ldsm_x4_t(tile_addr<D>(sv, kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1), c0 / 8 + 2 * jj + (lane >> 4)), bf);
        mma_bf16(o[2 * jj], af, bf[0], bf[1]);
        mma_bf16(o[2 * jj + 1], af, bf[2], bf[3]);
      }
    }
  }
  // Row sums live spread over group 0's quads: reduce, share, normalise, store bf16.
#pragma unroll
  for (int sh = 1; sh <= 2; sh <<= 1) {
    l_a += __shfl_xor_sync(0xffffffffu, l_a, sh);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, sh);
  }
  if constexpr (PARTS > 1) {
    __syncthreads();
    if (wg == 0 && qd == 0) {
      stat[kAttnBM + lr_a] = l_a;
      stat[kAttnBM + lr_b] = l_b;
    }
    __syncthreads();
    l_a = stat[kAttnBM + lr_a];
    l_b = stat[kAttnBM + lr_b];
  }
  const float inv_a = l_a > 0.f ? 1.f / l_a : 0.f, inv_b = l_b > 0.f ? 1.f / l_b : 0.f;
  __nv_bfloat16* oh = a.o + head * a.o_head + c0;
#pragma unroll
  for (int j = 0; j < kAttnDO / 8; ++j) {
    const int col = j * 8 + 2 * qd;
    if (row_a < a.t)
      *reinterpret_cast<uint32_t*>(oh + static_cast<int64_t>(row_a) * a.o_tok + col) =
          pack_bf16(o[j][0] * inv_a, o[j][1] * inv_a);
    if (row_b < a.t)
      *reinterpret_cast<uint32_t*>(oh + static_cast<int64_t>(row_b) * a.o_tok + col) =
          pack_bf16(o[j][2] * inv_b, o[j][3] * inv_b);
  }
}

}  // namespace w8

namespace w8host {

int require_sm100(int* device);

template <int D>
static int attention_go(const w8::AttnArgs& a, cudaStream_t stream) {
  constexpr int smem = (w8::kAttnBM + 2 * w8::kAttnBN) * D * 2 + w8::kAttnBM * w8::kAttnBN * 2 + 2 * w8::kAttnBM * 4;
  auto kern = w8::attention_kernel<D>;
  static bool done[64] = {};
  int device = 0;
  W8_CUDA_TRY(cudaGetDevice(&device));
  if (device < 0 || device >= 64) return W8_ERR_UNSUPPORTED;
  if (!done[device]) {
    W8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    done[device] = true;
  }
  const dim3 grid(static_cast<unsigned>((a.t + w8::kAttnBM - 1) / w8::kAttnBM), static_cast<unsigned>(a.heads), 1);
  kern<<<grid, 32 * w8::kAttnWarps * (D / w8::kAttnDO), smem, stream>>>(a);
  return cuda_status(cudaGetLastError());
}

}  // namespace w8host

namespace w8host {

int attention_tc(const uint16_t* q, int64_t q_head, int64_t q_tok, const uint16_t* k, int64_t k_head,
                 int64_t k_tok, const uint16_t* v, int64_t v_head, int64_t v_tok, uint16_t* o, int64_t o_head,
                 int64_t o_tok, int64_t t, int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t window,
                 int device, cudaStream_t stream);
bool attention_tc_quant_fits(int64_t heads, int64_t kv_heads, int64_t head_dim);
int attention_tc_quant(const uint16_t* q, int64_t q_head, int64_t q_tok, const uint16_t* k, int64_t k_head,
                       int64_t k_tok, const uint16_t* v, int64_t v_head, int64_t v_tok, int64_t t, int64_t heads,
                       int64_t kv_heads, int64_t window, int8_t* xq, int64_t ldq, float* xs, int device,
                       cudaStream_t stream);

// Argument checks shared by both schedules, then the tcgen05 one (tc) or the mma.sync one.
static int attention_entry(const uint16_t* q, int64_t q_head, int64_t q_tok, const uint16_t* k, int64_t k_head,
                           int64_t k_tok, const uint16_t* v, int64_t v_head, int64_t v_tok, uint16_t* o,
                           int64_t o_head, int64_t o_tok, int64_t t, int64_t heads, int64_t kv_heads,
                           int64_t head_dim, int64_t window, w8_stream_t stream, bool tc) {
  W8_CHECK_ARG(t >= 0 && t < (1ll << 31) && heads >= 0 && kv_heads >= 0 && window >= 0, "bad size");
  if (t == 0 || heads == 0) return W8_OK;
  W8_CHECK_ARG(head_dim == 256 || head_dim == 512, "head_dim = %lld must be 256 or 512", (long long)head_dim);
  W8_CHECK_ARG(kv_heads > 0 && heads % kv_heads == 0, "heads (%lld) must be a multiple of kv_heads (%lld)",
               (long long)heads, (long long)kv_heads);
  W8_CHECK_ARG(heads < 65536, "too many heads");
  W8_CHECK_ARG(q != nullptr && k != nullptr && v != nullptr && o != nullptr, "null pointer");
  W8_CHECK_ALIGN(aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(o, 16) && q_head % 8 == 0 &&
                     q_tok % 8 == 0 && k_head % 8 == 0 && k_tok % 8 == 0 && v_head % 8 == 0 && v_tok % 8 == 0 &&
                     o_head % 8 == 0 && o_tok % 8 == 0,
                 "q, k, v, o must be 16-byte aligned with pitches %% 8 == 0");
  W8_CHECK_ARG(q_tok >= head_dim && k_tok >= head_dim && v_tok >= head_dim && o_tok >= head_dim,
               "token pitch smaller than head_dim");
  int device = 0;
  const int st = require_sm100(&device);
  if (st != W8_OK) return st;
  if (tc)
    return attention_tc(q, q_head, q_tok, k, k_head, k_tok, v, v_head, v_tok, o, o_head, o_tok, t, heads, kv_heads,
                        head_dim, window, device, reinterpret_cast<cudaStream_t>(stream));
  w8::AttnArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.k = reinterpret_cast<const __nv_bfloat16*>(k);
  a.v = reinterpret_cast<const __nv_bfloat16*>(v);
  a.o = reinterpret_cast<__nv_bfloat16*>(o);
  a.q_head = q_head, a.q_tok = q_tok, a.k_head = k_head, a.k_tok = k_tok;
  a.v_head = v_head, a.v_tok = v_tok, a.o_head = o_head, a.o_tok = o_tok;
  a.t = static_cast<int>(t);
  a.heads = static_cast<int>(heads);
  a.kv_heads = static_cast<int>(kv_heads);
  a.window = static_cast<int>(window);
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return head_dim == 256 ? attention_go<256>(a, s) : attention_go<512>(a, s);
}

}  // namespace w8host

extern "C" int w8_attention_prefill_bf16(const uint16_t* q, int64_t q_head, int64_t q_tok, const uint16_t* k,
                                         int64_t k_head, int64_t k_tok, const uint16_t* v, int64_t v_head,
                                         int64_t v_tok, uint16_t* o, int64_t o_head, int64_t o_tok, int64_t t,
                                         int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t window,
                                         w8_stream_t stream) {
  return w8host::attention_entry(q, q_head, q_tok, k, k_head, k_tok, v, v_head, v_tok, o, o_head, o_tok, t, heads,
                                 kv_heads, head_dim, window, stream, true);
}

extern "C" int w8_attention_prefill_mma_bf16(const uint16_t* q, int64_t q_head, int64_t q_tok, const uint16_t* k,
                                             int64_t k_head, int64_t k_tok, const uint16_t* v, int64_t v_head,
                                             int64_t v_tok, uint16_t* o, int64_t o_head, int64_t o_tok, int64_t t,
                                             int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t window,
                                             w8_stream_t stream) {
  return w8host::attention_entry(q, q_head, q_tok, k, k_head, k_tok, v, v_head, v_tok, o, o_head, o_tok, t, heads,
                                 kv_heads, head_dim, window, stream, false);
}

extern "C" int w8_attention_prefill_quant(const uint16_t* q, int64_t q_head, int64_t q_tok, const uint16_t* k,
                                          int64_t k_head, int64_t k_tok, const uint16_t* v, int64_t v_head,
                                          int64_t v_tok, int64_t t, int64_t heads, int64_t kv_heads,
                                          int64_t head_dim, int64_t window, int8_t* xq, int64_t ldq, float* xs,
                                          w8_stream_t stream) {
  using namespace w8host;
  W8_CHECK_ARG(t >= 0 && t < (1ll << 31) && heads >= 0 && kv_heads >= 0 && window >= 0, "bad size");
  if (t == 0 || heads == 0) return W8_OK;
  if (!attention_tc_quant_fits(heads, kv_heads, head_dim)) {
    set_error("the fused attention + k_attn_out takes head_dim 256, one KV head and a power-of-two head count "
              "<= 16 (got head_dim %lld, heads %lld, kv_heads %lld)",
              (long long)head_dim, (long long)heads, (long long)kv_heads);
    return W8_ERR_UNSUPPORTED;
  }
  W8_CHECK_ARG(q != nullptr && k != nullptr && v != nullptr && xq != nullptr && xs != nullptr, "null pointer");
  W8_CHECK_ALIGN(aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && q_head % 8 == 0 && q_tok % 8 == 0 &&
                     k_head % 8 == 0 && k_tok % 8 == 0 && v_head % 8 == 0 && v_tok % 8 == 0,
                 "q, k, v must be 16-byte aligned with pitches %% 8 == 0");
  W8_CHECK_ALIGN(aligned(xq, 16) && ldq % 16 == 0 && aligned(xs, 4), "xq must be 16-byte aligned, ldq %% 16 == 0");
  W8_CHECK_ARG(q_tok >= head_dim && k_tok >= head_dim && v_tok >= head_dim && ldq >= heads * head_dim,
               "pitch too small");
  int device = 0;
  const int st = require_sm100(&device);
  if (st != W8_OK) return st;
  return attention_tc_quant(q, q_head, q_tok, k, k_head, k_tok, v, v_head, v_tok, t, heads, kv_heads, window, xq,
                            ldq, xs, device, reinterpret_cast<cudaStream_t>(stream));
}
