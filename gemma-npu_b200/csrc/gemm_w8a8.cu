// W8A8 prefill GEMM for sm_100a: C = A @ B with int8 operands and int32 accumulation
// on the 5th-generation tensor cores (tcgen05.mma kind::i8).
//
// Reference behaviour replaced: matmul_i8_k / mm_i8 (npu_kernels.py:40-64) -- a
// 512x512-tile Triton GEMM over row-major int8 A [M,K], B [K,N] producing int32 C --
// and, in the bf16 variant, the _dequant that follows it (gemma_npu.py:45-47,149-150;
// pipeline.py:55-57).
//
// Structure (one persistent CTA per SM, 6 warps):
//   warp 0      TMA producer: A [128 x 128B] and B [BN x 128B] boxes into a STAGES-deep
//               ring of 128-byte-swizzled shared-memory stages (mbarrier full/empty).
//   warp 1      TMEM owner + MMA issuer: one thread issues 4 x tcgen05.mma (K = 32 each)
//               per stage into a double-buffered int32 accumulator in TMEM
//               (2 x BN columns), commits free the stage and publish finished tiles.
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (warp w owns TMEM lanes
//               32*(w%4)..+31 = tile rows), optional dequant, vector stores to HBM;
//               the buffer is handed back to the MMA warp so the epilogue of tile i
//               overlaps the main loop of tile i+1.
// B may be K-major ([N,K], the resident layout shared with the decode GEMV) or
// MN-major ([K,N], the reference's mm_i8 layout); the instruction descriptor's
// B-major bit and the shared-memory descriptor strides absorb the difference.
// Tails in M, N and K are handled by TMA zero fill (loads) and masked stores.
// No cluster launch and no multicast: every CTA issues its own TMA loads.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace w8 {

// Sticky device-side error word of the GEMM kernels (bounded-wait timeouts).
__device__ int g_gemm_status = 0;

constexpr int kBM = 128;      // tile rows = TMEM lanes
constexpr int kBK = 128;      // K elements (= bytes) per stage: one 128-byte swizzle row
constexpr int kUmmaK = 32;    // K of one tcgen05.mma kind::i8
constexpr int kEpiWarps = 4;
constexpr int kThreads = 64 + 32 * kEpiWarps;

enum EpiKind : int { kEpiI32 = 0, kEpiBf16 = 1 };

struct GemmArgs {
  int m, n, k;
  int m_tiles, n_tiles, k_blocks;
  void* out;
  int64_t ldo;
  const float* sx;
  const float* sw;
  int vec_out;  // output base 16-byte aligned and row pitch a multiple of 16 bytes
  int vec_sw;   // sw 16-byte aligned
  int tma_out;  // the output tensor map is valid: epilogue stores go through TMA
};

constexpr int kEpiBufBytes = 32 * 128;  // one 32-row x 128-byte store box
constexpr int kEpiBufs = 2;             // per epilogue warp: fill one while TMA drains the other

constexpr uint32_t tmem_cols_for(int c) {
  return c <= 32 ? 32u : c <= 64 ? 64u : c <= 128 ? 128u : c <= 256 ? 256u : 512u;
}

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int kA = kBM * kBK;
  static constexpr int kB = BN * kBK;
  static constexpr int kStage = kA + kB;
  static constexpr int kEpiOff = STAGES * kStage;  // epilogue store staging, 1024-aligned
  static constexpr int kBarOff = kEpiOff + kEpiWarps * kEpiBufs * kEpiBufBytes;
  static constexpr int kNumBars = 2 * STAGES + 5;  // full[S], empty[S], tfull[2], tempty[2], done
  static constexpr int kTotal = kBarOff + kNumBars * 8 + 16;
  static constexpr int kAlloc = kTotal + 1024;  // slack to align the ring to 1024 B
  static constexpr uint32_t kTmemCols = tmem_cols_for(2 * BN);
  static_assert(kAlloc <= 232448, "shared memory budget of one CTA exceeded");
};

template <int EPI>
__device__ __forceinline__ void store_chunk(const GemmArgs& a, int row, int col0,
                                            const uint32_t (&r)[32], float sxr) {
  if (row >= a.m) return;
  if constexpr (EPI == kEpiI32) {
    int32_t* dst = static_cast<int32_t*>(a.out) + static_cast<int64_t>(row) * a.ldo + col0;
    if (a.vec_out && col0 + 32 <= a.n) {
      int4* d4 = reinterpret_cast<int4*>(dst);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        d4[j] = make_int4(static_cast<int>(r[4 * j]), static_cast<int>(r[4 * j + 1]),
                          static_cast<int>(r[4 * j + 2]), static_cast<int>(r[4 * j + 3]));
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < a.n) dst[j] = static_cast<int>(r[j]);
    }
  } else {
    // (float(acc) * sx[row]) * sw[col], each product rounded to fp32, then RNE to bf16:
    // the operation order of _deq (pipeline.py:57).
    __nv_bfloat16* dst =
        static_cast<__nv_bfloat16*>(a.out) + static_cast<int64_t>(row) * a.ldo + col0;
    if (a.vec_out && a.vec_sw && col0 + 32 <= a.n) {
      const float4* sw4 = reinterpret_cast<const float4*>(a.sw + col0);
      uint32_t packed[16];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 w = __ldg(sw4 + j);
        const float v0 = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[4 * j + 0])), sxr), w.x);
        const float v1 = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[4 * j + 1])), sxr), w.y);
        const float v2 = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[4 * j + 2])), sxr), w.z);
        const float v3 = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[4 * j + 3])), sxr), w.w);
        __nv_bfloat162 p0 = __floats2bfloat162_rn(v0, v1);
        __nv_bfloat162 p1 = __floats2bfloat162_rn(v2, v3);
        packed[2 * j] = *reinterpret_cast<uint32_t*>(&p0);
        packed[2 * j + 1] = *reinterpret_cast<uint32_t*>(&p1);
      }
      int4* d4 = reinterpret_cast<int4*>(dst);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        d4[j] = make_int4(static_cast<int>(packed[4 * j]), static_cast<int>(packed[4 * j + 1]),
                          static_cast<int>(packed[4 * j + 2]), static_cast<int>(packed[4 * j + 3]));
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (col0 + j >= a.n) continue;
        const float v = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[j])), sxr),
                                  __ldg(a.sw + col0 + j));
        dst[j] = __float2bfloat16_rn(v);
      }
    }
  }
}

// 32 int32 accumulators of columns col0.. -> 16 words of packed bf16 pairs,
// bf16((float(acc) * sx[row]) * sw[col]) with _deq's operation order.
__device__ __forceinline__ void dequant_pack(const GemmArgs& a, int col0, const uint32_t (&r)[32],
                                             float sxr, uint32_t* out) {
  float w[32];
  if (a.vec_sw && col0 + 32 <= a.n) {
    const float4* sw4 = reinterpret_cast<const float4*>(a.sw + col0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 t = __ldg(sw4 + j);
      w[4 * j] = t.x;
      w[4 * j + 1] = t.y;
      w[4 * j + 2] = t.z;
      w[4 * j + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) w[j] = col0 + j < a.n ? __ldg(a.sw + col0 + j) : 0.f;
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float v0 = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[2 * j])), sxr), w[2 * j]);
    const float v1 = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[2 * j + 1])), sxr), w[2 * j + 1]);
    __nv_bfloat162 p = __floats2bfloat162_rn(v0, v1);
    out[j] = *reinterpret_cast<uint32_t*>(&p);
  }
}

template <int BN, int STAGES, bool B_MN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_w8a8_kernel(const __grid_constant__ CUtensorMap tm_a,
                     const __grid_constant__ CUtensorMap tm_b,
                     const __grid_constant__ CUtensorMap tm_c, const GemmArgs args) {
  using L = GemmSmem<BN, STAGES>;
  static_assert(!B_MN || BN % 128 == 0, "MN-major B is loaded in 128-column boxes");
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // swizzle atoms need 1024-byte alignment
  uint8_t* smem = smem_raw + (base - raw);
  const uint32_t bar0 = base + L::kBarOff;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kBarOff + L::kNumBars * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
  const uint32_t done_bar = bar0 + 8u * (2 * STAGES + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), kEpiWarps);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_b);
    if (args.tma_out) prefetch_tmap(&tm_c);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = args.m_tiles * args.n_tiles;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int stage = 0;
      uint32_t phase = 0, issued_mask = 0, last_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int mb = tile % args.m_tiles;
        const int nb = tile / args.m_tiles;
        for (int kb = 0; kb < args.k_blocks; ++kb) {
          if (!mbar_wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, &g_gemm_status)) {
            ok = false;
            break;
          }
          const uint32_t sa = base + stage * L::kStage;
          const uint32_t sb = sa + L::kA;
          mbar_arrive_expect_tx(full_bar(stage), L::kStage);
          tma_load_2d(sa, &tm_a, full_bar(stage), kb * kBK, mb * kBM);
          if constexpr (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 128; ++j)
              tma_load_2d(sb + j * 128 * kBK, &tm_b, full_bar(stage), nb * BN + j * 128, kb * kBK);
          } else {
            tma_load_2d(sb, &tm_b, full_bar(stage), kb * kBK, nb * BN);
          }
          issued_mask |= 1u << stage;
          last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Our copies still in flight must land before the CTA may exit.
      for (int s = 0; s < STAGES; ++s)
        if (issued_mask & (1u << s)) mbar_wait_bounded(full_bar(s), (last_phase >> s) & 1u, nullptr, &g_gemm_status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc = idesc_i8(kBM, BN, B_MN);
      int stage = 0, local = 0;
      uint32_t phase = 0;
      bool ok = true, issued = false;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_bounded(tempty_bar(acc), acc_phase ^ 1u, abort_flag, &g_gemm_status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        for (int kb = 0; kb < args.k_blocks; ++kb) {
          if (!mbar_wait_bounded(full_bar(stage), phase, abort_flag, &g_gemm_status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + stage * L::kStage;
          const uint32_t sb = sa + L::kA;
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            const uint64_t ad = smem_desc_sw128(sa + k * kUmmaK, 16, 1024);
            const uint64_t bd = B_MN ? smem_desc_sw128(sb + k * kUmmaK * 128, 128 * kBK, 1024)
                                     : smem_desc_sw128(sb + k * kUmmaK, 16, 1024);
            mma_i8(d, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          issued = true;
          mma_commit(empty_bar(stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(tfull_bar(acc));
      }
      // Every MMA this thread issued must retire before the TMEM is released.
      if (issued) {
        mma_commit(done_bar);
        mbar_wait_bounded(done_bar, 0, nullptr, &g_gemm_status);
      }
    }
  } else {
    // ---------------- epilogue
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    // This warp's two store-staging boxes (32 rows x 128 B, 128-byte swizzled like TMA).
    const uint32_t stage_base = base + L::kEpiOff + (warp - 2) * kEpiBufs * kEpiBufBytes;
    uint32_t sbuf = 0;  // running box counter: box parity selects the buffer
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      const bool ok = mbar_wait_bounded(tfull_bar(acc), acc_phase, abort_flag, &g_gemm_status);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const int mb = tile % args.m_tiles;
      const int nb = tile / args.m_tiles;
      const int row0 = mb * kBM + quarter * 32;
      const int row = row0 + lane;
      float sxr = 0.f;
      if constexpr (EPI == kEpiBf16) sxr = row < args.m ? __ldg(args.sx + row) : 0.f;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      const int n_cols = min(BN, args.n - nb * BN);  // columns of this tile inside N
      if (args.tma_out) {
        // One store box = 32 rows x 128 bytes: 32 int32 or 64 bf16 columns.
        constexpr int kCols = EPI == kEpiI32 ? 32 : 64;
        const int n_chunks = (n_cols + kCols - 1) / kCols;
#pragma unroll 1
        for (int c = 0; c < n_chunks; ++c) {
          uint32_t v[32];  // this thread's 128-byte slice of its row
          if constexpr (EPI == kEpiI32) {
            tmem_ld_32x32b_x32(taddr + c * 32, v);
            tmem_wait_ld();
          } else {
            uint32_t r0[32], r1[32];
            tmem_ld_32x32b_x32(taddr + c * 64, r0);
            tmem_ld_32x32b_x32(taddr + c * 64 + 32, r1);
            tmem_wait_ld();
            const int col0 = nb * BN + c * 64;
            dequant_pack(args, col0, r0, sxr, v);
            dequant_pack(args, col0 + 32, r1, sxr, v + 16);
          }
          if (c == n_chunks - 1) {  // the accumulator is in registers: hand TMEM back
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(acc));
          }
          const uint32_t buf = stage_base + (sbuf & 1u) * kEpiBufBytes;
          ++sbuf;
          if (lane == 0) bulk_wait_group_read<kEpiBufs - 1>();  // the box last stored from buf is read
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            st_shared_v4(buf + lane * 128 + ((j ^ (lane & 7)) << 4), v[4 * j], v[4 * j + 1], v[4 * j + 2],
                         v[4 * j + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tm_c, buf, nb * BN + c * kCols, row0);
            bulk_commit_group();
          }
        }
      } else {
        const int n_chunks = (n_cols + 31) / 32;
#pragma unroll 1
        for (int c = 0; c < n_chunks; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(taddr + c * 32, r);
          tmem_wait_ld();
          store_chunk<EPI>(args, row, nb * BN + c * 32, r, sxr);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty_bar(acc));
      }
    }
    if (lane == 0) bulk_wait_group<0>();  // every store of this warp has landed
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

}  // namespace w8

// =====================================================================================
// Host side
// =====================================================================================
namespace w8host {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D tensor [outer, inner] with row pitch `pitch` bytes, 128-byte swizzled boxes.
static int encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* ptr, int64_t inner,
                     int64_t outer, int64_t pitch, uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return W8_ERR_CUDA;
  }
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch)};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed with CUresult %d (inner %lld, outer %lld, pitch %lld)",
              static_cast<int>(r), static_cast<long long>(inner), static_cast<long long>(outer),
              static_cast<long long>(pitch));
    return W8_ERR_CUDA;
  }
  return W8_OK;
}

int require_sm100(int* device);

template <int BN, int STAGES, bool B_MN, int EPI>
static int launch_gemm(int device, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                       const w8::GemmArgs& args, cudaStream_t stream) {
  using L = w8::GemmSmem<BN, STAGES>;
  auto kern = w8::gemm_w8a8_kernel<BN, STAGES, B_MN, EPI>;
  static bool attr_done[64] = {};
  if (device < 0 || device >= 64) return W8_ERR_UNSUPPORTED;
  if (!attr_done[device]) {
    W8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc));
    attr_done[device] = true;
  }
  int sms = 0;
  const int st = num_sms(&sms);
  if (st != W8_OK) return st;
  const int tiles = args.m_tiles * args.n_tiles;
  const int grid = tiles < sms ? tiles : sms;
  kern<<<grid, w8::kThreads, L::kAlloc, stream>>>(ta, tb, tc, args);
  return cuda_status(cudaGetLastError());
}

static int gemm_common(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, int b_layout,
                       void* out, int64_t ldo, int out_elem, const float* sx, const float* sw,
                       int64_t m, int64_t n, int64_t k, cudaStream_t stream, int epi) {
  W8_CHECK_ARG(m >= 0 && n >= 0 && k >= 0, "negative size (m=%lld n=%lld k=%lld)", (long long)m,
               (long long)n, (long long)k);
  W8_CHECK_ARG(m < (1ll << 31) && n < (1ll << 31) && k < (1ll << 31), "size beyond int32 range");
  W8_CHECK_ARG(b_layout == W8_B_KN || b_layout == W8_B_NK, "b_layout must be W8_B_KN or W8_B_NK");
  if (m == 0 || n == 0) return W8_OK;
  W8_CHECK_ARG(out != nullptr, "null output pointer");
  W8_CHECK_ARG(ldo >= n, "output row pitch %lld < n %lld", (long long)ldo, (long long)n);
  W8_CHECK_ALIGN(aligned(out, out_elem), "output must be aligned to its element size");
  if (epi == w8::kEpiBf16) W8_CHECK_ARG(sx != nullptr && sw != nullptr, "null scale pointer");
  int device = 0;
  int st = require_sm100(&device);
  if (st != W8_OK) return st;
  if (k == 0) {
    // An empty contraction: the product is all zeros (and so is its dequant).
    W8_CUDA_TRY(cudaMemset2DAsync(out, ldo * out_elem, 0, n * out_elem, m, stream));
    return W8_OK;
  }
  W8_CHECK_ARG(a != nullptr && b != nullptr, "null operand pointer");
  W8_CHECK_ARG(k % 16 == 0, "k = %lld must be a multiple of 16", (long long)k);
  W8_CHECK_ARG(lda >= k, "lda %lld < k %lld", (long long)lda, (long long)k);
  W8_CHECK_ALIGN(aligned(a, 16) && lda % 16 == 0, "A must be 16-byte aligned with lda %% 16 == 0");
  W8_CHECK_ALIGN(aligned(b, 16) && ldb % 16 == 0, "B must be 16-byte aligned with ldb %% 16 == 0");
  if (b_layout == W8_B_KN)
    W8_CHECK_ARG(ldb >= n, "ldb %lld < n %lld for a [K,N] B", (long long)ldb, (long long)n);
  else
    W8_CHECK_ARG(ldb >= k, "ldb %lld < k %lld for an [N,K] B", (long long)ldb, (long long)k);

  constexpr int BN = 256;
  constexpr int STAGES = 4;
  CUtensorMap ta, tb, tc;
  st = encode_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, a, k, m, lda, w8::kBK, w8::kBM);
  if (st != W8_OK) return st;
  if (b_layout == W8_B_NK)
    st = encode_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, b, k, n, ldb, w8::kBK, BN);
  else
    st = encode_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, b, n, k, ldb, 128, w8::kBK);
  if (st != W8_OK) return st;

  w8::GemmArgs args;
  args.m = static_cast<int>(m);
  args.n = static_cast<int>(n);
  args.k = static_cast<int>(k);
  args.m_tiles = static_cast<int>((m + w8::kBM - 1) / w8::kBM);
  args.n_tiles = static_cast<int>((n + BN - 1) / BN);
  args.k_blocks = static_cast<int>((k + w8::kBK - 1) / w8::kBK);
  args.out = out;
  args.ldo = ldo;
  args.sx = sx;
  args.sw = sw;
  args.vec_out = aligned(out, 16) && (ldo * out_elem) % 16 == 0;
  args.vec_sw = sw != nullptr && aligned(sw, 16);
  // Output through TMA when the tensor map can address it (16-byte base and pitch);
  // one box is 32 rows x 128 bytes.  Otherwise the epilogue stores directly.
  memset(&tc, 0, sizeof(tc));
  args.tma_out = 0;
  if (args.vec_out) {
    const bool i32 = epi == w8::kEpiI32;
    st = encode_2d(&tc, i32 ? CU_TENSOR_MAP_DATA_TYPE_INT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, out, n, m,
                   ldo * out_elem, i32 ? 32 : 64, 32);
    if (st != W8_OK) return st;
    args.tma_out = 1;
  }

  const bool mn = b_layout == W8_B_KN;
  if (epi == w8::kEpiI32)
    return mn ? launch_gemm<BN, STAGES, true, w8::kEpiI32>(device, ta, tb, tc, args, stream)
              : launch_gemm<BN, STAGES, false, w8::kEpiI32>(device, ta, tb, tc, args, stream);
  return mn ? launch_gemm<BN, STAGES, true, w8::kEpiBf16>(device, ta, tb, tc, args, stream)
            : launch_gemm<BN, STAGES, false, w8::kEpiBf16>(device, ta, tb, tc, args, stream);
}

// Read (and optionally clear) the GEMM kernels' sticky device status.
int gemm_device_status(int clear, int* out) {
  int v = 0;
  W8_CUDA_TRY(cudaDeviceSynchronize());
  W8_CUDA_TRY(cudaMemcpyFromSymbol(&v, w8::g_gemm_status, sizeof(int)));
  if (clear) {
    const int zero = 0;
    W8_CUDA_TRY(cudaMemcpyToSymbol(w8::g_gemm_status, &zero, sizeof(int)));
  }
  *out = v;
  return W8_OK;
}

}  // namespace w8host

extern "C" int w8_mm_i8(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, int b_layout,
                        int32_t* c, int64_t ldc, int64_t m, int64_t n, int64_t k,
                        w8_stream_t stream) {
  return w8host::gemm_common(a, lda, b, ldb, b_layout, c, ldc, 4, nullptr, nullptr, m, n, k,
                             reinterpret_cast<cudaStream_t>(stream), w8::kEpiI32);
}

extern "C" int w8_gemm_dequant_bf16(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb,
                                    int b_layout, const float* sx, const float* sw, uint16_t* y,
                                    int64_t ldy, int64_t m, int64_t n, int64_t k,
                                    w8_stream_t stream) {
  return w8host::gemm_common(a, lda, b, ldb, b_layout, y, ldy, 2, sx, sw, m, n, k,
                             reinterpret_cast<cudaStream_t>(stream), w8::kEpiBf16);
}
