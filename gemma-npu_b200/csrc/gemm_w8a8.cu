// W8A8 prefill GEMM for sm_100a: C = A @ B with int8 operands and int32 accumulation
// on the 5th-generation tensor cores (tcgen05.mma kind::i8).
//
// Reference behaviour replaced: matmul_i8_k / mm_i8 (npu_kernels.py:40-64) -- a
// 512x512-tile Triton GEMM over row-major int8 A [M,K], B [K,N] producing int32 C --
// and, in the bf16 variant, the _dequant that follows it (gemma_npu.py:45-47,149-150;
// pipeline.py:55-57).
//
// Two persistent, warp-specialised kernels (6 warps per CTA, one CTA per SM):
//
//   gemm_pair_kernel  (M > 128) a cluster of two CTAs on two SMs computes 256 x 256
//       tiles with tcgen05.mma.cta_group::2: each CTA stages its 128 rows of A and its
//       128 columns of B (K-blocks of 128 bytes, 128-byte swizzle, 6-stage ring) and
//       holds its 128 output rows in its own TMEM.  Per SM this halves the B operand
//       traffic of a 128 x 256 tile.
//   gemm_single_kernel (M <= 128) one CTA computes 128 x 256 tiles (cta_group::1,
//       4-stage ring), so a short prompt does not waste half of every pair.
//
// Roles in both: warp 0 issues the TMA loads; warp 1 owns TMEM and one of its threads
// issues the MMAs (in the pair kernel only the even CTA's) into a double-buffered
// int32 accumulator (2 x 256 TMEM columns); warps 2..5 are the epilogue: tcgen05.ld of
// the accumulator (warp w owns TMEM lanes 32*(w%4)..+31), optional dequant, staging in
// 128-byte-swizzled shared memory and TMA bulk tensor stores of 32-row x 128-byte
// boxes.  The accumulator is handed back as soon as it is in registers, so the
// epilogue of tile i overlaps the main loop of tile i+1.
//
// Work schedule ("workers" = CTA pairs or CTAs, as many as are co-resident):
//   data-parallel  worker w computes whole tiles w, w + W, w + 2W, ...
//   stream-K       (int32 output, when whole tiles would leave a ragged last wave)
//                  the (tile, K-block) units are cut into W equal contiguous ranges;
//                  a tile split between workers is finished exactly: the worker that
//                  owns its last K-block (the first thing that worker computes) stores
//                  its partial sum, and every other contributor adds its partial into C
//                  with a TMA reduce-add once a per-tile counter in the caller's
//                  workspace says the store has landed.  The last contributor resets
//                  the counter, so the workspace is all-zero again after every launch
//                  (and every replay of a captured graph).  int32 addition is exact
//                  and order-independent: the result is bit-identical to one pass.
//
// B may be K-major ([N,K], the resident layout shared with the decode GEMV) or
// MN-major ([K,N], the reference's mm_i8 layout); the instruction descriptor's B-major
// bit and the shared-memory descriptor strides absorb the difference.  Tails in M, N
// and K are handled by TMA zero fill (loads) and TMA clipping (stores).  Every CTA
// issues its own TMA loads into its own shared memory; no load is shared across the
// cluster.  Every wait is bounded (see common.cuh); all workers are co-resident, so a
// stream-K wait always ends.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace w8 {

// Sticky device-side error word of the GEMM kernels (bounded-wait timeouts).
__device__ int g_gemm_status = 0;

// Fault injection for the tests of the bounded stream-K wait (w8_inject_stream_k_stall):
// while g_sk_drop_signal is set, the owner of a split tile's last K-block stores its
// partial sum but never signals, so the other contributors' wait runs out after
// g_sk_wait_limit_ns (0: the default kWaitTimeoutNs).  Both are zero unless a test sets them.
__device__ int g_sk_drop_signal = 0;
__device__ unsigned long long g_sk_wait_limit_ns = 0;

constexpr int kBM = 128;      // rows per CTA = TMEM lanes
constexpr int kBN = 256;      // columns per tile = accumulator columns
constexpr int kBK = 128;      // K elements (= bytes) per stage: one 128-byte swizzle row
constexpr int kUmmaK = 32;    // K of one tcgen05.mma kind::i8
constexpr int kEpiWarps = 4;
constexpr uint32_t kTmemCols = 2 * kBN;  // two accumulators of 256 int32 columns

// kEpiI32: int32 accumulators.  kEpiBf16: _deq to bf16.  kEpiGeluUp: the gate/up glue
// k_gelu (pipeline.py:102-107) up to its quant: bf16(gelu_tanh(gate) * up) of the
// dequantised halves of each 256-column tile (packed weights: tile t holds gate rows
// 128t.. and up rows I + 128t..), 128 bf16 outputs per tile row, plus the row absmax.
// kEpiQkv: the qkv glue k_qkv (pipeline.py:72-86) for head_dim 256, one head per
// 256-column tile: dequant, the head's RMSNorm (q_norm / k_norm weight, none for v) and,
// for q and k heads, RoPE, stored head-major [heads, T, 256] as bf16.
enum EpiKind : int { kEpiI32 = 0, kEpiBf16 = 1, kEpiGeluUp = 2, kEpiQkv = 3 };

struct GemmArgs {
  int m, n, k;
  int m_tiles, n_tiles, k_blocks;
  void* out;
  int64_t ldo;
  const float* sx;
  const float* sw;
  int vec_out;       // output base 16-byte aligned and row pitch a multiple of 16 bytes
  int vec_sw;        // sw 16-byte aligned
  int tma_out;       // the output tensor map is valid: epilogue stores go through TMA
  int stream_k;      // 1: stream-K schedule (int32 + TMA output + flags only)
  uint32_t* flags;   // stream-K: one zero-initialised counter per tile
  int bn;            // output columns per tile: 256, or 192 on CTA pairs when it balances waves
  float* row_absmax; // kEpiGeluUp: per-row max |output| (fp32 bits, atomicMax), zero on entry
  // kEpiQkv: heads [0, q_heads) are q, [q_heads, q_heads + k_heads) k, the rest v.
  const __nv_bfloat16* cos;  // [T, >= 256] row pitch ldcs
  const __nv_bfloat16* sin;
  int64_t ldcs;   // [T, D] tables: the row pitch; 8-column tiled tables: the pitch of a tile
  int cs_tiled;   // cos / sin as [D / 8][T][8] (each token's 8 columns of a tile contiguous)
  const __nv_bfloat16* qw;   // q_norm weight [256]
  const __nv_bfloat16* kw;   // k_norm weight [256]
  float eps;
  int q_heads, k_heads;
};

constexpr int kEpiBufBytes = 32 * 128;  // one 32-row x 128-byte store box
constexpr int kEpiBufs = 2;             // per epilogue warp: fill one while TMA drains the other

// Epilogue warps of a CTA: one per TMEM lane quarter, each with two staging boxes.  The
// gate/up glue, whose per-element math outweighs its stores, takes four warps per quarter
// (each finishes 32 of the tile's 128 output columns, one 32-row x 64-byte box) with one
// staging box each: the same shared memory, four times the warps to hide the latency of
// the math (with two warps per quarter it waited on its own dependences, not on a unit).
constexpr int kGeluWarpsPerQuarter = 4;
constexpr int kGeluBufBytes = 32 * 64;
// The qkv glue: two warps per lane quarter (each finishes half of the head's RoPE column
// pairs), each with two 32-row x 64-byte staging boxes.
constexpr int kQkvWarpsPerQuarter = 2;
constexpr int kQkvBufs = 2;
constexpr int kQkvBufBytes = 32 * 64;
template <int EPI>
constexpr int epi_warps() {
  return EPI == kEpiGeluUp ? kGeluWarpsPerQuarter * kEpiWarps
                           : (EPI == kEpiQkv ? kQkvWarpsPerQuarter * kEpiWarps : kEpiWarps);
}
template <int EPI>
constexpr int epi_bufs() { return EPI == kEpiGeluUp ? 1 : (EPI == kEpiQkv ? kQkvBufs : kEpiBufs); }
template <int EPI>
constexpr int epi_buf_bytes() {
  return EPI == kEpiGeluUp ? kGeluBufBytes : (EPI == kEpiQkv ? kQkvBufBytes : kEpiBufBytes);
}
template <int EPI>
constexpr int threads_for() { return 64 + 32 * epi_warps<EPI>(); }
static_assert(kGeluWarpsPerQuarter * kEpiWarps * kGeluBufBytes == kEpiWarps * kEpiBufs * kEpiBufBytes,
              "staging layout differs");
static_assert(kQkvWarpsPerQuarter * kEpiWarps * kQkvBufs * kQkvBufBytes == kEpiWarps * kEpiBufs * kEpiBufBytes,
              "staging layout differs");

// Shared-memory plan of one CTA: the operand ring, the epilogue staging boxes, barriers.
template <int STAGES, int A_BYTES, int B_BYTES>
struct Smem {
  static constexpr int kA = A_BYTES;
  static constexpr int kStage = A_BYTES + B_BYTES;
  static constexpr int kEpiOff = STAGES * kStage;  // 1024-aligned
  static constexpr int kBarOff = kEpiOff + kEpiWarps * kEpiBufs * kEpiBufBytes;
  static constexpr int kNumBars = 2 * STAGES + 5;  // full[S], empty[S], tfull[2], tempty[2], done
  static constexpr int kTotal = kBarOff + kNumBars * 8 + 16;
  static constexpr int kAlloc = kTotal + 1024;  // slack to align the ring to 1024 B
  static_assert(kStage % 1024 == 0, "stages must keep 1024-byte alignment");
  static_assert(kAlloc <= 232448, "shared memory budget of one CTA exceeded");
};
// CTA pairs stage 256 K bytes at a time (two swizzle chunks per copy): the TMA engine of
// an SM moves large boxes far faster than small ones (measured on B200 with one CTA per
// SM streaming from L2: 28 B/clk with 16 KB boxes, 56 B/clk with 32 KB boxes), and the
// MMAs of a 128-row CTA consume about 50 B/clk at full rate.
constexpr int kPairBK = 256;
constexpr int kPairChunks = kPairBK / kBK;
constexpr int kPairStages = 3;
constexpr int kSingleStages = 4;
using PairSmem = Smem<kPairStages, kBM * kPairBK, 128 * kPairBK>;  // A half + B half per CTA
using SingleSmem = Smem<kSingleStages, kBM * kBK, kBN * kBK>;  // A + whole B tile

// ---------------------------------------------------------------- schedule
struct Segment {
  int tile, kb0, kb1;  // K-blocks [kb0, kb1) of one output tile
  int contributors;    // workers that contribute to this tile (1 = whole tile here)
};

// The segments one worker computes, in order; every role of the worker walks the same list.
struct Schedule {
  int64_t u, u_end, units;  // stream-K cursor over (tile, K-block) units
  int tile, workers;        // data-parallel cursor
  bool sk;

  __device__ Schedule(const GemmArgs& a, int worker, int nworkers) {
    sk = a.stream_k != 0;
    workers = nworkers;
    units = static_cast<int64_t>(a.m_tiles) * a.n_tiles * a.k_blocks;
    u = units * worker / nworkers;
    u_end = units * (worker + 1) / nworkers;
    tile = worker;
  }
  // Worker that owns unit x (the largest w with floor(w * units / workers) <= x).
  __device__ int owner(int64_t x) const { return static_cast<int>(((x + 1) * workers - 1) / units); }

  __device__ bool next(const GemmArgs& a, Segment& s) {
    if (!sk) {
      if (tile >= a.m_tiles * a.n_tiles) return false;
      s.tile = tile;
      s.kb0 = 0;
      s.kb1 = a.k_blocks;
      s.contributors = 1;
      tile += workers;
      return true;
    }
    if (u >= u_end) return false;
    s.tile = static_cast<int>(u / a.k_blocks);
    s.kb0 = static_cast<int>(u - static_cast<int64_t>(s.tile) * a.k_blocks);
    const int64_t left = u_end - u;
    s.kb1 = left < a.k_blocks - s.kb0 ? s.kb0 + static_cast<int>(left) : a.k_blocks;
    u += s.kb1 - s.kb0;
    const int64_t first = static_cast<int64_t>(s.tile) * a.k_blocks;
    s.contributors = owner(first + a.k_blocks - 1) - owner(first) + 1;
    return true;
  }
};

// ---------------------------------------------------------------- epilogue
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
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (col0 + j >= a.n) continue;
      const float v = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[j])), sxr),
                                __ldg(a.sw + col0 + j));
      dst[j] = __float2bfloat16_rn(v);
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
  const uint64_t sx2 = f2_pack(sxr, sxr);
#pragma unroll
  for (int j = 0; j < 16; ++j) {  // two columns per packed f32x2 multiply
    const uint64_t a = f2_pack(__int2float_rn(static_cast<int>(r[2 * j])), __int2float_rn(static_cast<int>(r[2 * j + 1])));
    float v0, v1;
    f2_unpack(f2_mul(f2_mul(a, sx2), f2_pack(w[2 * j], w[2 * j + 1])), v0, v1);
    __nv_bfloat162 p = __floats2bfloat162_rn(v0, v1);
    out[j] = *reinterpret_cast<uint32_t*>(&p);
  }
}

// The weight scales of 16 gate columns (GEMM columns gcol0..) and of the 16 up columns
// 128 columns to their right.
__device__ __forceinline__ void gelu_up_scales16(const GemmArgs& a, int gcol0, float (&wg)[16], float (&wu)[16]) {
  if (a.vec_sw) {
    const float4* g4 = reinterpret_cast<const float4*>(a.sw + gcol0);
    const float4* u4 = reinterpret_cast<const float4*>(a.sw + gcol0 + 128);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 t = __ldg(g4 + j), v = __ldg(u4 + j);
      wg[4 * j] = t.x, wg[4 * j + 1] = t.y, wg[4 * j + 2] = t.z, wg[4 * j + 3] = t.w;
      wu[4 * j] = v.x, wu[4 * j + 1] = v.y, wu[4 * j + 2] = v.z, wu[4 * j + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      wg[j] = __ldg(a.sw + gcol0 + j);
      wu[j] = __ldg(a.sw + gcol0 + 128 + j);
    }
  }
}

// 16 gate and 16 up accumulators with their scales -> 8 words of packed bf16
// a = bf16(gelu(_deq(gate)) * _deq(up)); `amax2` accumulates max |a| in two bf16 lanes.
// Two columns at a time on packed f32x2 instructions, in gelu_tanh_bf16's operation
// order; the product of the two bf16 factors is one packed bf16 multiply.
__device__ __forceinline__ void gelu_up_pack16(const uint32_t (&rg)[16], const uint32_t (&ru)[16],
                                               const float (&wg)[16], const float (&wu)[16], float sxr,
                                               uint32_t* out, uint32_t& amax2) {
  const uint64_t sx2 = f2_pack(sxr, sxr);
  const uint64_t kappa2 = f2_pack(kGeluKappa, kGeluKappa), beta2 = f2_pack(kGeluBeta, kGeluBeta);
  const uint64_t m2l2e2 = f2_pack(-2.8853900817779268f, -2.8853900817779268f);  // -2 log2(e)
  const uint64_t one2 = f2_pack(1.f, 1.f), two2 = f2_pack(2.f, 2.f), half2 = f2_pack(0.5f, 0.5f);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int c = 2 * j;
    uint32_t bits;
    const uint64_t gi = f2_pack(__int2float_rn(static_cast<int>(rg[c])), __int2float_rn(static_cast<int>(rg[c + 1])));
    const uint64_t ui = f2_pack(__int2float_rn(static_cast<int>(ru[c])), __int2float_rn(static_cast<int>(ru[c + 1])));
    const uint64_t g = f2_round_bf16(f2_mul(f2_mul(gi, sx2), f2_pack(wg[c], wg[c + 1])), bits);
    const uint32_t ub = bf16x2_from_f2(f2_mul(f2_mul(ui, sx2), f2_pack(wu[c], wu[c + 1])));
    // gelu_tanh_bf16 on both: 1 + tanh(z) = 2 / (1 + e^(-2z)).
    const uint64_t g3 = f2_mul(f2_mul(g, g), g);
    const uint64_t inner = f2_mul(beta2, f2_add(g, f2_mul(kappa2, g3)));
    float a0, a1;
    f2_unpack(f2_mul(inner, m2l2e2), a0, a1);
    float e0, e1;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(a0));
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(a1));
    float d0, d1, r0, r1;
    f2_unpack(f2_add(one2, f2_pack(e0, e1)), d0, d1);
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(d0));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(d1));
    const uint32_t gb = bf16x2_from_f2(f2_mul(f2_mul(half2, g), f2_mul(two2, f2_pack(r0, r1))));
    out[j] = bf16x2_mul(gb, ub);
    asm("max.bf16x2 %0, %0, %1;" : "+r"(amax2) : "r"(out[j] & 0x7FFF7FFFu));
  }
}

// Stage one 32-row x 128-byte box in this warp's swizzled buffer and store it with TMA
// (or add it, for a stream-K partial) at column x, row row0.
template <int BUFS>
__device__ __forceinline__ void put_box(const CUtensorMap* tm_c, const uint32_t (&v)[32], uint32_t stage_base,
                                       uint32_t& sbuf, int lane, int x, int row0, bool reduce) {
  const uint32_t buf = stage_base + (sbuf & (BUFS - 1u)) * kEpiBufBytes;
  ++sbuf;
  if (lane == 0) bulk_wait_group_read<BUFS - 1>();  // the box last stored from buf is read
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 8; ++j)
    st_shared_v4(buf + lane * 128 + ((j ^ (lane & 7)) << 4), v[4 * j], v[4 * j + 1], v[4 * j + 2],
                 v[4 * j + 3]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (reduce)
      tma_reduce_add_2d(tm_c, buf, x, row0);
    else
      tma_store_2d(tm_c, buf, x, row0);
    bulk_commit_group();
  }
}

// Stage one 32-row x 64-byte box (32 bf16 columns, row = lane, no swizzle) in this warp's
// buffer and store it with TMA at column x, row row0.
__device__ __forceinline__ void put_box64(const CUtensorMap* tm_c, const uint32_t (&v)[16], uint32_t buf,
                                          int lane, int x, int row0) {
  if (lane == 0) bulk_wait_group_read<0>();  // the previous box stored from buf is read
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 4; ++j) st_shared_v4(buf + lane * 64 + j * 16, v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tm_c, buf, x, row0);
    bulk_commit_group();
  }
}

// Stage one 32-row x 64-byte box (32 bf16 columns, row = lane, no swizzle) in one of this
// warp's two buffers and store it with TMA into a 3-D [heads, T, D] output at (x, row0, z).
__device__ __forceinline__ void put_box64_3d(const CUtensorMap* tm_c, const uint32_t (&v)[16], uint32_t stage_base,
                                             uint32_t& sbuf, int lane, int x, int row0, int z) {
  const uint32_t buf = stage_base + (sbuf & 1u) * kQkvBufBytes;
  ++sbuf;
  if (lane == 0) bulk_wait_group_read<1>();  // the box last stored from buf is read
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 4; ++j) st_shared_v4(buf + lane * 64 + j * 16, v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_3d(tm_c, buf, x, row0, z);
    bulk_commit_group();
  }
}

// 16 words of bf16 pairs: columns c0 .. c0 + 31 (c0 % 8 == 0) of token `row` of an
// 8-column tiled table [D / 8][T][8] whose tiles lie `pitch` elements apart, or zeros for a
// row past M.  The 32 lanes (32 consecutive tokens) of a warp read 512 contiguous bytes
// per load.
__device__ __forceinline__ void load_row32_tiled(const __nv_bfloat16* base, int64_t pitch, int row, int c0, bool valid,
                                                 uint32_t (&out)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 v = valid ? __ldg(reinterpret_cast<const uint4*>(base + ((c0 >> 3) + j) * pitch + static_cast<int64_t>(row) * 8))
                          : make_uint4(0u, 0u, 0u, 0u);
    out[4 * j] = v.x, out[4 * j + 1] = v.y, out[4 * j + 2] = v.z, out[4 * j + 3] = v.w;
  }
}

// 16 words of bf16 pairs (32 consecutive columns of one row) from global memory, or zeros
// for a row past M.
__device__ __forceinline__ void load_row32_bf16(const __nv_bfloat16* p, bool valid, uint32_t (&out)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 v = valid ? __ldg(reinterpret_cast<const uint4*>(p) + j) : make_uint4(0u, 0u, 0u, 0u);
    out[4 * j] = v.x, out[4 * j + 1] = v.y, out[4 * j + 2] = v.z, out[4 * j + 3] = v.w;
  }
}

// k_qkv for one head (256 columns) of this thread's row (pipeline.py:72-86), the operation
// order of the row kernel w8_qkv_norm_rope_bf16, so the output bits are the same:
//   pass 1: y = _deq(acc) (bf16); 32 partial sums of y^2 over 8 consecutive columns,
//           combined in the row kernel's lane-then-xor-tree order; r = rsqrt(sum/256 + eps)
//   pass 2: x = bf16(y * r * w) (v heads: bf16(y * r)); q / k heads:
//           out = bf16(bf16(x * cos) + bf16(rotate_half(x) * sin)) on packed bf16 pairs.
// `part` (0 or 1) picks the RoPE column pairs (c, c + 128) this warp finishes:
// c in [64 part, 64 part + 64).
template <typename Release>
__device__ __forceinline__ void qkv_epilogue_rows(const GemmArgs& args, const CUtensorMap* tm_c, uint32_t taddr,
                                                  int row0, int col_base, float sxr, uint32_t stage_base,
                                                  uint32_t& sbuf, int lane, int part, Release release) {
  const int head = col_base >> 8;
  const int row = row0 + lane;
  const bool valid = row < args.m;
  // ---- pass 1: the row's sum of squares of the dequantised bf16 values
  float ps[32];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint32_t r[32], y[16];
    tmem_ld_32x32b_x32(taddr + c * 32, r);
    tmem_wait_ld();
    dequant_pack(args, col_base + c * 32, r, sxr, y);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      float acc = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float lo = __uint_as_float(y[4 * g + e] << 16), hi = __uint_as_float(y[4 * g + e] & 0xFFFF0000u);
        acc = __fmaf_rn(lo, lo, acc);
        acc = __fmaf_rn(hi, hi, acc);
      }
      ps[4 * c + g] = acc;
    }
  }
  // A warp's xor-butterfly sum, as lane 0 of the row kernel forms it (v + shfl_xor(v, o)
  // for o = 16, 8, 4, 2, 1; addition is commutative, so every lane holds these bits).
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int i = 0; i < o; ++i) ps[i] = __fadd_rn(ps[i], ps[i + o]);
  const float rn = __frsqrt_rn(__fadd_rn(__fdiv_rn(ps[0], 256.f), args.eps));
  const uint64_t r2 = f2_pack(rn, rn);
  const bool is_q = head < args.q_heads;
  const bool is_k = !is_q && head < args.q_heads + args.k_heads;
  const __nv_bfloat16* wnorm = is_q ? args.qw : (is_k ? args.kw : nullptr);
  const __nv_bfloat16* crow = args.cos + (args.cs_tiled ? 0 : static_cast<int64_t>(row) * args.ldcs);
  const __nv_bfloat16* srow = args.sin + (args.cs_tiled ? 0 : static_cast<int64_t>(row) * args.ldcs);
  // ---- pass 2: this warp's column pairs (c, c + 128), 32 columns at a time
#pragma unroll 1
  for (int cc = 0; cc < 2; ++cc) {
    const int c0 = part * 64 + cc * 32;  // first half: columns c0..c0+31; second: c0+128..
    uint32_t ra[32], rb[32], xa[16], xb[16];
    tmem_ld_32x32b_x32(taddr + c0, ra);
    tmem_ld_32x32b_x32(taddr + 128 + c0, rb);
    tmem_wait_ld();
    if (cc == 1) {  // this warp's columns are in registers: hand TMEM back
      tc_fence_before();
      __syncwarp();
      if (lane == 0) release();
    }
    dequant_pack(args, col_base + c0, ra, sxr, xa);
    dequant_pack(args, col_base + 128 + c0, rb, sxr, xb);
    if (wnorm != nullptr) {
      uint32_t wa[16], wb[16];
      load_row32_bf16(wnorm + c0, true, wa);
      load_row32_bf16(wnorm + 128 + c0, true, wb);
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        xa[q] = bf16x2_from_f2(f2_mul(f2_mul(f2_from_bf16x2(xa[q]), r2), f2_from_bf16x2(wa[q])));
        xb[q] = bf16x2_from_f2(f2_mul(f2_mul(f2_from_bf16x2(xb[q]), r2), f2_from_bf16x2(wb[q])));
      }
    } else {
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        xa[q] = bf16x2_from_f2(f2_mul(f2_from_bf16x2(xa[q]), r2));
        xb[q] = bf16x2_from_f2(f2_mul(f2_from_bf16x2(xb[q]), r2));
      }
    }
    if (wnorm != nullptr) {  // q and k heads: RoPE with rotate_half's partner c <-> c + 128
      uint32_t ca[16], cb[16], sa[16], sb[16];
      if (args.cs_tiled) {
        load_row32_tiled(args.cos, args.ldcs, row, c0, valid, ca);
        load_row32_tiled(args.cos, args.ldcs, row, 128 + c0, valid, cb);
        load_row32_tiled(args.sin, args.ldcs, row, c0, valid, sa);
        load_row32_tiled(args.sin, args.ldcs, row, 128 + c0, valid, sb);
      } else {
        load_row32_bf16(crow + c0, valid, ca);
        load_row32_bf16(crow + 128 + c0, valid, cb);
        load_row32_bf16(srow + c0, valid, sa);
        load_row32_bf16(srow + 128 + c0, valid, sb);
      }
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const uint32_t oa = bf16x2_add(bf16x2_mul(xa[q], ca[q]), bf16x2_mul(xb[q] ^ 0x80008000u, sa[q]));
        const uint32_t ob = bf16x2_add(bf16x2_mul(xb[q], cb[q]), bf16x2_mul(xa[q], sb[q]));
        xa[q] = oa;
        xb[q] = ob;
      }
    }
    put_box64_3d(tm_c, xa, stage_base, sbuf, lane, c0, row0, head);
    put_box64_3d(tm_c, xb, stage_base, sbuf, lane, 128 + c0, row0, head);
  }
}

// Drain one 32-row slice of a finished accumulator (called by one whole epilogue warp).
// `taddr` addresses the warp's TMEM lanes at the accumulator's first column; rows
// row0.. and columns col_base.. of the output.  `release` hands the accumulator back to
// the MMA issuer once its last columns are in registers.  With `reduce`, the boxes are
// added into C (TMA reduce-add) instead of stored.
template <int EPI, typename Release>
__device__ __forceinline__ void epilogue_rows(const GemmArgs& args, const CUtensorMap* tm_c,
                                              uint32_t taddr, int row0, int col_base, float sxr,
                                              uint32_t stage_base, uint32_t& sbuf, int lane,
                                              bool reduce, int part, Release release) {
  const int n_cols = min(args.bn, args.n - col_base);  // columns of this tile inside N
  const int row = row0 + lane;
  if constexpr (EPI == kEpiQkv) {
    qkv_epilogue_rows(args, tm_c, taddr, row0, col_base, sxr, stage_base, sbuf, lane, part, release);
    return;
  }
  if constexpr (EPI == kEpiGeluUp) {
    // 256 accumulator columns = 128 gate + 128 up -> output columns col_base / 2 ..+128;
    // this warp (`part` of the four of its lane quarter) finishes output columns
    // 32 part .. 32 part + 31 of its 32 rows, 16 at a time.
    uint32_t amax2 = 0u;  // max |a| in two bf16 lanes
    {
      uint32_t v[16];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = part * 32 + h * 16;
        uint32_t rg[16], ru[16];
        tmem_ld_32x32b_x16(taddr + c, rg);
        tmem_ld_32x32b_x16(taddr + 128 + c, ru);
        tmem_wait_ld();
        float wg[16], wu[16];
        gelu_up_scales16(args, col_base + c, wg, wu);
        if (h == 1) {  // this warp's columns are in registers: hand TMEM back
          tc_fence_before();
          __syncwarp();
          if (lane == 0) release();
        }
        gelu_up_pack16(rg, ru, wg, wu, sxr, v + h * 8, amax2);
      }
      (void)sbuf;
      put_box64(tm_c, v, stage_base, lane, col_base / 2 + part * 32, row0);
    }
    const float amax = fmaxf(__uint_as_float(amax2 << 16), __uint_as_float(amax2 & 0xFFFF0000u));
    if (row < args.m) atomicMax(reinterpret_cast<int*>(args.row_absmax) + row, __float_as_int(amax));
    return;
  }
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
        const int col0 = col_base + c * 64;
        dequant_pack(args, col0, r0, sxr, v);
        dequant_pack(args, col0 + 32, r1, sxr, v + 16);
      }
      if (c == n_chunks - 1) {  // the accumulator is in registers: hand TMEM back
        tc_fence_before();
        __syncwarp();
        if (lane == 0) release();
      }
      put_box<epi_bufs<EPI>()>(tm_c, v, stage_base, sbuf, lane, col_base + c * kCols, row0, reduce);
    }
  } else {
    const int n_chunks = (n_cols + 31) / 32;
#pragma unroll 1
    for (int c = 0; c < n_chunks; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(taddr + c * 32, r);
      tmem_wait_ld();
      store_chunk<EPI>(args, row, col_base + c * 32, r, sxr);
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) release();
  }
}

// One epilogue warp's part of a segment: for a stream-K tile split between workers,
// the owner of the last K-block stores and signals; the others wait, then add.
// `warps_per_contrib` epilogue warps make up one contributor.
template <int EPI, typename Release>
__device__ __forceinline__ void epilogue_segment(const GemmArgs& args, const CUtensorMap* tm_c,
                                                 const Segment& s, uint32_t taddr, int row0,
                                                 int col_base, float sxr, uint32_t stage_base,
                                                 uint32_t& sbuf, int lane, int warps_per_contrib,
                                                 int part, Release release) {
  const bool split = s.contributors > 1;
  const bool tail = s.kb1 == args.k_blocks;  // owns the tile's last K-block: stores first
  uint32_t* flag = split ? args.flags + s.tile : nullptr;
  if (split && !tail) {
    bool ok = true;
    if (lane == 0) {
      const unsigned long long limit = g_sk_wait_limit_ns ? g_sk_wait_limit_ns : kWaitTimeoutNs;
      ok = wait_counter_bounded(flag, static_cast<uint32_t>(warps_per_contrib), &g_gemm_status, limit);
      fence_proxy_async_global();
    }
    __syncwarp();
    (void)ok;  // on a timeout the sum is wrong and the status says so; the launch still ends
  }
  epilogue_rows<EPI>(args, tm_c, taddr, row0, col_base, sxr, stage_base, sbuf, lane, split && !tail,
                     part, release);
  if (split && lane == 0) {
    bulk_wait_group<0>();  // this warp's boxes have landed in C
    __threadfence();
    const uint32_t total = static_cast<uint32_t>(warps_per_contrib * s.contributors);
    if (!(tail && g_sk_drop_signal))
      if (atomicAdd(flag, 1u) == total - 1) atomicExch(flag, 0u);  // last one: reset for the next launch
  }
  __syncwarp();
}

// =====================================================================================
// 256 x BN tiles on a CTA pair (tcgen05 cta_group::2); BN = 256 or 192 (args.bn == BN).
// BN is a template parameter so the MMA instruction descriptor is a compile-time constant.
// =====================================================================================
template <bool B_MN, int EPI, int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(threads_for<EPI>(), 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                     const __grid_constant__ CUtensorMap tm_c, const GemmArgs args) {
  static_assert(BN % 64 == 0 && BN <= kBN, "tile width must be a multiple of 64 up to 256");
  using L = PairSmem;
  constexpr int STAGES = kPairStages;
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
  const uint32_t rank = cluster_ctarank();  // 0 = the CTA that issues the MMAs
  const uint32_t peer = rank ^ 1u;
  pdl_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);   // leader: one arrive.expect_tx + both CTAs' TMA bytes
      mbar_init(empty_bar(s), 1);  // both: one MMA commit
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);               // both: one MMA commit
      mbar_init(tempty_bar(a), 2 * epi_warps<EPI>());  // leader: the epilogue warps of both CTAs
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_b);
    if (args.tma_out) prefetch_tmap(&tm_c);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  pdl_wait();  // the previous kernel's writes (our A, B) are visible from here on
  const uint32_t tmem_base = *tmem_slot;
  const int worker = blockIdx.x >> 1;
  const int workers = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs): this CTA's A rows and B columns
      // Bytes both CTAs land on the leader's full barrier per stage: A halves + B halves.
      constexpr uint32_t stage_tx = 2u * (L::kA + (BN / 2) * kPairBK);
      Schedule sched(args, worker, workers);
      Segment sg;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      while (ok && sched.next(args, sg)) {
        const int mb = sg.tile % args.m_tiles;
        const int nb = sg.tile / args.m_tiles;
        const int a_row = mb * 2 * kBM + static_cast<int>(rank) * kBM;
        const int b_col = nb * BN + static_cast<int>(rank) * (BN / 2);
        for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
          if (!mbar_wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, &g_gemm_status)) {
            ok = false;
            break;
          }
          const uint32_t sa = base + stage * L::kStage;
          const uint32_t sb = sa + L::kA;
          const uint32_t fb = mapa_shared(full_bar(stage), 0);  // the leader's full barrier
          if (rank == 0) mbar_arrive_expect_tx(full_bar(stage), stage_tx);
          tma_load_3d_pair(sa, &tm_a, fb, 0, a_row, kb * kPairChunks);
          if constexpr (B_MN)
            tma_load_2d_pair(sb, &tm_b, fb, b_col, kb * kPairBK);
          else
            tma_load_3d_pair(sb, &tm_b, fb, 0, b_col, kb * kPairChunks);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Every copy issued here was consumed by the leader's MMA (it waited on the full
      // barrier that counts both CTAs' bytes) unless a wait gave up; either way the
      // closing cluster barrier keeps both CTAs resident until the end.
    }
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      // ---------------- MMA issuer (leader CTA only)
      constexpr uint32_t idesc = idesc_i8(2 * kBM, BN, B_MN);
      const int k_chunks = args.k / kBK;  // K is a multiple of 128 on CTA pairs
      const uint32_t empty_peer0 = mapa_shared(empty_bar(0), peer);
      const uint32_t tfull_peer0 = mapa_shared(tfull_bar(0), peer);
      Schedule sched(args, worker, workers);
      Segment sg;
      int stage = 0, local = 0;
      uint32_t phase = 0;
      bool ok = true, issued = false;
      while (ok && sched.next(args, sg)) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        ++local;
        if (!mbar_wait_bounded(tempty_bar(acc), acc_phase ^ 1u, abort_flag, &g_gemm_status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * kBN;
        for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
          if (!mbar_wait_bounded(full_bar(stage), phase, abort_flag, &g_gemm_status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + stage * L::kStage;
          const uint32_t sb = sa + L::kA;
          // The second chunk of the last stage may lie beyond K (odd K / 128): skip it.
          const int chunks = min(kPairChunks, k_chunks - kb * kPairChunks);
#pragma unroll
          for (int k = 0; k < kPairBK / kUmmaK; ++k) {
            constexpr int kPerChunk = kBK / kUmmaK;
            const int c = k / kPerChunk, j = k % kPerChunk;
            if (c >= chunks) break;
            const uint64_t ad = smem_desc_sw128(sa + c * (kBM * kBK) + j * kUmmaK, 16, 1024);
            const uint64_t bd = B_MN ? smem_desc_sw128(sb + k * kUmmaK * 128, 128 * kPairBK, 1024)
                                     : smem_desc_sw128(sb + c * ((BN / 2) * kBK) + j * kUmmaK, 16, 1024);
            mma_i8_pair(d, ad, bd, idesc, (kb > sg.kb0 || k > 0) ? 1u : 0u);
          }
          issued = true;
          mma_commit_pair(empty_bar(stage));           // our stage is free ...
          mma_commit_pair(empty_peer0 + 8u * stage);   // ... and the peer's
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit_pair(tfull_bar(acc));
        mma_commit_pair(tfull_peer0 + 8u * acc);
      }
      // Every MMA must retire before either CTA releases its TMEM.
      if (issued) {
        mma_commit_pair(done_bar);
        mbar_wait_bounded(done_bar, 0, nullptr, &g_gemm_status);
      }
    }
  } else {
    // ---------------- epilogue (both CTAs): this CTA's 128 rows of every 256 x 256 tile
    const int quarter = warp & 3;     // TMEM lane quarter this warp may access
    const int part = (warp - 2) / 4;  // which share of the tile's columns (gate/up glue)
    const uint32_t stage_base = base + L::kEpiOff + (warp - 2) * epi_bufs<EPI>() * epi_buf_bytes<EPI>();
    const uint32_t tempty_leader0 = mapa_shared(tempty_bar(0), 0);
    Schedule sched(args, worker, workers);
    Segment sg;
    uint32_t sbuf = 0;
    int local = 0;
    while (sched.next(args, sg)) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      ++local;
      const bool ok = mbar_wait_bounded(tfull_bar(acc), acc_phase, abort_flag, &g_gemm_status);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const int mb = sg.tile % args.m_tiles;
      const int nb = sg.tile / args.m_tiles;
      const int row0 = mb * 2 * kBM + static_cast<int>(rank) * kBM + quarter * 32;
      float sxr = 0.f;
      if constexpr (EPI != kEpiI32) sxr = row0 + lane < args.m ? __ldg(args.sx + row0 + lane) : 0.f;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kBN;
      epilogue_segment<EPI>(args, &tm_c, sg, taddr, row0, nb * args.bn, sxr, stage_base, sbuf, lane,
                            2 * epi_warps<EPI>(), part, [&] { mbar_arrive_tmem_handoff(tempty_leader0 + 8u * acc); });
    }
    if (lane == 0) bulk_wait_group<0>();  // every store of this warp has landed
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still touch its barriers or TMEM
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

// =====================================================================================
// 128 x 256 tiles on one CTA (tcgen05 cta_group::1), for M <= 128
// =====================================================================================
template <bool B_MN, int EPI>
__global__ void __launch_bounds__(threads_for<EPI>(), 1)
    gemm_single_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                       const __grid_constant__ CUtensorMap tm_c, const GemmArgs args) {
  using L = SingleSmem;
  constexpr int STAGES = kSingleStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
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
  pdl_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), epi_warps<EPI>());
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_b);
    if (args.tma_out) prefetch_tmap(&tm_c);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();  // the previous kernel's writes (our A, B) are visible from here on
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      Schedule sched(args, blockIdx.x, gridDim.x);
      Segment sg;
      int stage = 0;
      uint32_t phase = 0, issued_mask = 0, last_phase = 0;
      bool ok = true;
      while (ok && sched.next(args, sg)) {
        const int mb = sg.tile % args.m_tiles;
        const int nb = sg.tile / args.m_tiles;
        for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
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
            for (int j = 0; j < kBN / 128; ++j)
              tma_load_2d(sb + j * 128 * kBK, &tm_b, full_bar(stage), nb * kBN + j * 128, kb * kBK);
          } else {
            tma_load_2d(sb, &tm_b, full_bar(stage), kb * kBK, nb * kBN);
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
        if (issued_mask & (1u << s))
          mbar_wait_bounded(full_bar(s), (last_phase >> s) & 1u, nullptr, &g_gemm_status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc = idesc_i8(kBM, kBN, B_MN);
      Schedule sched(args, blockIdx.x, gridDim.x);
      Segment sg;
      int stage = 0, local = 0;
      uint32_t phase = 0;
      bool ok = true, issued = false;
      while (ok && sched.next(args, sg)) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        ++local;
        if (!mbar_wait_bounded(tempty_bar(acc), acc_phase ^ 1u, abort_flag, &g_gemm_status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * kBN;
        for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
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
            mma_i8(d, ad, bd, idesc, (kb > sg.kb0 || k > 0) ? 1u : 0u);
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
      if (issued) {
        mma_commit(done_bar);
        mbar_wait_bounded(done_bar, 0, nullptr, &g_gemm_status);
      }
    }
  } else {
    // ---------------- epilogue
    const int quarter = warp & 3;
    const int part = (warp - 2) / 4;
    const uint32_t stage_base = base + L::kEpiOff + (warp - 2) * epi_bufs<EPI>() * epi_buf_bytes<EPI>();
    Schedule sched(args, blockIdx.x, gridDim.x);
    Segment sg;
    uint32_t sbuf = 0;
    int local = 0;
    while (sched.next(args, sg)) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      ++local;
      const bool ok = mbar_wait_bounded(tfull_bar(acc), acc_phase, abort_flag, &g_gemm_status);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const int mb = sg.tile % args.m_tiles;
      const int nb = sg.tile / args.m_tiles;
      const int row0 = mb * kBM + quarter * 32;
      float sxr = 0.f;
      if constexpr (EPI != kEpiI32) sxr = row0 + lane < args.m ? __ldg(args.sx + row0 + lane) : 0.f;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kBN;
      epilogue_segment<EPI>(args, &tm_c, sg, taddr, row0, nb * kBN, sxr, stage_base, sbuf, lane,
                            epi_warps<EPI>(), part, [&] { mbar_arrive(tempty_bar(acc)); });
    }
    if (lane == 0) bulk_wait_group<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
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

// 2-D tensor [outer, inner] with row pitch `pitch` bytes, 128-byte swizzled boxes (or
// `swizzle`).
static int encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* ptr, int64_t inner,
                     int64_t outer, int64_t pitch, uint32_t box_inner, uint32_t box_outer,
                     CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
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
                         CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed with CUresult %d (inner %lld, outer %lld, pitch %lld)",
              static_cast<int>(r), static_cast<long long>(inner), static_cast<long long>(outer),
              static_cast<long long>(pitch));
    return W8_ERR_CUDA;
  }
  return W8_OK;
}

// A K-major int8 operand [rows, K] (K % 128 == 0) viewed in 3-D as (128-byte chunk,
// row, chunk index): a box of {128, box_rows, kPairChunks} lands in shared memory as
// kPairChunks consecutive swizzle-128 blocks of box_rows rows each.
static int encode_kchunks(CUtensorMap* map, const void* ptr, int64_t k, int64_t rows, int64_t pitch,
                          uint32_t box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return W8_ERR_CUDA;
  }
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(w8::kBK), static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(k / w8::kBK)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(pitch), static_cast<cuuint64_t>(w8::kBK)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(w8::kBK), box_rows, static_cast<cuuint32_t>(w8::kPairChunks)};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (3-D) failed with CUresult %d (k %lld, rows %lld, pitch %lld)",
              static_cast<int>(r), static_cast<long long>(k), static_cast<long long>(rows),
              static_cast<long long>(pitch));
    return W8_ERR_CUDA;
  }
  return W8_OK;
}

// The head-major qkv output [heads, T, D] (bf16) as a 3-D tensor (D, T, heads) with
// 32-column x 32-row x 1-head boxes, unswizzled: stores clip at T and at the last head.
static int encode_heads_out(CUtensorMap* map, const void* ptr, int64_t d, int64_t t, int64_t heads,
                            int64_t ld_tok, int64_t ld_head) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return W8_ERR_CUDA;
  }
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(t), static_cast<cuuint64_t>(heads)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld_tok * 2), static_cast<cuuint64_t>(ld_head * 2)};
  const cuuint32_t box[3] = {32, 32, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (heads) failed with CUresult %d (d %lld, t %lld, heads %lld)",
              static_cast<int>(r), static_cast<long long>(d), static_cast<long long>(t), static_cast<long long>(heads));
    return W8_ERR_CUDA;
  }
  return W8_OK;
}

// Arguments of the fused qkv glue epilogue (w8_gemm_qkv_norm_rope).
struct QkvEpiParams {
  const uint16_t* cos;
  const uint16_t* sin;
  int64_t ldcs;
  int cs_tiled;
  const uint16_t* qw;
  const uint16_t* kw;
  float eps;
  int q_heads, k_heads;
  int64_t ld_head, ld_tok;
};

int require_sm100(int* device);

template <typename Kernel>
static int set_smem_once(int device, Kernel kern, int bytes, bool* done) {
  if (device < 0 || device >= 64) return W8_ERR_UNSUPPORTED;
  if (!done[device]) {
    W8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done[device] = true;
  }
  return W8_OK;
}

// Co-resident CTA pairs of the pair kernel on this device (a GPC with an odd number of
// SMs leaves one idle), cached per device.
template <bool B_MN, int EPI, int BN>
static int pair_capacity(int device, int* out) {
  auto kern = w8::gemm_pair_kernel<B_MN, EPI, BN>;
  static bool done[64] = {};
  static int cap[64] = {};
  int st = set_smem_once(device, kern, w8::PairSmem::kAlloc, done);
  if (st != W8_OK) return st;
  if (cap[device] == 0) {
    int sms = 0;
    st = num_sms(&sms);
    if (st != W8_OK) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms & ~1, 1, 1);
    cfg.blockDim = dim3(w8::threads_for<EPI>(), 1, 1);
    cfg.dynamicSmemBytes = w8::PairSmem::kAlloc;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    W8_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
    cap[device] = n > 0 ? n : 1;
  }
  *out = cap[device];
  return W8_OK;
}

// Launch with programmatic stream serialization: the kernel may be scheduled while the
// previous kernel on the stream drains; it waits (griddepcontrol.wait) before touching
// global memory, so only its launch and prologue overlap.
template <typename Kernel>
static int launch_pdl(Kernel kern, int grid, int threads, int smem, cudaStream_t stream, const CUtensorMap& ta,
                      const CUtensorMap& tb, const CUtensorMap& tc, const w8::GemmArgs& args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, ta, tb, tc, args));
}

// Schedule of the last GEMM launched from this thread (w8_gemm_last_schedule).
struct LastSchedule {
  int stream_k, workers, tile_n, pair;
};
static thread_local LastSchedule g_last_schedule = {0, 0, 0, 0};

// Stream-K pays off when whole tiles would leave the last wave of workers mostly idle
// and each tile is long enough (K) that splitting it costs little next to its MMAs.
// One wave of whole tiles that keeps at least half the workers busy stays whole: there the
// split tiles' waits and reduce-adds cost more than the idle workers give back (down
// 1536 x 6144 at M = 1607, 42 tiles on 74 pairs: 22.5 us whole, 23.7 us stream-K; at
// M = 858, 24 tiles: 21.5 us whole, 19.5 us stream-K).
static bool want_stream_k(int64_t tiles, int workers, int k) {
  if (k < 24 * w8::kBK) return false;
  const int64_t waves = (tiles + workers - 1) / workers;
  if (waves == 1 && 2 * tiles >= workers) return false;
  return tiles * 100 < waves * workers * 90;  // whole-tile efficiency below 90 %
}

template <bool B_MN, int EPI, int BN>
static int launch_pair(int device, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                       w8::GemmArgs args, int64_t flag_words, cudaStream_t stream) {
  auto kern = w8::gemm_pair_kernel<B_MN, EPI, BN>;
  int cap = 0;
  int st = pair_capacity<B_MN, EPI, BN>(device, &cap);
  if (st != W8_OK) return st;
  const int64_t tiles = static_cast<int64_t>(args.m_tiles) * args.n_tiles;
  int workers = static_cast<int>(tiles < cap ? tiles : cap);
  args.stream_k = 0;
  if (EPI == w8::kEpiI32 && args.tma_out && args.flags != nullptr && flag_words >= tiles &&
      want_stream_k(tiles, cap, args.k)) {
    const int64_t units = tiles * args.k_blocks;
    workers = static_cast<int>(units < cap ? units : cap);
    args.stream_k = 1;
  }
  g_last_schedule = {args.stream_k, workers, BN, 1};
  return launch_pdl(kern, 2 * workers, w8::threads_for<EPI>(), w8::PairSmem::kAlloc, stream, ta, tb, tc, args);
}

template <bool B_MN, int EPI>
static int launch_single(int device, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                         w8::GemmArgs args, int64_t flag_words, cudaStream_t stream) {
  auto kern = w8::gemm_single_kernel<B_MN, EPI>;
  static bool done[64] = {};
  int st = set_smem_once(device, kern, w8::SingleSmem::kAlloc, done);
  if (st != W8_OK) return st;
  int sms = 0;
  st = num_sms(&sms);
  if (st != W8_OK) return st;
  const int64_t tiles = static_cast<int64_t>(args.m_tiles) * args.n_tiles;
  int workers = static_cast<int>(tiles < sms ? tiles : sms);
  args.stream_k = 0;
  if (EPI == w8::kEpiI32 && args.tma_out && args.flags != nullptr && flag_words >= tiles &&
      want_stream_k(tiles, sms, args.k)) {
    const int64_t units = tiles * args.k_blocks;
    workers = static_cast<int>(units < sms ? units : sms);
    args.stream_k = 1;
  }
  g_last_schedule = {args.stream_k, workers, w8::kBN, 0};
  return launch_pdl(kern, workers, w8::threads_for<EPI>(), w8::SingleSmem::kAlloc, stream, ta, tb, tc, args);
}

static int gemm_common(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, int b_layout,
                       void* out, int64_t ldo, int out_elem, const float* sx, const float* sw,
                       int64_t m, int64_t n, int64_t k, void* workspace, int64_t workspace_bytes,
                       cudaStream_t stream, int epi, float* row_absmax = nullptr,
                       int64_t clear_words = 0, const QkvEpiParams* qkv = nullptr) {
  // Output columns: the GEMM's N, or N / 2 for the gate/up glue (gelu(gate) * up).
  const int64_t n_out = epi == w8::kEpiGeluUp ? n / 2 : n;
  W8_CHECK_ARG(m >= 0 && n >= 0 && k >= 0, "negative size (m=%lld n=%lld k=%lld)", (long long)m,
               (long long)n, (long long)k);
  W8_CHECK_ARG(m < (1ll << 31) && n < (1ll << 31) && k < (1ll << 31), "size beyond int32 range");
  W8_CHECK_ARG(b_layout == W8_B_KN || b_layout == W8_B_NK, "b_layout must be W8_B_KN or W8_B_NK");
  W8_CHECK_ARG(workspace_bytes >= 0, "negative workspace size");
  if (m == 0 || n == 0) return W8_OK;
  W8_CHECK_ARG(out != nullptr, "null output pointer");
  W8_CHECK_ARG(ldo >= n_out, "output row pitch %lld < %lld columns", (long long)ldo, (long long)n_out);
  W8_CHECK_ALIGN(aligned(out, out_elem), "output must be aligned to its element size");
  if (epi != w8::kEpiI32) W8_CHECK_ARG(sx != nullptr && sw != nullptr, "null scale pointer");
  if (epi == w8::kEpiGeluUp) {
    W8_CHECK_ARG(b_layout == W8_B_NK, "the gate/up glue takes packed [2I, K] weights (W8_B_NK)");
    W8_CHECK_ARG(n % 256 == 0, "2 * inter = %lld must be a multiple of 256", (long long)n);
    W8_CHECK_ARG(row_absmax != nullptr, "null row absmax scratch");
    W8_CHECK_ALIGN(aligned(row_absmax, 4), "row absmax scratch must be 4-byte aligned");
    W8_CHECK_ALIGN(aligned(out, 16) && (ldo * out_elem) % 16 == 0,
                   "the gate/up glue output must be 16-byte aligned with a 16-byte row pitch");
  }
  W8_CHECK_ALIGN(workspace == nullptr || aligned(workspace, 4), "workspace must be 4-byte aligned");
  int device = 0;
  int st = require_sm100(&device);
  if (st != W8_OK) return st;
  if (k == 0) {
    // An empty contraction: the product is all zeros (and so is its dequant).
    W8_CUDA_TRY(cudaMemset2DAsync(out, ldo * out_elem, 0, n_out * out_elem, m, stream));
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

  // 256-row tiles on CTA pairs; their operand copies cover two 128-byte K chunks, which
  // needs K to be a multiple of 128.  Otherwise one CTA per 128 x 256 tile.
  bool pair = m > w8::kBM && k % w8::kBK == 0;
  if (pair && epi == w8::kEpiQkv) {
    // The qkv glue needs whole 256-column tiles (one head each), so its wave count cannot
    // be evened out by a narrower tile: take 128-row tiles on single CTAs when they need
    // fewer waves than 256-row tiles on CTA pairs (M = 3658, 10 heads: 290 tiles on 148
    // SMs in 2 waves, against 150 on 74 pairs in 3, the last with 2 tiles).
    int cap = 0, sms = 0;
    st = pair_capacity<false, w8::kEpiQkv, w8::kBN>(device, &cap);
    if (st != W8_OK) return st;
    st = num_sms(&sms);
    if (st != W8_OK) return st;
    const int64_t heads_n = n / 256;
    const int64_t pair_waves = ((m + 255) / 256 * heads_n + cap - 1) / cap;
    const int64_t single_waves = ((m + 127) / 128 * heads_n + sms - 1) / sms;
    if (single_waves < pair_waves) pair = false;
  }
  int rows_per_tile = pair ? 2 * w8::kBM : w8::kBM;
  // Tile width on CTA pairs over a K-major B: the narrowest of 64, 128, 192 and 256
  // columns that needs no more waves of workers than any other.  A narrower tile costs
  // more per column (a 192-wide tile ~1.28x of a 256-wide one, a 64-wide one ~3x) but
  // finishes sooner, so it pays only where it adds no wave: N = 2560 / 1536 at M = 3658
  // take 192, while GEMMs with one wave of tiles or less (the 1536 -> 256 PLE gate, short
  // prompts) take 64 or 128 and spread over more SMs (measured, bf16 out: PLE gate at
  // M = 3658 11.2 -> 8.6 us, qkv at M = 207 10.1 -> 8.5 us, o at M = 858 11.4 -> 10.7 us).
  // Shapes that stream-K will balance keep 256.
  if (epi == w8::kEpiQkv) {
    W8_CHECK_ARG(qkv != nullptr && b_layout == W8_B_NK, "the qkv glue takes [N, K] weights and its parameters");
    W8_CHECK_ARG(n % 256 == 0, "n = %lld must be a whole number of 256-wide heads", (long long)n);
  }
  int bn = w8::kBN;
  if (pair && b_layout == W8_B_NK && epi != w8::kEpiGeluUp && epi != w8::kEpiQkv &&
      !(epi == w8::kEpiI32 && workspace != nullptr && k >= 24 * w8::kBK)) {
    int cap = 0;
    st = pair_capacity<false, w8::kEpiI32, w8::kBN>(device, &cap);
    if (st != W8_OK) return st;
    const int64_t m_tiles = (m + rows_per_tile - 1) / rows_per_tile;
    auto waves = [&](int64_t w) { return (m_tiles * ((n + w - 1) / w) + cap - 1) / cap; };
    const int widths[4] = {256, 192, 128, 64};
    int64_t best = waves(256);
    for (int w : widths) {
      const int64_t v = waves(w);
      if (v <= best) {
        best = v;
        bn = w;
      }
    }
    // 128 x 256 tiles on single CTAs instead, when they need fewer waves than the best pair
    // width and that width is a narrow one (its tiles already cost more per column): qkv
    // 3658 x 2560 x 1536 as 290 single-CTA tiles on 148 SMs takes 2 waves and 18.5 us,
    // against 3 waves of 210 192-wide pair tiles, 21.1 us.  Against 256-wide pair tiles the
    // pairs stay faster even with a wave more (PLE 8960 x 1536: 51.6 against 52.3 us).
    if (bn < w8::kBN) {
      int sms = 0;
      st = num_sms(&sms);
      if (st != W8_OK) return st;
      const int64_t single_waves = ((m + w8::kBM - 1) / w8::kBM * ((n + w8::kBN - 1) / w8::kBN) + sms - 1) / sms;
      if (single_waves < best) {
        pair = false;
        rows_per_tile = w8::kBM;
        bn = w8::kBN;
      }
    }
  } else if (pair && b_layout == W8_B_NK && epi == w8::kEpiI32 && workspace != nullptr && k >= 24 * w8::kBK) {
    // Stream-K over at most half a wave of pair tiles: single CTAs give it twice the
    // workers (down 1536 x 6144 at M = 207 13.6 against 15.4 us, at M = 858 17.6 against
    // 19.8 us).
    int cap = 0;
    st = pair_capacity<false, w8::kEpiI32, w8::kBN>(device, &cap);
    if (st != W8_OK) return st;
    const int64_t pair_tiles = (m + rows_per_tile - 1) / rows_per_tile * ((n + w8::kBN - 1) / w8::kBN);
    if (2 * pair_tiles <= cap) {
      pair = false;
      rows_per_tile = w8::kBM;
    }
  }
  const uint32_t b_box_n = pair ? bn / 2 : w8::kBN;  // B columns one CTA stages per K-block
  CUtensorMap ta, tb, tc;
  const int stage_k = pair ? w8::kPairBK : w8::kBK;  // K bytes per pipeline stage
  if (pair)
    st = encode_kchunks(&ta, a, k, m, lda, w8::kBM);
  else
    st = encode_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, a, k, m, lda, w8::kBK, w8::kBM);
  if (st != W8_OK) return st;
  if (b_layout == W8_B_NK && pair)
    st = encode_kchunks(&tb, b, k, n, ldb, b_box_n);
  else if (b_layout == W8_B_NK)
    st = encode_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, b, k, n, ldb, w8::kBK, b_box_n);
  else
    st = encode_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, b, n, k, ldb, 128, stage_k);
  if (st != W8_OK) return st;

  w8::GemmArgs args;
  args.m = static_cast<int>(m);
  args.n = static_cast<int>(n);
  args.k = static_cast<int>(k);
  args.m_tiles = static_cast<int>((m + rows_per_tile - 1) / rows_per_tile);
  args.n_tiles = static_cast<int>((n + bn - 1) / bn);
  args.bn = bn;
  args.k_blocks = static_cast<int>((k + stage_k - 1) / stage_k);
  args.out = out;
  args.ldo = ldo;
  args.sx = sx;
  args.sw = sw;
  args.vec_out = aligned(out, 16) && (ldo * out_elem) % 16 == 0;
  args.vec_sw = sw != nullptr && aligned(sw, 16);
  args.stream_k = 0;
  args.flags = static_cast<uint32_t*>(workspace);
  args.row_absmax = row_absmax;
  args.cos = args.sin = args.qw = args.kw = nullptr;
  args.ldcs = 0;
  args.cs_tiled = 0;
  args.eps = 0.f;
  args.q_heads = args.k_heads = 0;
  if (qkv != nullptr) {
    args.cos = reinterpret_cast<const __nv_bfloat16*>(qkv->cos);
    args.sin = reinterpret_cast<const __nv_bfloat16*>(qkv->sin);
    args.ldcs = qkv->ldcs;
    args.cs_tiled = qkv->cs_tiled;
    args.qw = reinterpret_cast<const __nv_bfloat16*>(qkv->qw);
    args.kw = reinterpret_cast<const __nv_bfloat16*>(qkv->kw);
    args.eps = qkv->eps;
    args.q_heads = qkv->q_heads;
    args.k_heads = qkv->k_heads;
  }
  const int64_t flag_words = workspace_bytes / 4;
  // Output through TMA when the tensor map can address it (16-byte base and pitch);
  // one box is 32 rows x 128 bytes.  Otherwise the epilogue stores directly.
  memset(&tc, 0, sizeof(tc));
  args.tma_out = 0;
  if (epi == w8::kEpiQkv) {
    st = encode_heads_out(&tc, out, 256, m, n / 256, qkv->ld_tok, qkv->ld_head);
    if (st != W8_OK) return st;
    args.tma_out = 1;
  } else if (args.vec_out) {
    const bool i32 = epi == w8::kEpiI32;
    // The gate/up glue stores 32-row x 32-column bf16 boxes (one per epilogue warp,
    // unswizzled 64-byte rows).
    st = epi == w8::kEpiGeluUp
             ? encode_2d(&tc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, out, n_out, m, ldo * out_elem, 32, 32,
                         CU_TENSOR_MAP_SWIZZLE_NONE)
             : encode_2d(&tc, i32 ? CU_TENSOR_MAP_DATA_TYPE_INT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, out, n_out,
                         m, ldo * out_elem, i32 ? 32 : 64, 32);
    if (st != W8_OK) return st;
    args.tma_out = 1;
  }

  // Counters the caller asked to have cleared (the allocation-free entry point's shared
  // scratch) are cleared only now, after every argument check: a rejected call leaves
  // them as they were.
  if (clear_words > 0) W8_CUDA_TRY(cudaMemsetAsync(workspace, 0, static_cast<size_t>(clear_words) * 4, stream));

  const bool mn = b_layout == W8_B_KN;
  const bool i32 = epi == w8::kEpiI32;
  if (epi == w8::kEpiGeluUp)
    return pair ? launch_pair<false, w8::kEpiGeluUp, 256>(device, ta, tb, tc, args, flag_words, stream)
                : launch_single<false, w8::kEpiGeluUp>(device, ta, tb, tc, args, flag_words, stream);
  if (epi == w8::kEpiQkv)
    return pair ? launch_pair<false, w8::kEpiQkv, 256>(device, ta, tb, tc, args, flag_words, stream)
                : launch_single<false, w8::kEpiQkv>(device, ta, tb, tc, args, flag_words, stream);
  if (pair) {
    if (mn)
      return i32 ? launch_pair<true, w8::kEpiI32, 256>(device, ta, tb, tc, args, flag_words, stream)
                 : launch_pair<true, w8::kEpiBf16, 256>(device, ta, tb, tc, args, flag_words, stream);
    if (i32) {
      switch (bn) {
        case 64: return launch_pair<false, w8::kEpiI32, 64>(device, ta, tb, tc, args, flag_words, stream);
        case 128: return launch_pair<false, w8::kEpiI32, 128>(device, ta, tb, tc, args, flag_words, stream);
        case 192: return launch_pair<false, w8::kEpiI32, 192>(device, ta, tb, tc, args, flag_words, stream);
        default: return launch_pair<false, w8::kEpiI32, 256>(device, ta, tb, tc, args, flag_words, stream);
      }
    }
    switch (bn) {
      case 64: return launch_pair<false, w8::kEpiBf16, 64>(device, ta, tb, tc, args, flag_words, stream);
      case 128: return launch_pair<false, w8::kEpiBf16, 128>(device, ta, tb, tc, args, flag_words, stream);
      case 192: return launch_pair<false, w8::kEpiBf16, 192>(device, ta, tb, tc, args, flag_words, stream);
      default: return launch_pair<false, w8::kEpiBf16, 256>(device, ta, tb, tc, args, flag_words, stream);
    }
  }
  if (i32)
    return mn ? launch_single<true, w8::kEpiI32>(device, ta, tb, tc, args, flag_words, stream)
              : launch_single<false, w8::kEpiI32>(device, ta, tb, tc, args, flag_words, stream);
  return mn ? launch_single<true, w8::kEpiBf16>(device, ta, tb, tc, args, flag_words, stream)
            : launch_single<false, w8::kEpiBf16>(device, ta, tb, tc, args, flag_words, stream);
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

// ---------------------------------------------------------------- allocation-free entry point
// Scratch of w8_mm_i8_noalloc: the stream-K tile counters live in this library-owned
// array instead of a caller workspace.  Every GPU that loads the library holds it
// (64 KiB) until the process exits.  In host code the name is only a stand-in for the
// device object: its device address comes from cudaGetSymbolAddress.
namespace w8 {
constexpr int64_t kNoAllocMaxTiles = 16384;
static __device__ __align__(256) uint32_t g_noalloc_counters[kNoAllocMaxTiles];
}  // namespace w8

namespace w8host {
// Device address of g_noalloc_counters, looked up once per device with that device current.
static int noalloc_counters(int device, uint32_t** out) {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static uint32_t* ptr[kMaxDevices] = {};
  if (device < 0 || device >= kMaxDevices) {
    set_error("w8_mm_i8_noalloc: device ordinal %d out of range", device);
    return W8_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (ptr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, w8::g_noalloc_counters);
    if (e != cudaSuccess) return cuda_status(e);
    ptr[device] = static_cast<uint32_t*>(p);
  }
  *out = ptr[device];
  return W8_OK;
}
}  // namespace w8host

extern "C" int w8_mm_i8_noalloc(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb,
                                int b_layout, int32_t* c, int64_t ldc, int64_t m, int64_t n, int64_t k,
                                w8_stream_t stream) {
  W8_CHECK_ARG(m >= 0 && n >= 0 && k >= 0, "negative size (m=%lld n=%lld k=%lld)", (long long)m,
               (long long)n, (long long)k);
  if (m == 0 || n == 0) return W8_OK;
  const int64_t tiles = ((m + w8::kBM - 1) / w8::kBM) * ((n + w8::kBN - 1) / w8::kBN);
  W8_CHECK_ARG(tiles <= w8::kNoAllocMaxTiles,
               "w8_mm_i8_noalloc: %lld x %lld needs %lld tile counters; its static scratch holds %lld "
               "(M/128 * N/256 rounded up must be <= %lld); use w8_mm_i8_ws with a workspace",
               (long long)m, (long long)n, (long long)tiles, (long long)w8::kNoAllocMaxTiles,
               (long long)w8::kNoAllocMaxTiles);
  int device = 0;
  int st = w8host::require_sm100(&device);
  if (st != W8_OK) return st;
  uint32_t* counters = nullptr;
  st = w8host::noalloc_counters(device, &counters);
  if (st != W8_OK) return st;
  // The array keeps whatever the last call left: gemm_common clears this call's counters,
  // after its argument checks and just before the launch.
  return w8host::gemm_common(a, lda, b, ldb, b_layout, c, ldc, 4, nullptr, nullptr, m, n, k, counters,
                             tiles * 4, reinterpret_cast<cudaStream_t>(stream), w8::kEpiI32, nullptr, tiles);
}

extern "C" int w8_gemm_last_schedule(int* stream_k, int* workers, int* tile_n) {
  const w8host::LastSchedule& s = w8host::g_last_schedule;
  if (stream_k != nullptr) *stream_k = s.stream_k;
  if (workers != nullptr) *workers = s.workers;
  if (tile_n != nullptr) *tile_n = s.tile_n;
  return s.pair;
}

extern "C" int w8_inject_stream_k_stall(int drop_signal, uint64_t wait_limit_ns) {
  int device = 0;
  int st = w8host::require_sm100(&device);
  if (st != W8_OK) return st;
  const int drop = drop_signal ? 1 : 0;
  const unsigned long long limit = wait_limit_ns;
  W8_CUDA_TRY(cudaDeviceSynchronize());  // no GEMM of this device is in flight while the hook changes
  W8_CUDA_TRY(cudaMemcpyToSymbol(w8::g_sk_drop_signal, &drop, sizeof(int)));
  W8_CUDA_TRY(cudaMemcpyToSymbol(w8::g_sk_wait_limit_ns, &limit, sizeof(limit)));
  return W8_OK;
}

extern "C" int64_t w8_mm_i8_workspace_bytes(int64_t m, int64_t n, int64_t k) {
  (void)k;
  if (m <= 0 || n <= 0) return 0;
  // One 32-bit counter per output tile of whichever tiling the launch picks.
  const int64_t single = ((m + w8::kBM - 1) / w8::kBM) * ((n + w8::kBN - 1) / w8::kBN);
  const int64_t pair192 = ((m + 2 * w8::kBM - 1) / (2 * w8::kBM)) * ((n + 191) / 192);
  return 4 * (single > pair192 ? single : pair192);
}

extern "C" int w8_mm_i8(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, int b_layout,
                        int32_t* c, int64_t ldc, int64_t m, int64_t n, int64_t k,
                        w8_stream_t stream) {
  return w8host::gemm_common(a, lda, b, ldb, b_layout, c, ldc, 4, nullptr, nullptr, m, n, k, nullptr,
                             0, reinterpret_cast<cudaStream_t>(stream), w8::kEpiI32);
}

extern "C" int w8_mm_i8_ws(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, int b_layout,
                           int32_t* c, int64_t ldc, int64_t m, int64_t n, int64_t k, void* workspace,
                           int64_t workspace_bytes, w8_stream_t stream) {
  return w8host::gemm_common(a, lda, b, ldb, b_layout, c, ldc, 4, nullptr, nullptr, m, n, k, workspace,
                             workspace_bytes, reinterpret_cast<cudaStream_t>(stream), w8::kEpiI32);
}

namespace w8host {
int quant_rows_absmax_bf16(const uint16_t* y, int64_t ldy, float* absmax, int8_t* q, int64_t ldq, float* s,
                           int64_t m, int64_t k, cudaStream_t stream);
}  // namespace w8host

extern "C" int w8_gemm_gelu_up_quant(const int8_t* a, int64_t lda, const int8_t* w, int64_t ldw,
                                     const float* sx, const float* sw, int64_t m, int64_t inter, int64_t k,
                                     uint16_t* y, int64_t ldy, float* row_absmax, int8_t* q, int64_t ldq,
                                     float* s, w8_stream_t stream) {
  W8_CHECK_ARG(inter >= 0 && inter % 128 == 0, "inter = %lld must be a multiple of 128", (long long)inter);
  if (m == 0 || inter == 0) return W8_OK;
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int r = w8host::gemm_common(a, lda, w, ldw, W8_B_NK, y, ldy, 2, sx, sw, m, 2 * inter, k, nullptr, 0,
                                    st, w8::kEpiGeluUp, row_absmax);
  if (r != W8_OK) return r;
  return w8host::quant_rows_absmax_bf16(y, ldy, row_absmax, q, ldq, s, m, inter, st);
}

extern "C" int w8_gemm_dequant_bf16(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb,
                                    int b_layout, const float* sx, const float* sw, uint16_t* y,
                                    int64_t ldy, int64_t m, int64_t n, int64_t k,
                                    w8_stream_t stream) {
  return w8host::gemm_common(a, lda, b, ldb, b_layout, y, ldy, 2, sx, sw, m, n, k, nullptr, 0,
                             reinterpret_cast<cudaStream_t>(stream), w8::kEpiBf16);
}

namespace w8host {
static int qkv_norm_rope_common(const int8_t* a, int64_t lda, const int8_t* w, int64_t ldw, const float* sx,
                                const float* sw, int64_t m, int64_t heads, int64_t kv_heads, int shared,
                                const uint16_t* cos, const uint16_t* sin, int64_t ldcs, int tiled, const uint16_t* qw,
                                const uint16_t* kw, float eps, uint16_t* out, int64_t ld_head, int64_t ld_tok,
                                int64_t k, w8_stream_t stream) {
  W8_CHECK_ARG(m >= 0 && heads >= 0 && kv_heads >= 0 && heads < 4096 && kv_heads < 4096, "bad size");
  const int64_t per_tok = shared ? heads : heads + 2 * kv_heads;
  if (m == 0 || per_tok == 0) return W8_OK;
  W8_CHECK_ARG(cos != nullptr && sin != nullptr && qw != nullptr && out != nullptr, "null pointer");
  W8_CHECK_ARG(shared || kv_heads == 0 || kw != nullptr, "null k_norm weight");
  W8_CHECK_ARG(ldcs >= (tiled ? 8 * m : 256) && ld_tok >= 256 && ld_head >= ld_tok * m, "pitch too small");
  W8_CHECK_ALIGN(aligned(cos, 16) && aligned(sin, 16) && ldcs % 8 == 0 && aligned(qw, 16) &&
                     (kw == nullptr || aligned(kw, 16)) && aligned(out, 16) && ld_head % 8 == 0 && ld_tok % 8 == 0,
                 "weights, cos/sin and the output must be 16-byte aligned with pitches %% 8 == 0");
  QkvEpiParams q;
  q.cos = cos;
  q.sin = sin;
  q.ldcs = ldcs;
  q.cs_tiled = tiled;
  q.qw = qw;
  q.kw = kw;
  q.eps = eps;
  q.q_heads = static_cast<int>(heads);
  q.k_heads = shared ? 0 : static_cast<int>(kv_heads);
  q.ld_head = ld_head;
  q.ld_tok = ld_tok;
  return gemm_common(a, lda, w, ldw, W8_B_NK, out, per_tok * 256, 2, sx, sw, m, per_tok * 256, k, nullptr, 0,
                     reinterpret_cast<cudaStream_t>(stream), w8::kEpiQkv, nullptr, 0, &q);
}
}  // namespace w8host

extern "C" int w8_gemm_qkv_norm_rope(const int8_t* a, int64_t lda, const int8_t* w, int64_t ldw, const float* sx,
                                     const float* sw, int64_t m, int64_t heads, int64_t kv_heads, int shared,
                                     const uint16_t* cos, const uint16_t* sin, int64_t ldcs, const uint16_t* qw,
                                     const uint16_t* kw, float eps, uint16_t* out, int64_t ld_head, int64_t ld_tok,
                                     int64_t k, w8_stream_t stream) {
  return w8host::qkv_norm_rope_common(a, lda, w, ldw, sx, sw, m, heads, kv_heads, shared, cos, sin, ldcs, 0, qw, kw,
                                      eps, out, ld_head, ld_tok, k, stream);
}

extern "C" int w8_gemm_qkv_norm_rope_tiled(const int8_t* a, int64_t lda, const int8_t* w, int64_t ldw,
                                           const float* sx, const float* sw, int64_t m, int64_t heads,
                                           int64_t kv_heads, int shared, const uint16_t* cos_t,
                                           const uint16_t* sin_t, int64_t tile_pitch, const uint16_t* qw,
                                           const uint16_t* kw, float eps, uint16_t* out, int64_t ld_head,
                                           int64_t ld_tok, int64_t k, w8_stream_t stream) {
  return w8host::qkv_norm_rope_common(a, lda, w, ldw, sx, sw, m, heads, kv_heads, shared, cos_t, sin_t, tile_pitch,
                                      1, qw, kw, eps, out, ld_head, ld_tok, k, stream);
}
