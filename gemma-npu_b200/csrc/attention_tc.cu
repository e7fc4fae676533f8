// Prefill attention on the 5th-generation tensor cores (tcgen05, accumulators in TMEM): the
// contract of attention.cu (pipeline.py:139-180, full_attention / sliding_attention with
// q_start = 0: causal, window W > 0 or none, scale 1.0, grouped-query heads, bf16 in and
// out, fp32 softmax and accumulation) on a schedule built for sm_100a.
//
// A cluster of two CTAs on two SMs (tcgen05 cta_group::2) owns 256 query rows and one
// 256-column half of the output; each CTA holds 128 of the rows (its TMEM lanes).  The rows
// of a CTA are PK heads of one KV group times 128 / PK consecutive queries (grouped-query
// packing: heads that share a K / V stream read it once), PK the largest power of two
// <= 16 dividing the group size; the two CTAs take consecutive query blocks.  Per CTA,
// warp 0 loads with TMA, warps 2-5 run the softmax with one thread per row; warp 1 of
// the even CTA issues the pair's MMAs.  Per 128-key tile j:
//   S_j  = Q K_j^T     tcgen05.mma kind::f16 (bf16 x bf16 -> fp32), M 256 x N 128, into one
//                      of two 128-column S buffers in each CTA's TMEM; each CTA stages 64
//                      of the 128 keys (the B operand is split along N)
//   P_j  = 2^(S_j log2(e) - m)   softmax threads: tcgen05.ld the row, mask (boundary tiles
//                      only), row max m and sum l; P_j (bf16 pairs) is stored back into the
//                      first 64 columns of its S buffer with tcgen05.st
//   O   += P_j V_j     tcgen05.mma with A = P_j read from TMEM, M 256 x N 256, O fp32 in
//                      TMEM; each CTA stages 128 of V's 256 columns
// Splitting both B operands across the pair halves the K / V bytes every SM loads per
// MMA, which is what bounds a single-CTA schedule (its TMA copies, not its MMAs).
// The MMA warp issues S_{j+1} before O += P_j V_j, so while the softmax threads work on
// S_j the tensor cores run O += P_{j-1} V_{j-1} and S_{j+1}; tcgen05.mma operations
// execute in issue order, so S_{j+2} overwrites P_j only after O += P_j V_j read it.
// A row's reference maximum m moves only when the tile maximum exceeds it by more than 8
// (log2 units): P is then <= 2^8, O is rescaled in TMEM (tcgen05.ld / st) only on such
// moves, and the final O / l is the same softmax.  head_dim 512 runs two clusters per row
// block, one per output half, each computing the full S (TMEM holds two S buffers and a
// 256-column O, not a 512-column one).
//
// Shared memory per CTA: its Q rows resident (head_dim / 64 swizzled [128 x 64] blocks)
// and a ring of 16 KB slots of 64 keys x 128 columns (two swizzled [64 x 64] blocks),
// loaded in the order the MMAs consume them: for S the CTA's 64 keys of the tile, 128
// columns of the reduction per slot; for O its 128 columns of V, 64 keys per slot.  Every
// mbarrier wait is bounded; on a timeout the kernel records W8_ERR_DEVICE_TIMEOUT, drains
// its own copies and MMAs, frees TMEM and returns.
#include "common.cuh"
#include "rowquant.cuh"

#include <algorithm>
#include <mutex>

namespace w8 {

__device__ int g_attn_status = 0;

constexpr int kTcBM = 128;                  // rows per CTA (TMEM lanes); 256 per pair
constexpr int kTcBN = 128;                  // keys per tile
constexpr int kTcDV = 256;                  // output columns per pair
constexpr int kTcSoftWarps = 8;             // two per TMEM lane quarter, 64 keys each
constexpr int kTcThreads = 32 * (2 + kTcSoftWarps);  // TMA warp, MMA warp, softmax warps
constexpr int kSlotBytes = 32768;           // K: 64 keys x 256 columns; V: 128 keys x 128 columns
constexpr int kKeysPerCta = kTcBN / 2;      // keys of a tile each CTA stages for S
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 2 * kTcBN;       // S buffers at columns 0 and 128, O from 256

template <int D>
struct TcCfg {
  static constexpr int kQBytes = kTcBM * D * 2;
  static constexpr int kSlots = D == 256 ? 5 : 3;
  static constexpr int kKSlots = D / 256;                // slots per K tile (per CTA)
  static constexpr int kOffRing = kQBytes;
  static constexpr int kOffBar = kOffRing + kSlots * kSlotBytes;
  // full[kSlots], empty[kSlots], q_full, s_full[2], p_full[2], pv_done[2], o_ready
  static constexpr int kNumBars = 2 * kSlots + 8;
  static constexpr int kOffXch = kOffBar + kNumBars * 8 + 16;  // float [2][128]: the partner's row max / sum
  static constexpr int kSmem = kOffXch + 2 * kTcBM * 4 + 1024;
  static_assert(kSmem <= 232448, "shared memory budget exceeded");
};

struct AttnTcArgs {
  __nv_bfloat16* o;
  int64_t o_head, o_tok;
  int t, heads, kv_heads, window;
  int pack;  // heads per CTA (PK); 128 / PK queries per CTA
  // k_attn_out fused (head_dim 256, PK = heads): the per-token _quant of the output rows,
  // q [T, heads * 256] int8 (row pitch ldq) and s [T] fp32, instead of o.
  int8_t* q;
  int64_t ldq;
  float* s;
};

// kind::f16 instruction descriptor: bf16 A and B, fp32 D, M x N, A K-major, B K- or MN-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n, bool b_mn_major) {
  return (1u << 4)                                 // D format: F32
         | (1u << 7)                               // A format: BF16
         | (1u << 10)                              // B format: BF16
         | ((b_mn_major ? 1u : 0u) << 16)          // B major
         | (static_cast<uint32_t>(n >> 3) << 17)   // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);  // M / 16
}

// Pair MMA, D[tmem] (+)= A[smem desc] * B[smem desc], bf16 -> fp32; the descriptors name
// the same shared-memory offsets in both CTAs.
__device__ __forceinline__ void mma_bf16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Pair MMA with A read from TMEM: each CTA's A rows in its lanes, K packed two bf16 per
// 32-bit column.
__device__ __forceinline__ void mma_bf16_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 4-D tiled load (plain, one destination CTA) into this CTA's shared memory, completion counted on `bar`,
// a shared::cluster barrier address that may lie in the peer CTA.
__device__ __forceinline__ void tma_load_4d_pair(uint32_t dst, const CUtensorMap* m, uint32_t bar, int x, int y,
                                                 int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// 4-D tiled store shared -> global (bulk-group completion); the box is clipped at the
// tensor bounds.  Coordinates are non-negative and x = 0.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* m, uint32_t src, int x, int y, int z, int w) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(src), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}

// Warp-wide registers -> TMEM, the inverse of tmem_ld_32x32b_x32.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// mbar_wait_bounded with a non-blocking probe first: a phase that completed already costs
// one test instead of a suspended try-wait.
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0 || mbar_wait_bounded(bar, parity, abort_flag, status);
}

__device__ __forceinline__ float ex2_tc(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h2 = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h2);
}

template <int D>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTcThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                        const AttnTcArgs a) {
  using C = TcCfg<D>;
  constexpr int kSplit = D / kTcDV;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw);
  const uint32_t ring = base + C::kOffRing;
  const uint32_t bar0 = base + C::kOffBar;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffBar + C::kNumBars * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto full_bar = [&](uint32_t s) { return bar0 + 8u * s; };
  auto empty_bar = [&](uint32_t s) { return bar0 + 8u * (C::kSlots + s); };
  const uint32_t q_full = bar0 + 8u * (2 * C::kSlots);
  auto s_full = [&](int b) { return q_full + 8u * (1 + b); };
  auto p_full = [&](int b) { return q_full + 8u * (3 + b); };
  auto pv_done = [&](int b) { return q_full + 8u * (5 + b); };
  const uint32_t o_ready = q_full + 8u * 7;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = the CTA that issues the MMAs
  const uint32_t peer = rank ^ 1u;
  const int pk = a.pack, qb_rows = kTcBM / pk;
  // Heaviest row blocks first: pair ids run over (head group, half) fastest.
  const int per_pair = (a.heads / pk) * kSplit;
  const int npairs = (gridDim.x >> 1) / per_pair;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int pb = npairs - 1 - pair / per_pair;
  const int rest = pair % per_pair;
  const int hg = rest / kSplit, half = rest % kSplit;
  const int pq0 = pb * 2 * qb_rows;                           // first query of the pair
  const int q0 = pq0 + static_cast<int>(rank) * qb_rows;      // first query of this CTA
  const int head0 = hg * pk;
  const int kvh = head0 / (a.heads / a.kv_heads);
  const int last_key = min(pq0 + 2 * qb_rows, a.t) - 1;      // the pair shares its key tiles
  const int first_key = a.window > 0 ? max(0, pq0 - a.window + 1) : 0;
  const int kt0 = first_key / kTcBN;
  const int ntiles = last_key / kTcBN - kt0 + 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kSlots; ++s) {
      mbar_init(full_bar(s), 1);   // leader: one arrive.expect_tx + both CTAs' bytes
      mbar_init(empty_bar(s), 1);  // both: one MMA commit
    }
    mbar_init(q_full, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(s_full(b), 1);
      mbar_init(p_full(b), 2 * kTcSoftWarps);  // leader: the softmax warps of both CTAs
      mbar_init(pv_done(b), 1);
    }
    mbar_init(o_ready, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    prefetch_tmap(&tm_o);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  // Programmatic dependent launch: the setup above overlapped the previous kernel's tail;
  // q, k, v (its output) are read only from here on.
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer (both CTAs): Q once, then the ring in the MMA order; every copy
      // completes on the leader's barrier, which expects both CTAs' bytes.
      const uint32_t q_full_l = mapa_shared(q_full, 0);
      if (rank == 0) mbar_arrive_expect_tx(q_full, 2 * C::kQBytes);
      tma_load_4d_pair(base, &tm_q, q_full_l, 0, q0, head0, 0);
      uint32_t g = 0;
      bool ok = true;
      auto put = [&](const CUtensorMap* m, int key0, int block0) {
        if (!ok) return;
        const uint32_t slot = g % C::kSlots, use = g / C::kSlots;
        ok = wait_phase(empty_bar(slot), (use & 1u) ^ 1u, abort_flag, &g_attn_status);
        if (!ok) return;
        if (rank == 0) mbar_arrive_expect_tx(full_bar(slot), 2 * kSlotBytes);
        tma_load_4d_pair(ring + slot * kSlotBytes, m, mapa_shared(full_bar(slot), 0), 0, key0, block0, kvh);
        ++g;
      };
      // K: this CTA's 64 keys of the tile, 256 columns of the reduction per slot.  V: all
      // 128 keys of the tile, this CTA's 128 of the half's 256 columns.
      const int kk0 = static_cast<int>(rank) * kKeysPerCta;
      const int vb0 = half * (kTcDV / 64) + static_cast<int>(rank) * 2;
      for (int c = 0; c < C::kKSlots; ++c) put(&tm_k, kt0 * kTcBN + kk0, 4 * c);
      for (int i = 0; i < ntiles && ok; ++i) {
        if (i + 1 < ntiles)
          for (int c = 0; c < C::kKSlots; ++c) put(&tm_k, (kt0 + i + 1) * kTcBN + kk0, 4 * c);
        put(&tm_v, (kt0 + i) * kTcBN, vb0);
      }
      // Every copy issued was awaited by the leader's MMA thread unless a wait gave up
      // (after seconds); then give the last copies time to land before the CTA may exit.
      if (!ok) {
        const unsigned long long t0 = globaltimer();
        while (globaltimer() - t0 < 50000ull) {
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      // ---- MMA issuer (leader CTA only)
      constexpr uint32_t id_s = idesc_bf16(2 * kTcBM, kTcBN, false);
      constexpr uint32_t id_o = idesc_bf16(2 * kTcBM, kTcDV, true);
      const uint32_t empty_p0 = mapa_shared(empty_bar(0), peer);
      const uint32_t s_full_p0 = mapa_shared(s_full(0), peer);
      const uint32_t pv_done_p0 = mapa_shared(pv_done(0), peer);
      // Descriptors of the operand bases; an offset of o bytes adds o / 16 (no carry out of
      // the 14-bit address field below 256 KB).
      const uint64_t q_desc = smem_desc_sw128(base, 16, 1024);
      const uint64_t k_desc = smem_desc_sw128(ring, 16, 1024);
      const uint64_t v_desc = smem_desc_sw128(ring, kTcBN * 128, 1024);
      uint32_t g = 0;
      bool ok = wait_phase(q_full, 0, abort_flag, &g_attn_status);
      auto take = [&]() {
        const uint32_t slot = g % C::kSlots, use = g / C::kSlots;
        ok = ok && wait_phase(full_bar(slot), use & 1u, abort_flag, &g_attn_status);
        return slot;
      };
      auto release = [&](uint32_t slot) {
        mma_commit_pair(empty_bar(slot));
        mma_commit_pair(empty_p0 + 8u * slot);
        ++g;
      };
      // S_i into buffer i % 2.  Buffer i % 2 last held P_{i-2}, read by O += P_{i-2} V_{i-2},
      // which this thread issued earlier (MMAs execute in issue order).
      auto issue_s = [&](int i) {
        const int b = i & 1;
        for (int c = 0; c < C::kKSlots && ok; ++c) {
          const uint32_t slot = take();
          if (!ok) return;
          tc_fence_after();
          // Slot: 4 blocks of [64 keys x 64 columns]; Q block 4 c + h holds the same columns.
#pragma unroll
          for (int h = 0; h < 4; ++h)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_bf16_ss_pair(tmem + b * kTcBN, q_desc + (((4 * c + h) * (kTcBM * 128) + kk * 32) >> 4),
                               k_desc + ((slot * kSlotBytes + h * (kKeysPerCta * 128) + kk * 32) >> 4), id_s,
                               (c | h | kk) ? 1u : 0u);
          release(slot);
        }
        if (ok) {
          mma_commit_pair(s_full(b));
          mma_commit_pair(s_full_p0 + 8u * b);
        }
      };
      issue_s(0);
      for (int i = 0; i < ntiles && ok; ++i) {
        if (i + 1 < ntiles) issue_s(i + 1);
        const int b = i & 1;
        ok = ok && wait_phase(p_full(b), (i >> 1) & 1, abort_flag, &g_attn_status);
        const uint32_t slot = take();
        if (!ok) break;
        tc_fence_after();
        // A = P keys [16 s, 16 s + 16): TMEM columns b * 128 + 8 s (bf16 pairs).  B = V
        // [16 keys x 128 columns] per CTA, MN-major: the two 64-column blocks 16 KB apart
        // (LBO), 8-key groups 1 KB apart (SBO); the next 16 keys 2 KB further.
#pragma unroll
        for (int s = 0; s < kTcBN / 16; ++s)
          mma_bf16_ts_pair(tmem + kColO, tmem + b * kTcBN + 8 * s, v_desc + ((slot * kSlotBytes + s * 16 * 128) >> 4),
                           id_o, (i | s) ? 1u : 0u);
        release(slot);
        mma_commit_pair(pv_done(b));
        mma_commit_pair(pv_done_p0 + 8u * b);
      }
      mma_commit_pair(o_ready);
      mma_commit_pair(mapa_shared(o_ready, peer));
      // Drain: no MMA may still write TMEM when it is freed.
      mbar_wait_bounded(o_ready, 0, nullptr, &g_attn_status);
    }
  } else {
    // ---- softmax (both CTAs): row r = TMEM lane r is shared by warps w and w + 4 (warp w
    // may access lanes 32 (w % 4) ..), each taking 64 of the tile's 128 keys and 128 of
    // the 256 output columns; the two exchange their row maxima (and at the end their
    // sums) through shared memory under a 64-thread named barrier.
    const int quarter = warp & 3;
    const int hv = (warp - 2) >> 2;  // which half of the keys / output columns
    const int r = quarter * 32 + lane;
    const int qpos = q0 + r % qb_rows;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t p_full_l0 = mapa_shared(p_full(0), 0);
    volatile float* xch = reinterpret_cast<volatile float*>(smem + C::kOffXch);
    auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory"); };
    constexpr float kLog2e = 1.4426950408889634f;
    float m = -INFINITY, l = 0.f;  // m in log2 units, l over this warp's keys
    bool ok = true;
    // Every warp runs every iteration and meets its partner at the same pair barriers on
    // every path: after a timeout it only skips its waits and its work.
    for (int i = 0; i < ntiles; ++i) {
      const int b = i & 1, k0 = (kt0 + i) * kTcBN;
      if (ok) ok = mbar_wait_bounded(s_full(b), (i >> 1) & 1, abort_flag, &g_attn_status);
      // O += P_{i-2} V_{i-2} has completed (it ran before S_i); observing it keeps the
      // phase of pv_done(b) known for the wait on O += P_{i-1} V_{i-1} below.
      if (ok && i >= 2) ok = mbar_wait_bounded(pv_done(b), ((i - 2) >> 1) & 1, abort_flag, &g_attn_status);
      ok = __all_sync(0xffffffffu, ok);
      uint32_t sv[2][32];
      float mx = -INFINITY;
      if (ok) {
        tc_fence_after();
        tmem_ld_32x32b_x32(tmem + lane_off + b * kTcBN + 64 * hv, sv[0]);
        tmem_ld_32x32b_x32(tmem + lane_off + b * kTcBN + 64 * hv + 32, sv[1]);
        tmem_wait_ld();
        // Boundary tiles (causal diagonal, window edge, keys past T) are masked per element.
        const bool interior = k0 + kTcBN - 1 <= q0 && k0 + kTcBN <= a.t &&
                              (a.window == 0 || k0 >= q0 + qb_rows - a.window);
        if (!interior) {
          const int hi = min(qpos, a.t - 1) - k0 - 64 * hv;  // valid keys: lo <= key <= hi
          const int lo = a.window > 0 ? qpos - a.window + 1 - k0 - 64 * hv : -1;
          // The valid keys as one bit per column of each 32-column half, so that each
          // element takes one bit test instead of two range compares.
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int l = max(lo - 32 * j, 0), h = min(hi - 32 * j, 31);
            const uint32_t keep = h < l ? 0u : (0xFFFFFFFFu >> (31 - h)) & (0xFFFFFFFFu << l);
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (!((keep >> c) & 1u)) sv[j][c] = __float_as_uint(-INFINITY);
          }
        }
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < 64; ++c) m4[c & 3] = fmaxf(m4[c & 3], __uint_as_float(sv[c >> 5][c & 31]));
        mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      }
      xch[hv * kTcBM + r] = mx;
      tc_fence_before();
      pair_sync();  // both halves of S are in registers and both maxima are posted
      tc_fence_after();
      mx = fmaxf(mx, xch[(hv ^ 1) * kTcBM + r]);
      pair_sync();  // the partner's maximum is read before either posts the next one
      if (!ok) continue;
      const float mt = mx * kLog2e;
      const bool move = mt > m + 8.f;
      if (__any_sync(0xffffffffu, move)) {
        const float mn = move ? mt : m;
        const float corr = move ? ex2_tc(m - mn) : 1.f;  // m = -inf: 0 (O and l are still 0)
        if (i > 0) {
          // O must hold tiles < i before it is rescaled: wait for O += P_{i-1} V_{i-1}.
          ok = mbar_wait_bounded(pv_done((i - 1) & 1), ((i - 1) >> 1) & 1, abort_flag, &g_attn_status);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) continue;
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < kTcDV / 64; ++c) {
            uint32_t ov[32];
            const uint32_t col = kColO + 128 * hv + c * 32;
            tmem_ld_32x32b_x32(tmem + lane_off + col, ov);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * corr);
            tmem_st_32x32b_x32(tmem + lane_off + col, ov);
          }
        }
        l *= corr;
        m = mn;
      }
      const float ref = m == -INFINITY ? 0.f : m;
      // P (bf16 pairs) of this warp's 64 keys into columns [32 hv, 32 hv + 32) of the S
      // buffer: S values both warps already hold in registers (first pair barrier).
      float l4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pw[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const float p0 = ex2_tc(fmaf(__uint_as_float(sv[e >> 4][(2 * e) & 31]), kLog2e, -ref));
        const float p1 = ex2_tc(fmaf(__uint_as_float(sv[e >> 4][(2 * e + 1) & 31]), kLog2e, -ref));
        l4[e & 3] += p0 + p1;
        pw[e] = pack_bf16x2(p0, p1);
      }
      tmem_st_32x32b_x32(tmem + lane_off + b * kTcBN + 32 * hv, pw);
      l += (l4[0] + l4[1]) + (l4[2] + l4[3]);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      // P is TMEM data, complete (tcgen05.wait::st) and fenced above: the peer's warps
      // arrive on the leader's barrier with no cluster-scope release of generic memory.
      if (lane == 0) {
        if (rank == 0)
          mbar_arrive(p_full(b));
        else
          mbar_arrive_tmem_handoff(p_full_l0 + 8u * b);
      }
    }
    if (ok) ok = mbar_wait_bounded(o_ready, 0, abort_flag, &g_attn_status);
    const bool good = __all_sync(0xffffffffu, ok);
    // The row sum over both halves of the keys (the pair barriers stay matched on every path).
    xch[hv * kTcBM + r] = l;
    pair_sync();
    const float lt = l + xch[(hv ^ 1) * kTcBM + r];
    auto softmax_sync = [&]() { asm volatile("bar.sync 5, %0;" ::"n"(32 * kTcSoftWarps) : "memory"); };
    if (a.q != nullptr) {
      // ---- k_attn_out fused (pipeline.py:88-92): every head of each of this CTA's tokens is
      // one of its rows, so the token's _quant over heads * 256 values happens here: the
      // bf16 output values (the ones o would hold), max |.| per token through shared
      // memory, then the int8 codes with _quant's scale and rounding.
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      uint32_t pw[64];  // this thread's 128 bf16 output values, packed pairs
      uint32_t am2 = 0u;  // max |.| in two bf16 lanes
      if (good) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < kTcDV / 64; ++c) {
          uint32_t ov[32];
          tmem_ld_32x32b_x32(tmem + lane_off + kColO + 128 * hv + c * 32, ov);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float v0 = __uint_as_float(ov[2 * e]) * inv, v1 = __uint_as_float(ov[2 * e + 1]) * inv;
            pw[16 * c + e] = pack_bf16x2(v0, v1);
          }
#pragma unroll
          for (int e = 0; e < 4; ++e)
            am2 = bf16x2_absmax8(make_uint4(pw[16 * c + 4 * e], pw[16 * c + 4 * e + 1], pw[16 * c + 4 * e + 2],
                                            pw[16 * c + 4 * e + 3]),
                                 am2);
        }
      }
      const float am = bf16x2_max_lanes(am2);
      const int qi = r % qb_rows, slot = (r / qb_rows) * 2 + hv;  // token, (head, half)
      softmax_sync();  // every row sum above is read before xch is reused
      xch[qi * 2 * pk + slot] = am;
      softmax_sync();
      float tam = 0.f;
      for (int i = 0; i < 2 * pk; ++i) tam = fmaxf(tam, xch[qi * 2 * pk + i]);
      const float sc = __fdiv_rn(fmaxf(tam, 1e-8f), 127.f);
      const float rc = __frcp_rn(sc);
      if (good && qpos < a.t) {
        const int head = head0 + r / qb_rows;
        int8_t* dst = a.q + static_cast<int64_t>(qpos) * a.ldq + head * kTcDV + 128 * hv;
#pragma unroll
        for (int j = 0; j < 8; ++j) {  // 16 values -> 16 bytes
          const uint2 lo = quant8_bf16_codes(make_uint4(pw[8 * j], pw[8 * j + 1], pw[8 * j + 2], pw[8 * j + 3]), sc, rc);
          const uint2 hi =
              quant8_bf16_codes(make_uint4(pw[8 * j + 4], pw[8 * j + 5], pw[8 * j + 6], pw[8 * j + 7]), sc, rc);
          *reinterpret_cast<uint4*>(dst + 16 * j) = make_uint4(lo.x, lo.y, hi.x, hi.y);
        }
        if (slot == 0) a.s[qpos] = sc;
      }
    } else {
      // ---- O / l -> bf16 rows staged in shared memory (the ring is idle once O is final)
      // in the output map's box layout, then one TMA store (rows past T are clipped).
      if (good) {
        tc_fence_after();
        const float inv = lt > 0.f ? 1.f / lt : 0.f;
#pragma unroll 1
        for (int c = 0; c < kTcDV / 64; ++c) {
          uint32_t ov[32];
          const int col = 128 * hv + c * 32;  // this warp's columns col .. col + 31
          tmem_ld_32x32b_x32(tmem + lane_off + kColO + col, ov);
          tmem_wait_ld();
          // block col / 64, 16-byte chunks 4 (col / 32 % 2) .. + 3
          const uint32_t row = ring + (col >> 6) * (kTcBM * 128) + r * 128;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              w[e] = pack_bf16x2(__uint_as_float(ov[8 * j + 2 * e]) * inv,
                                 __uint_as_float(ov[8 * j + 2 * e + 1]) * inv);
            const int chunk = 4 * ((col >> 5) & 1) + j;
            st_shared_v4(row + ((chunk ^ (r & 7)) << 4), w[0], w[1], w[2], w[3]);
          }
        }
        fence_proxy_async_smem();
      }
      // All softmax warps meet here on every path; the tile is stored only if each of them
      // staged its rows.
      uint32_t all_good;
      asm volatile(
          "{\n\t.reg .pred p, q;\n\t"
          "setp.ne.u32 q, %1, 0;\n\t"
          "bar.red.and.pred p, 5, %2, q;\n\t"
          "selp.u32 %0, 1, 0, p;\n\t}"
          : "=r"(all_good)
          : "r"(good ? 1u : 0u), "n"(32 * kTcSoftWarps)
          : "memory");
      if (all_good && warp == 2 && lane == 0) {
        tma_store_4d(&tm_o, ring, 0, q0, head0, half * (kTcDV / 64));
        bulk_commit_group();
        bulk_wait_group<0>();
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still touch its barriers, TMEM or copies
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

}  // namespace w8

namespace w8host {

using AttnEncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static AttnEncodeFn attn_encode_fn() {
  static AttnEncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AttnEncodeFn>(p);
  });
  return fn;
}

// 4-D tiled map over a head-major bf16 tensor (element (h, t, d) at ptr[h * ld_head +
// t * ld_tok + d]) with 128-byte swizzled boxes of 64 columns.  kv layout: dimensions
// (64 columns, token, 64-column block, head); a box {64, rows, blocks, 1} lands in shared
// memory as `blocks` consecutive [rows x 64] blocks.  q layout: dimensions (64 columns,
// token, head, 64-column block); a box {64, rows, heads, blocks} lands as `blocks`
// consecutive [heads * rows x 64] blocks, row = head * rows + token.
static int encode_heads(CUtensorMap* map, const void* ptr, int64_t d, int64_t heads, int64_t t, int64_t ld_head,
                        int64_t ld_tok, bool q_layout, uint32_t rows, uint32_t box_heads, uint32_t blocks) {
  AttnEncodeFn enc = attn_encode_fn();
  if (enc == nullptr) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return W8_ERR_CUDA;
  }
  const cuuint64_t tok_stride = static_cast<cuuint64_t>(ld_tok * 2), head_stride = static_cast<cuuint64_t>(ld_head * 2);
  cuuint64_t dims[4], strides[3];
  cuuint32_t box[4];
  dims[0] = 64;
  dims[1] = static_cast<cuuint64_t>(t);
  strides[0] = tok_stride;
  box[0] = 64;
  box[1] = rows;
  if (q_layout) {
    dims[2] = static_cast<cuuint64_t>(heads), dims[3] = static_cast<cuuint64_t>(d / 64);
    strides[1] = head_stride, strides[2] = 128;
    box[2] = box_heads, box[3] = blocks;
  } else {
    dims[2] = static_cast<cuuint64_t>(d / 64), dims[3] = static_cast<cuuint64_t>(heads);
    strides[1] = 128, strides[2] = head_stride;
    box[2] = blocks, box[3] = 1;
  }
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (attention, 4-D) failed with CUresult %d (t %lld, ld_tok %lld, ld_head %lld)",
              static_cast<int>(r), static_cast<long long>(t), static_cast<long long>(ld_tok),
              static_cast<long long>(ld_head));
    return W8_ERR_CUDA;
  }
  return W8_OK;
}

template <int D>
static int attention_tc_go(const uint16_t* q, int64_t q_head, int64_t q_tok, const uint16_t* k, int64_t k_head,
                           int64_t k_tok, const uint16_t* v, int64_t v_head, int64_t v_tok, uint16_t* o,
                           int64_t o_head, int64_t o_tok, int64_t t, int64_t heads, int64_t kv_heads,
                           int64_t window, int device, cudaStream_t stream, int8_t* xq = nullptr,
                           int64_t ldq = 0, float* xs = nullptr) {
  using C = w8::TcCfg<D>;
  // Heads per CTA: the largest power of two <= 16 dividing the query-group size.
  const int64_t group = heads / kv_heads;
  const int pack = static_cast<int>(std::min<int64_t>(group & -group, 16));
  const uint32_t rows = static_cast<uint32_t>(w8::kTcBM / pack);
  CUtensorMap tq, tk, tv;
  int st = encode_heads(&tq, q, D, heads, t, q_head, q_tok, true, rows, static_cast<uint32_t>(pack), D / 64);
  if (st != W8_OK) return st;
  st = encode_heads(&tk, k, D, kv_heads, t, k_head, k_tok, false, w8::kKeysPerCta, 1, 4);
  if (st != W8_OK) return st;
  st = encode_heads(&tv, v, D, kv_heads, t, v_head, v_tok, false, w8::kTcBN, 1, 2);
  if (st != W8_OK) return st;
  CUtensorMap to;
  st = encode_heads(&to, o, D, heads, t, o_head, o_tok, true, rows, static_cast<uint32_t>(pack), w8::kTcDV / 64);
  if (st != W8_OK) return st;
  static bool done[64] = {};
  if (device < 0 || device >= 64) return W8_ERR_UNSUPPORTED;
  if (!done[device]) {
    W8_CUDA_TRY(cudaFuncSetAttribute(w8::attention_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     C::kSmem));
    done[device] = true;
  }
  w8::AttnTcArgs a;
  a.o = reinterpret_cast<__nv_bfloat16*>(o);
  a.o_head = o_head;
  a.o_tok = o_tok;
  a.t = static_cast<int>(t);
  a.heads = static_cast<int>(heads);
  a.kv_heads = static_cast<int>(kv_heads);
  a.window = static_cast<int>(window);
  a.pack = pack;
  a.q = xq;
  a.ldq = ldq;
  a.s = xs;
  // Two CTAs (a cluster) per 2 * rows queries, head group and output half.
  const int64_t blocks = 2 * ((t + 2 * rows - 1) / (2 * rows)) * (heads / pack) * (D / w8::kTcDV);
  W8_CHECK_ARG(blocks < (1ll << 31), "too many query blocks");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks), 1, 1);
  cfg.blockDim = dim3(w8::kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, w8::attention_tc_kernel<D>, tq, tk, tv, to, a));
}

// The tcgen05 schedule of w8_attention_prefill_bf16 (arguments checked by the caller).
int attention_tc(const uint16_t* q, int64_t q_head, int64_t q_tok, const uint16_t* k, int64_t k_head,
                 int64_t k_tok, const uint16_t* v, int64_t v_head, int64_t v_tok, uint16_t* o, int64_t o_head,
                 int64_t o_tok, int64_t t, int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t window,
                 int device, cudaStream_t stream) {
  if (head_dim == 256)
    return attention_tc_go<256>(q, q_head, q_tok, k, k_head, k_tok, v, v_head, v_tok, o, o_head, o_tok, t, heads,
                                kv_heads, window, device, stream);
  return attention_tc_go<512>(q, q_head, q_tok, k, k_head, k_tok, v, v_head, v_tok, o, o_head, o_tok, t, heads,
                              kv_heads, window, device, stream);
}

// Whether attention_tc_quant takes a shape: head_dim 256 and every head of a token in one
// CTA (one KV head, heads a power of two <= 16).
bool attention_tc_quant_fits(int64_t heads, int64_t kv_heads, int64_t head_dim) {
  return head_dim == 256 && kv_heads == 1 && heads >= 1 && heads <= 16 && (heads & (heads - 1)) == 0;
}

// Attention with k_attn_out fused (arguments checked by the caller, the shape fits): the
// int8 rows q [T, heads * 256] (pitch ldq) and scales s [T] instead of the bf16 output.
int attention_tc_quant(const uint16_t* q, int64_t q_head, int64_t q_tok, const uint16_t* k, int64_t k_head,
                       int64_t k_tok, const uint16_t* v, int64_t v_head, int64_t v_tok, int64_t t, int64_t heads,
                       int64_t kv_heads, int64_t window, int8_t* xq, int64_t ldq, float* xs, int device,
                       cudaStream_t stream) {
  // The output tensor map is never used on this path: it is encoded over q (valid bf16).
  return attention_tc_go<256>(q, q_head, q_tok, k, k_head, k_tok, v, v_head, v_tok, const_cast<uint16_t*>(q), q_head,
                              q_tok, t, heads, kv_heads, window, device, stream, xq, ldq, xs);
}

// Read (and optionally clear) the attention kernel's sticky device status.
int attention_device_status(int clear, int* out) {
  int v = 0;
  W8_CUDA_TRY(cudaMemcpyFromSymbol(&v, w8::g_attn_status, sizeof(int)));
  if (clear) {
    const int zero = 0;
    W8_CUDA_TRY(cudaMemcpyToSymbol(w8::g_attn_status, &zero, sizeof(int)));
  }
  *out = v;
  return W8_OK;
}

}  // namespace w8host
