// Device-side helpers shared by the W8A8 kernels: inline PTX for mbarriers, TMA,
// tcgen05 (TMEM alloc / MMA / commit / load) and bounded waits, plus the host-side
// status plumbing of the C ABI.
//
// Every wait on an mbarrier is bounded by %globaltimer: a wait that runs past
// kWaitTimeoutNs records W8_ERR_DEVICE_TIMEOUT in the caller's device status word and
// returns false, and the caller unwinds (waits for its own copies in flight, frees
// TMEM) instead of spinning forever.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/w8a8_b200.h"

namespace w8 {

constexpr unsigned long long kWaitTimeoutNs = 2000000000ull;  // 2 s; kernels here run for < 10 ms

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- programmatic dependent launch
// Kernels here are launched with programmatic stream serialization: the next kernel on
// the stream may be scheduled before this one ends.  launch_dependents allows that;
// grid_dependency_wait blocks until every prerequisite grid has completed and its
// memory is visible, so each kernel calls it before its first global-memory access.
// Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase of `bar` with the given parity to complete.
// `abort_flag` (shared memory) lets one role that gave up release the others early;
// `status` is the sticky device-side error word of the calling kernel's unit.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  volatile int* abort_flag, int* status) {
#pragma unroll 1
  for (int i = 0; i < 256; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
#pragma unroll 1
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort_flag != nullptr && *abort_flag) return false;
    if (globaltimer() - t0 > kWaitTimeoutNs) {
      atomicExch(status, W8_ERR_DEVICE_TIMEOUT);
      if (abort_flag != nullptr) *abort_flag = 1;
      return false;
    }
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// 2-D tiled bulk tensor load global -> shared, completion counted on `bar` in bytes.
// x is the innermost (contiguous) coordinate in elements, y the row coordinate.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* m, uint32_t bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// 2-D tiled bulk tensor store shared -> global (bulk-group completion); the box is
// clipped at the tensor bounds.  x (innermost coordinate) * element size must be a
// multiple of 16 bytes and neither coordinate may be negative.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, uint32_t src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
// 3-D tiled bulk tensor store (innermost coordinate x, then y, then z), clipped at the
// tensor bounds; the same alignment rule on x as the 2-D store.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* m, uint32_t src, int32_t x, int32_t y, int32_t z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(src), "r"(x), "r"(y), "r"(z)
               : "memory");
}
// Same box, added element-wise into global memory (s32 add for an INT32 tensor map);
// performed at L2, so concurrent adds from other CTAs combine exactly.
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* m, uint32_t src, int32_t x,
                                                  int32_t y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
// Order this thread's earlier generic-proxy global accesses before its later async-proxy ones.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Bounded spin until *p >= target (gpu-scope acquire); false (and a status) after
// `limit_ns` nanoseconds.
__device__ __forceinline__ bool wait_counter_bounded(const uint32_t* p, uint32_t target, int* status,
                                                     unsigned long long limit_ns = kWaitTimeoutNs) {
#pragma unroll 1
  for (int i = 0; i < 64; ++i)
    if (ld_acquire_gpu(p) >= target) return true;
  const unsigned long long t0 = globaltimer();
#pragma unroll 1
  while (true) {
    if (ld_acquire_gpu(p) >= target) return true;
    __nanosleep(64);
    if (globaltimer() - t0 > limit_ns) {
      atomicExch(status, W8_ERR_DEVICE_TIMEOUT);
      return false;
    }
  }
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until at most N of this thread's bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until at most N of this thread's bulk groups are still in flight.
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// Make generic-proxy shared-memory writes visible to the async proxy (TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Warp-wide: allocate `ncols` TMEM columns (power of two >= 32); the address lands in smem.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], int8 x int8 -> int32.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// Warp-wide TMEM -> registers: lane i of the warp reads TMEM lane (taddr.lane + i),
// 32 consecutive 32-bit columns starting at taddr.col.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- CTA pairs (cta_group::2)
// A cluster of two CTAs on two SMs shares one 256-row MMA: each CTA holds half of A
// and half of B in its own shared memory; one thread of the even CTA issues the MMA.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// All threads of both CTAs: release our writes, wait for the peer's.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// Arrive on an mbarrier in this CTA or the peer CTA of the pair when what the waiter needs
// is TMEM that this thread's tcgen05 loads or stores touched: tcgen05.wait has completed
// them and tcgen05.fence::before_thread_sync orders them before the arrive, and the waiter
// issues its tcgen05 operations after tcgen05.fence::after_thread_sync.  No generic memory
// is handed over, so the arrive keeps the default CTA-scope release: a cluster-scope release
// first drains this thread's outstanding memory operations (about 1000 cycles measured
// here, on the critical path of every tile).
__device__ __forceinline__ void mbar_arrive_tmem_handoff(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on `bar`, a
// shared::cluster barrier address that may lie in the peer CTA of the pair.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* m, uint32_t bar,
                                                 int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
// The same for a 3-D box: {x, y, z} with x innermost.  A K-major operand viewed as
// (128-byte K chunk, row, chunk index) lands as [chunk][row][128 B]: consecutive
// swizzle-128 K blocks, so one copy brings several K blocks of the same rows.
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* m, uint32_t bar,
                                                 int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the barrier at shared::cluster address `bar` when every pair MMA
// issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// Shared-memory matrix descriptor for tcgen05 (SM100 format, version 1) with the
// 128-byte swizzle. Offsets are in bytes; the 4 low bits are dropped by the format.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version for tcgen05
  d |= 2ull << 61;  // layout: SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::i8: signed A and B, int32 accumulator, M x N tile.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n, bool b_mn_major) {
  return (2u << 4)                               // D format: S32
         | (1u << 7)                             // A format: signed int8
         | (1u << 10)                            // B format: signed int8
         | (0u << 15)                            // A K-major
         | ((b_mn_major ? 1u : 0u) << 16)        // B major
         | (static_cast<uint32_t>(n >> 3) << 17) // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);  // M / 16
}

// ---------------------------------------------------------------- packed f32x2
// Two fp32 values in one 64-bit register pair, for sm_100's packed f32x2 instructions:
// each lane of a packed mul / add is one IEEE fp32 operation rounded to nearest, so a
// pair of outputs takes one instruction per step and the same bits as two.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// Both values rounded to bf16 (nearest even); returns them as fp32 and sets `bits` to the
// packed bf16 pair.
__device__ __forceinline__ uint64_t f2_round_bf16(uint64_t v, uint32_t& bits) {
  float lo, hi;
  f2_unpack(v, lo, hi);
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  bits = *reinterpret_cast<uint32_t*>(&p);
  return f2_pack(__uint_as_float(bits << 16), __uint_as_float(bits & 0xFFFF0000u));
}

__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// A packed bf16 pair (low half = first element) <-> the fp32 pair, exact both ways for
// bf16 values; the way back rounds to nearest even.
__device__ __forceinline__ uint64_t f2_from_bf16x2(uint32_t w) {
  return f2_pack(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}
__device__ __forceinline__ uint32_t bf16x2_from_f2(uint64_t v) {
  float lo, hi;
  f2_unpack(v, lo, hi);
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&p);
}

// Packed bf16 pair arithmetic, each lane rounded once to bf16 (nearest even).  On bf16
// operands this is exactly what eager torch computes for bf16 tensors, the fp32 result
// rounded to bf16: fp32 holds the product of two bf16 exactly, and for a sum its 24 bits
// (>= 2 * 8 + 2) make the double rounding innocuous (S. A. Figueroa, "When is double
// rounding innocuous?", ACM SIGNUM Newsletter 30(3), 1995).
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2_add(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// ---------------------------------------------------------------- gelu (tanh form)
constexpr float kGeluBeta = 0.7978845608028654f;  // sqrt(2 / pi)
constexpr float kGeluKappa = 0.044715f;

__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// 1 + tanh(z) = 2 / (1 + e^(-2z)), from one ex2.approx and one rcp.approx (relative error
// a few 2^-23).  Like 1 + tanhf(z) in fp32 it is exactly 2 for large z and exactly 0 for
// very negative z (e^(-2z) overflows to +inf, whose reciprocal is 0).
__device__ __forceinline__ float one_plus_tanh(float z) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(__fmul_rn(z, -2.8853900817779268f)));  // -2 log2(e)
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(__fadd_rn(1.f, e)));
  return 2.f * r;
}

// bf16 of F.gelu(g, approximate="tanh") for a bf16 value g: ATen's fp32 operation order
// 0.5 * g * (1 + tanh(sqrt(2/pi) * (g + 0.044715 * g^3))) with every product and sum
// rounded (no FMA contraction), rounded once to bf16 at the end.  Only 1 + tanh comes
// from the approximation above, so the result is the reference's except for a bf16
// rounding flip about once in 10^4 values.
__device__ __forceinline__ float gelu_tanh_bf16(float g) {
  const float g3 = __fmul_rn(__fmul_rn(g, g), g);
  const float inner = __fmul_rn(kGeluBeta, __fadd_rn(g, __fmul_rn(kGeluKappa, g3)));
  return round_bf16(__fmul_rn(__fmul_rn(0.5f, g), one_plus_tanh(inner)));
}

// gelu_tanh_bf16 of a packed bf16 pair, returned packed: the same operations in the same
// order, two values per packed f32x2 step (each lane one IEEE fp32 operation).
__device__ __forceinline__ uint32_t gelu_tanh_bf16x2(uint32_t gbits) {
  const uint64_t g = f2_from_bf16x2(gbits);
  const uint64_t g3 = f2_mul(f2_mul(g, g), g);
  const uint64_t inner = f2_mul(f2_pack(kGeluBeta, kGeluBeta), f2_add(g, f2_mul(f2_pack(kGeluKappa, kGeluKappa), g3)));
  float a0, a1, e0, e1, d0, d1, r0, r1;
  f2_unpack(f2_mul(inner, f2_pack(-2.8853900817779268f, -2.8853900817779268f)), a0, a1);  // -2 log2(e)
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(a0));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(a1));
  f2_unpack(f2_add(f2_pack(1.f, 1.f), f2_pack(e0, e1)), d0, d1);
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(d0));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(d1));
  return bf16x2_from_f2(f2_mul(f2_mul(f2_pack(0.5f, 0.5f), g), f2_mul(f2_pack(2.f, 2.f), f2_pack(r0, r1))));
}

}  // namespace w8

// ---------------------------------------------------------------- host helpers
namespace w8host {

// Map a CUDA runtime error to the C-ABI status and remember its text.
int cuda_status(cudaError_t e);
void set_error(const char* fmt, ...);

#define W8_CHECK_ARG(cond, ...)             \
  do {                                      \
    if (!(cond)) {                          \
      ::w8host::set_error(__VA_ARGS__);     \
      return W8_ERR_INVALID_ARG;            \
    }                                       \
  } while (0)

#define W8_CHECK_ALIGN(cond, ...)           \
  do {                                      \
    if (!(cond)) {                          \
      ::w8host::set_error(__VA_ARGS__);     \
      return W8_ERR_ALIGNMENT;              \
    }                                       \
  } while (0)

#define W8_CUDA_TRY(expr)                                   \
  do {                                                      \
    cudaError_t _e = (expr);                                \
    if (_e != cudaSuccess) return ::w8host::cuda_status(_e); \
  } while (0)

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int num_sms(int* out);

}  // namespace w8host
