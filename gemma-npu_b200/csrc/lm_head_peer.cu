// The column-sharded LM head with its all-gather fused in, over NVLink peer memory.
//
// Reference behaviour replaced: Int8Head.forward (gemma_npu.py:170-172) followed by the
// final logit softcap (pipeline.py:335-338) and the greedy token (gemma_npu.py:291),
// computed on one CPU.  Here the [V, K] head weight is split by rows over the G ranks
// of a node (one process per GPU).  Rank g computes the softcapped fp32 logits of its
// rows with the weight-only int8 GEMV arithmetic of gemv.cu (bit-identical per row) and
// stores each logit straight into every rank's gathered [V] buffer through CUDA IPC
// peer pointers, so the all-gather rides on the GEMV instead of following it as an NCCL
// collective.  Every rank's buffer (one cudaMalloc, shared by IPC handle) holds:
//
//   logits [V padded to 64] fp32 | keys [8] u64 | flags [8] u32 | ready [8] u32 |
//   state [4] u32 (CTAs done, epoch, abort, -) | best [1] u64
//
// One call, at epoch t = (this rank's epoch word) + 1:
//   1. every CTA sets ready[me] = t in every rank's buffer ("I have started call t",
//      which by stream order means I have consumed call t - 1's logits), then waits
//      until every peer's ready[r] here has reached t before it writes into any peer;
//   2. rows as int8_gemv_kernel computes them, each logit stored into all G buffers;
//      each warp folds its greedy key (global row ids) into this rank's best word;
//   3. the last CTA of this rank to finish (a counter) publishes this rank's key into
//      every rank's keys[me], then flags[me] = t (release, system scope), waits until
//      every rank's flag here has reached t (acquire), writes the winning key, resets
//      the counter and stores epoch t.
// When the kernel ends, this rank's buffer holds all V logits.  Every wait is bounded:
// a rank that never arrives makes the others record W8_ERR_DEVICE_TIMEOUT and return
// (nothing is written into a peer that has not signalled ready).  No multicast object
// and no multicast load is used: plain stores to peer memory and flag words.
#include <cstring>

#include "common.cuh"
#include "gemv_rows.cuh"

namespace w8 {

constexpr int kPeerMax = 8;

__device__ int g_peer_status = 0;  // sticky device status of the sharded head

struct PeerHeadArgs {
  int world, me;
  int n, k;    // rows of this rank's shard, K
  int row0;    // global id of the shard's first row
  float cap;
  float* logits[kPeerMax];               // every rank's gathered logits
  unsigned long long* keys[kPeerMax];    // every rank's key slots [kPeerMax]
  uint32_t* flags[kPeerMax];             // every rank's data flags [kPeerMax]
  uint32_t* ready[kPeerMax];             // every rank's ready flags [kPeerMax]
  uint32_t* state;                       // this rank's: [0] CTAs done, [1] epoch, [2] abort
  unsigned long long* best_local;        // this rank's greedy key of the call
  unsigned long long* best;              // output: the greedy key over all ranks (or null)
  int keys_only;                         // 1: only the greedy keys travel; logits stay local
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until every word words[r] (r < world, r != skip) reaches t; false and a
// timeout status (plus the abort word) on expiry, or false at once if the abort word is set.
__device__ __forceinline__ bool wait_all_sys(const uint32_t* words, int world, int skip, uint32_t t,
                                             uint32_t* abort_word) {
  const unsigned long long t0 = globaltimer();
#pragma unroll 1
  for (uint32_t spin = 0;; ++spin) {
    bool all = true;
    for (int r = 0; r < world; ++r)
      if (r != skip && ld_acquire_sys(words + r) < t) all = false;
    if (all) return true;
    if (ld_relaxed_gpu(abort_word) != 0u) return false;
    if (spin > 1024) __nanosleep(100);
    if (globaltimer() - t0 > kWaitTimeoutNs) {
      atomicExch(&g_peer_status, W8_ERR_DEVICE_TIMEOUT);
      atomicExch(abort_word, 1u);
      return false;
    }
  }
}

template <int J, int S, int R>
__global__ void __launch_bounds__(kGemvThreads)
    lm_head_peer_kernel(const __nv_bfloat16* __restrict__ x, const int8_t* __restrict__ w,
                        const __nv_bfloat16* __restrict__ s, const __grid_constant__ PeerHeadArgs a) {
  static_assert(kGemvWarps % S == 0, "S must divide the CTA's warps");
  constexpr int kTeams = kGemvWarps / S;
  __shared__ float red[kTeams][S][R];
  // A CTA finishes kChunk contiguous rows per step; they are sent to the other ranks as
  // 16-byte stores of whole chunks (a 4-byte remote store per logit made the transfer,
  // not the GEMV, the cost).  Two buffers, so a step's stores need one barrier.
  constexpr int kChunk = kTeams * R;
  constexpr bool kVec = kChunk % 4 == 0;
  __shared__ __align__(16) float tile[2][kChunk];
  __shared__ uint32_t s_epoch;
  __shared__ int s_ok;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int team = warp / S;
  const int sl = warp % S;
  const int n = a.n, k = a.k;
  unsigned long long mine = 0ull;
  pdl_launch_dependents();

  const int stride = gridDim.x * kChunk;
  const int cta_first = blockIdx.x * kChunk;
  const int first = cta_first + team * R;
  uint4 wv[R][J];
  auto load_w = [&](int n0) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int c = 0; c < J; ++c) {
        const int k0 = ((sl * J + c) * 32 + lane) * 16;
        const int row = n0 + r;
        wv[r][c] = (row < n && k0 < k) ? ldg_stream(w + static_cast<int64_t>(row) * k + k0)
                                       : make_uint4(0u, 0u, 0u, 0u);
      }
  };
  load_w(first);  // the weights do not depend on the previous kernel
  // The wait in its own basic block (k >= 16 on every launch), so that the weight loads
  // above stay ahead of it (as in int8_gemv_kernel).
  if (k > 0) pdl_wait();

  uint32_t* const abort_word = a.state + 2;
  const bool vec = kVec && a.row0 % 4 == 0;
  const bool send = !a.keys_only;  // the logits go to the other ranks (not for keys only)
  if (threadIdx.x == 0) {
    const uint32_t t = ld_relaxed_gpu(a.state + 1) + 1u;
    // "This rank has started call t": written by every CTA (the same value), so the
    // signal does not depend on which of this rank's CTAs runs first.
    for (int r = 0; r < a.world; ++r) st_relaxed_sys(a.ready[r] + a.me, t);
    s_epoch = t;
    // Rows whose logits go out one by one (no 16-byte chunks) wait for every peer here;
    // chunked rows are computed first and only the sending warp waits, before its first
    // send (by then the peers have started as well).
    s_ok = (vec || !send) ? 1 : (wait_all_sys(a.ready[a.me], a.world, a.me, t, abort_word) ? 1 : 0);
  }
  __syncthreads();
  const bool ok = s_ok != 0;
  const uint32_t epoch = s_epoch;
  bool peers_ready = !vec;  // warp 0's knowledge that every peer has started this call

  // This lane's 16-element pieces of the activation row as 16-bit fixed point.
  uint32_t xh[J][4], xl[J][4];
  float dq[J];
#pragma unroll
  for (int c = 0; c < J; ++c) {
    const int k0 = ((sl * J + c) * 32 + lane) * 16;
    uint32_t words[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
    if (k0 < k) {
      const uint4* p = reinterpret_cast<const uint4*>(x + k0);
      const uint4 u = __ldg(p), v = __ldg(p + 1);
      words[0] = u.x, words[1] = u.y, words[2] = u.z, words[3] = u.w;
      words[4] = v.x, words[5] = v.y, words[6] = v.z, words[7] = v.w;
    }
    dq[c] = piece_codes(words, xh[c], xl[c]);
  }

  int buf = 0;
  bool vec_failed = false;
  // Every thread of the CTA walks the same steps (the barriers below need it); a team
  // whose rows lie past n computes zeros and writes nothing.
  for (int base = cta_first; ok && base < n; base += stride, buf ^= 1) {
    const int n0 = base + team * R;
    if (base != cta_first) load_w(n0);
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float v = 0.f;
#pragma unroll
      for (int c = 0; c < J; ++c) {
        int hi = 0, lo = 0;
        dot16_q(wv[r][c], xh[c], xl[c], hi, lo);
        v = fmaf(static_cast<float>(256 * hi + lo), dq[c], v);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      acc[r] = v;
    }
    float v = 0.f;
    bool writer = false;
    if constexpr (S == 1) {
      v = acc[0];
#pragma unroll
      for (int r = 1; r < R; ++r) v = lane == r ? acc[r] : v;
      writer = lane < R && n0 + lane < n;
    } else {
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < R; ++r) red[team][sl][r] = acc[r];
      }
      asm volatile("bar.sync %0, %1;" ::"r"(1 + team), "r"(S * 32) : "memory");
      if (sl == 0 && lane < R && n0 + lane < n) {
        v = red[team][0][lane];
#pragma unroll
        for (int q = 1; q < S; ++q) v += red[team][q][lane];
        writer = true;
      }
      asm volatile("bar.sync %0, %1;" ::"r"(1 + team), "r"(S * 32) : "memory");
    }
    if (writer) {
      const int row = n0 + lane;
      // write_out's rounding and softcap into this rank's buffer, then to the others
      const float f = write_out<true>(a.logits[a.me], a.row0 + row, v, s[row], a.cap);
      mine = max(mine, argmax_key(f, a.row0 + row));
      if (vec) {
        tile[buf][n0 - base + lane] = f;
      } else if (send) {
        for (int r = 0; r < a.world; ++r)
          if (r != a.me) a.logits[r][a.row0 + row] = f;
      }
    }
    if (vec && send) {
      __syncthreads();
      if (warp == 0 && !peers_ready) {
        bool seen = false;
        if (lane == 0) seen = wait_all_sys(a.ready[a.me], a.world, a.me, epoch, abort_word);
        peers_ready = __shfl_sync(0xffffffffu, seen, 0);
        if (!peers_ready) vec_failed = true;  // the abort word is set: nothing is sent
      }
      if (warp == 0 && !vec_failed) {
        const int valid = min(kChunk, n - base);
        for (int e = 4 * lane; e < kChunk; e += 128) {
          if (e + 4 <= valid) {
            const float4 v4 = *reinterpret_cast<const float4*>(&tile[buf][e]);
            for (int r = 0; r < a.world; ++r)
              if (r != a.me) *reinterpret_cast<float4*>(a.logits[r] + a.row0 + base + e) = v4;
          } else {
            for (int j = e; j < valid; ++j)
              for (int r = 0; r < a.world; ++r)
                if (r != a.me) a.logits[r][a.row0 + base + j] = tile[buf][j];
          }
        }
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mine = max(mine, __shfl_xor_sync(0xffffffffu, mine, o));
  if (lane == 0 && mine != 0ull) atomicMax(a.best_local, mine);

  __syncthreads();
  if (threadIdx.x == 0) {
    // This CTA's stores into every rank's buffer are ordered before its count at GPU
    // scope (the CTA barrier above makes them this thread's to order); the last CTA,
    // having seen every count, orders them all at system scope with one fence before it
    // raises this rank's flags (release is cumulative), so only one CTA per call pays a
    // system-scope fence.
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    if (atomicAdd(a.state + 0, 1u) == gridDim.x - 1u) {
      // The last CTA of this rank: publish the rank's key and flag, then wait for all.
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      const uint32_t t = epoch;
      // A peer's key slot may be written only once it has started this call.
      const bool healthy = ld_relaxed_gpu(abort_word) == 0u &&
                           wait_all_sys(a.ready[a.me], a.world, a.me, t, abort_word);
      if (healthy) {
        const unsigned long long key = *reinterpret_cast<volatile unsigned long long*>(a.best_local);
        for (int r = 0; r < a.world; ++r) a.keys[r][a.me] = key;
        // each release orders the key stores (and the counted CTAs' logits) before the flag
        for (int r = 0; r < a.world; ++r) st_release_sys(a.flags[r] + a.me, t);
        if (wait_all_sys(a.flags[a.me], a.world, -1, t, abort_word) && a.best != nullptr) {
          unsigned long long m = 0ull;
          for (int r = 0; r < a.world; ++r)
            m = max(m, *reinterpret_cast<volatile unsigned long long*>(a.keys[a.me] + r));
          *a.best = m;
        }
      }
      *a.best_local = 0ull;
      a.state[0] = 0u;
      a.state[1] = t;
      __threadfence();
    }
  }
}

}  // namespace w8

// ---------------------------------------------------------------- host side
namespace w8host {

int require_sm100(int* device);

constexpr int64_t kPeerTailBytes = 256;  // keys, flags, ready, state, best

static int64_t logits_pad(int64_t vocab) { return (vocab + 63) / 64 * 64; }

int peer_device_status(int clear, int* out) {
  int v = 0;
  W8_CUDA_TRY(cudaDeviceSynchronize());
  W8_CUDA_TRY(cudaMemcpyFromSymbol(&v, w8::g_peer_status, sizeof(int)));
  if (clear) {
    const int zero = 0;
    W8_CUDA_TRY(cudaMemcpyToSymbol(w8::g_peer_status, &zero, sizeof(int)));
  }
  *out = v;
  return W8_OK;
}

template <int J, int S, int R>
static int launch_peer(const __nv_bfloat16* x, const int8_t* w, const __nv_bfloat16* s, const w8::PeerHeadArgs& a,
                       cudaStream_t stream) {
  auto kern = w8::lm_head_peer_kernel<J, S, R>;
  int sms = 0;
  int st = num_sms(&sms);
  if (st != W8_OK) return st;
  int per_sm = 0;
  W8_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, w8::kGemvThreads, 0));
  if (per_sm < 1) per_sm = 1;
  if (per_sm > 2) per_sm = 2;
  constexpr int rows_per_cta = (w8::kGemvWarps / S) * R;
  const int64_t need = (static_cast<int64_t>(a.n) + rows_per_cta - 1) / rows_per_cta;
  const int64_t cap_blocks = static_cast<int64_t>(sms) * per_sm;
  const int grid = static_cast<int>(need < 1 ? 1 : (need < cap_blocks ? need : cap_blocks));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(w8::kGemvThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, x, w, s, a));
}

}  // namespace w8host

extern "C" int64_t w8_lm_head_peer_bytes(int64_t vocab) {
  return vocab <= 0 ? 0 : 4 * w8host::logits_pad(vocab) + w8host::kPeerTailBytes;
}

extern "C" int w8_peer_alloc(int64_t bytes, void** ptr, void* handle) {
  W8_CHECK_ARG(bytes > 0 && ptr != nullptr && handle != nullptr, "bad peer buffer request");
  int device = 0;
  int st = w8host::require_sm100(&device);
  if (st != W8_OK) return st;
  void* p = nullptr;
  W8_CUDA_TRY(cudaMalloc(&p, static_cast<size_t>(bytes)));
  cudaError_t e = cudaMemset(p, 0, static_cast<size_t>(bytes));
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return w8host::cuda_status(e);
  }
  *ptr = p;
  return W8_OK;
}

extern "C" int w8_peer_open(const void* handle, void** ptr) {
  W8_CHECK_ARG(handle != nullptr && ptr != nullptr, "null handle or output");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  W8_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return W8_OK;
}

extern "C" int w8_peer_close(void* ptr) {
  W8_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return W8_OK;
}

extern "C" int w8_peer_free(void* ptr) {
  W8_CUDA_TRY(cudaFree(ptr));
  return W8_OK;
}

namespace w8host {
static int lm_head_peer(const uint16_t* x, const int8_t* w, const uint16_t* s, float cap, int64_t n, int64_t k,
                        int64_t row0, int64_t vocab, int world, int rank, void* const* bufs, uint64_t* best,
                        int keys_only, w8_stream_t stream);
}  // namespace w8host

extern "C" int w8_lm_head_peer_f32(const uint16_t* x, const int8_t* w, const uint16_t* s, float cap, int64_t n,
                                   int64_t k, int64_t row0, int64_t vocab, int world, int rank, void* const* bufs,
                                   uint64_t* best, w8_stream_t stream) {
  return w8host::lm_head_peer(x, w, s, cap, n, k, row0, vocab, world, rank, bufs, best, 0, stream);
}

extern "C" int w8_lm_head_peer_argmax(const uint16_t* x, const int8_t* w, const uint16_t* s, float cap, int64_t n,
                                      int64_t k, int64_t row0, int64_t vocab, int world, int rank,
                                      void* const* bufs, uint64_t* best, w8_stream_t stream) {
  W8_CHECK_ARG(best != nullptr, "null greedy-key output");
  return w8host::lm_head_peer(x, w, s, cap, n, k, row0, vocab, world, rank, bufs, best, 1, stream);
}

int w8host::lm_head_peer(const uint16_t* x, const int8_t* w, const uint16_t* s, float cap, int64_t n, int64_t k,
                         int64_t row0, int64_t vocab, int world, int rank, void* const* bufs, uint64_t* best,
                         int keys_only, w8_stream_t stream) {
  using namespace w8host;
  W8_CHECK_ARG(world >= 1 && world <= w8::kPeerMax && rank >= 0 && rank < world,
               "world %d / rank %d out of range (1..%d ranks)", world, rank, w8::kPeerMax);
  W8_CHECK_ARG(vocab > 0 && vocab < (1ll << 31) - 1 && n >= 0 && row0 >= 0 && row0 + n <= vocab,
               "shard rows [%lld, %lld) outside the vocabulary of %lld", (long long)row0, (long long)(row0 + n),
               (long long)vocab);
  W8_CHECK_ARG(k > 0 && k % 16 == 0 && k <= 16384, "k = %lld must be a multiple of 16 up to 16384", (long long)k);
  W8_CHECK_ARG(x != nullptr && bufs != nullptr && (n == 0 || (w != nullptr && s != nullptr)), "null pointer");
  W8_CHECK_ALIGN(aligned(x, 16) && (n == 0 || aligned(w, 16)), "x and w must be 16-byte aligned");
  W8_CHECK_ALIGN(best == nullptr || aligned(best, 8), "best must be 8-byte aligned");
  w8::PeerHeadArgs a = {};
  a.world = world;
  a.me = rank;
  a.n = static_cast<int>(n);
  a.k = static_cast<int>(k);
  a.row0 = static_cast<int>(row0);
  a.cap = cap;
  const int64_t off = 4 * logits_pad(vocab);
  for (int r = 0; r < world; ++r) {
    W8_CHECK_ARG(bufs[r] != nullptr, "null buffer of rank %d", r);
    W8_CHECK_ALIGN(aligned(bufs[r], 256), "the buffer of rank %d must be 256-byte aligned", r);
    uint8_t* b = static_cast<uint8_t*>(bufs[r]);
    a.logits[r] = reinterpret_cast<float*>(b);
    a.keys[r] = reinterpret_cast<unsigned long long*>(b + off);
    a.flags[r] = reinterpret_cast<uint32_t*>(b + off + 64);
    a.ready[r] = reinterpret_cast<uint32_t*>(b + off + 96);
  }
  uint8_t* own = static_cast<uint8_t*>(bufs[rank]);
  a.state = reinterpret_cast<uint32_t*>(own + off + 128);
  a.best_local = reinterpret_cast<unsigned long long*>(own + off + 144);
  a.best = reinterpret_cast<unsigned long long*>(best);
  a.keys_only = keys_only;
  int device = 0;
  const int st = require_sm100(&device);
  if (st != W8_OK) return st;
  const auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  const auto* sb = reinterpret_cast<const __nv_bfloat16*>(s);
  const cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  // The (J, S) K split of the standalone GEMV for the same K, so every logit has its bits.
  int sms = 0;
  const int st2 = num_sms(&sms);
  if (st2 != W8_OK) return st2;
#define W8_PEER(J, S, R)                                                          \
  return n < static_cast<int64_t>(sms) * (w8::kGemvWarps / (S)) * (R)           \
             ? launch_peer<J, S, 1>(xb, w, sb, a, cs)                              \
             : launch_peer<J, S, R>(xb, w, sb, a, cs)
  if (k <= 512) W8_PEER(1, 1, 4);
  if (k <= 1024) W8_PEER(2, 1, 4);
  if (k <= 1536) W8_PEER(3, 1, 4);
  if (k <= 2048) W8_PEER(4, 1, 2);
  if (k <= 3072) W8_PEER(3, 2, 4);
  if (k <= 4096) W8_PEER(4, 2, 2);
  if (k <= 6144) W8_PEER(3, 4, 4);
  if (k <= 8192) W8_PEER(4, 4, 2);
  if (k <= 12288) W8_PEER(3, 8, 4);
  W8_PEER(4, 8, 2);
#undef W8_PEER
}
