// tc_gemm.cuh -- persistent 3xTF32 GEMM engine on the sm_100a tensor cores.
//
// Computes D[M,N] = sum_k A[m,k] * B[k,n] with fp32-class accuracy for every
// contraction on the hot path (Dense forward / backward, implicit-GEMM Conv2D
// forward / input grad / filter grad).  An operand "view" says how to gather
// a piece of one tile row of A or B from global memory, so the same engine
// runs row-major matrices, transposed operands and im2col views without
// materialising them.
//
// Output tiles are 128 x BN (BN a multiple of 16, <= 256); K is walked in
// 32-element blocks through a ring of shared-memory stages; split-K slices
// are extra tiles.  One CTA per SM loops over tiles (static round robin),
// with three warp roles:
//
//   warps 0-7   producers.  A stage holds (128 + BN) rows x 32 k of fp32;
//               each thread owns fixed 8-element pieces of 2 A rows and up to
//               4 B rows, loads them, splits x = hi + lo (hi = tf32(x),
//               lo = tf32(x - hi), round to nearest) and stores both into
//               K-major no-swizzle UMMA layouts (conflict-free: the 8 lanes
//               of a quarter warp write one 128-byte core matrix), then
//               fence.proxy.async and arrive on the stage's FULL barrier.
//   warp 8      allocates TMEM: two chunk accumulators P0, P1 and a running
//               sum S, BN fp32 columns each.  Lane 0 waits FULL and issues, per
//               8-wide k step, P += Alo*Bhi + Ahi*Blo + Ahi*Bhi
//               (tcgen05.mma.cta_group::1.kind::tf32, M=128, N=BN), commits
//               each stage's EMPTY barrier, and after at most kChunkKB
//               k-blocks commits the chunk (CHUNK_FULL) and switches to the
//               other P.
//   warps 9-12  epilogue.  Per chunk: wait CHUNK_FULL, read their 32 TMEM
//               lanes of P (tcgen05.ld 32x32b), add the running sum S in fp32
//               with round-to-nearest, and either write S back (tcgen05.st) or,
//               after the tile's last chunk, store rows of D (+ bias) or fp32
//               split-K partials; then release P (CHUNK_EMPTY) while the MMA
//               warp fills the other one.
//
// Why chunks: the tensor core's fp32 accumulation rounds on every update, so
// the error of one accumulator grows with the number of k steps it absorbs
// (measured ~7e-9 relative per k).  Folding every 256 k into S with
// round-to-nearest adds keeps long reductions (filter gradients over
// 500k pixels, K = 4096 GEMMs) at fp32-class accuracy; tiles whose K fits in
// one chunk go straight from P to global memory.
//
// Every mbarrier wait is bounded by a wall-clock limit (a launch parameter);
// on expiry the thread counts the event in g_tc_timeouts (read by
// b2_device_timeouts()), sets the library's host-mapped expiry word (the op
// calls that follow fail with B2_ERR_TIMEOUT) and the CTA stops issuing work,
// waits for the MMAs it issued, frees its TMEM and exits.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "b2_internal.cuh"

namespace b2 {
namespace tc {

constexpr int BM = 128;  // UMMA M (cta_group::1)
constexpr int BK = 32;   // fp32 elements of K per stage
constexpr int kProducerWarps = 8;
constexpr int kMmaWarp = kProducerWarps;
constexpr int kEpiWarp0 = kProducerWarps + 1;
constexpr int kThreads = 32 * (kProducerWarps + 1 + 4);
constexpr int kMaxStages = 6;
constexpr int kUnit = 8;  // k elements per producer unit
constexpr int kChunkKB = 8;  // k-blocks accumulated in one TMEM chunk (256 k)
constexpr int kMaxBN = 160;  // three BN-column regions must fit in 512 TMEM columns
constexpr uint64_t kWaitLimitNs = kDefaultWaitLimitNs;  // drain waits after an abort (fixed)

// Count of bounded waits that expired, read by the host through
// b2_device_timeouts() (internal linkage: one counter per translation unit
// that includes this header; the tensor-core ops all live in gemm_ops.cu).
static __device__ unsigned int g_tc_timeouts = 0;

// ------------------------------------------------------------ PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Three independent non-blocking probes in one asm block: their
// shared-memory round trips overlap instead of queueing one after the other
// behind other warps' shared-memory traffic.  Bit i of the result: barrier i
// has completed the phase of its parity.
__device__ __forceinline__ uint32_t mbar_probe3(uint64_t* b0, uint32_t p0, uint64_t* b1, uint32_t p1, uint64_t* b2,
                                                uint32_t p2) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred q0, q1, q2;\n\t.reg .b32 t0, t1, t2;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 q0, [%1], %2;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 q1, [%3], %4;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 q2, [%5], %6;\n\t"
      "selp.b32 t0, 1, 0, q0;\n\t"
      "selp.b32 t1, 2, 0, q1;\n\t"
      "selp.b32 t2, 4, 0, q2;\n\t"
      "or.b32 t0, t0, t1;\n\t"
      "or.b32 %0, t0, t2;\n\t}"
      : "=r"(r)
      : "r"(smem_u32(b0)), "r"(p0), "r"(smem_u32(b1)), "r"(p1), "r"(smem_u32(b2)), "r"(p2)
      : "memory");
  return r;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Per-CTA state of the bounded waits, in shared memory: the abort flag the
// first expired wait raises (every other wait of the CTA then gives up too),
// the limit of one wait and the library's host-mapped expiry word.
struct WaitState {
  int abort;
  uint64_t limit_ns;
  unsigned int* expired;
};

// Thread 0 of the CTA, before the block-wide barrier that precedes any wait.
__device__ __forceinline__ void wait_state_init(WaitState* ws, const WaitParams& wp) {
  ws->abort = 0;
  ws->limit_ns = wp.limit_ns;
  ws->expired = wp.expired;
}

__device__ __forceinline__ bool aborted(const WaitState* ws) {
  return *reinterpret_cast<const volatile int*>(&ws->abort) != 0;
}

// Record an expired wait: the device counter, the host-visible word.
__device__ __forceinline__ void note_expiry(unsigned int* expired) {
  atomicAdd(&g_tc_timeouts, 1u);
  if (expired) {
    *reinterpret_cast<volatile unsigned int*>(expired) = 1u;
    __threadfence_system();
  }
}

// Bounded wait for the phase of parity `parity` on `bar`.  On expiry: record
// it, raise the CTA's abort flag and return false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, WaitState* ws) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0) {  // the clock and the abort flag: after the second failed try, then every 256
      if (aborted(ws)) return false;
      if (global_ns() - t0 > ws->limit_ns) {
        note_expiry(ws->expired);
        *reinterpret_cast<volatile int*>(&ws->abort) = 1;
        return false;
      }
    }
  }
}

// Wait bounded by the fixed drain limit only (used while tearing down after
// an abort, for work already issued: copies in flight, MMAs issued).
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity, unsigned int* expired = nullptr) {
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > kWaitLimitNs) {
      note_expiry(expired);
      return;
    }
  }
}

__device__ __forceinline__ uint32_t tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// K-major, no-swizzle canonical layout ((8,n),2):((16B,SBO),LBO): core
// matrices of 8 rows x 16 B; LBO = 128 B between core matrices adjacent along
// K, SBO = 1024 B between 8-row groups.  Element (r, k) of a tile lives at
//   (r/8)*1024 + (k/4)*128 + (r%8)*16 + (k%4)*4   bytes.
constexpr uint32_t kLBO = 128;
constexpr uint32_t kSBO = 1024;

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)(kLBO >> 4) << 16) | ((uint64_t)(kSBO >> 4) << 32) |
         (1ull << 46);  // version 1 (sm_100), base offset 0, layout SWIZZLE_NONE
}

// Instruction descriptor: D fp32, A/B tf32, both K-major, M=128, N=n.
__host__ __device__ constexpr uint32_t idesc_tf32(int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Split 8 values (k offsets 8q..8q+7) of tile row r into hi/lo tf32 and store.
__device__ __forceinline__ void store_unit_split(uint8_t* hi_tile, uint8_t* lo_tile, int r, int q,
                                                 const float (&v)[kUnit]) {
  const uint32_t off = (uint32_t)(r >> 3) * kSBO + (uint32_t)(2 * q) * kLBO + (uint32_t)(r & 7) * 16u;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float x = v[c * 4 + j];
      h[j] = tf32_rna(x);
      l[j] = tf32_rna(x - __uint_as_float(h[j]));
    }
    *reinterpret_cast<uint4*>(hi_tile + off + c * kLBO) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo_tile + off + c * kLBO) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

__device__ __forceinline__ void zero_unit(float (&v)[kUnit]) {
#pragma unroll
  for (int i = 0; i < kUnit; ++i) v[i] = 0.0f;
}

// --------------------------------------------------------- operand views
//
// A view exposes, for tile row r (an M index for A, an N index for B):
//   Ctx row(int64_t r) const;                          per-row state
//   void load8(const Ctx&, int64_t k, int64_t k_end, float (&v)[8]) const;
// filling v[i] = op(r, k + i) for k + i < k_end, 0 otherwise, and 0 for
// rows outside the matrix.  k is a multiple of 8.

// op(r, k) = p[r * ld + k]   (K contiguous)
struct KContig {
  const float* p;
  int64_t rows, ld;
  bool vec;  // p and ld allow 16-byte loads
  struct Ctx {
    const float* base;
    bool valid;
  };
  __device__ Ctx row(int64_t r) const { return Ctx{p + r * ld, r < rows}; }
  __device__ void load8(const Ctx& c, int64_t k, int64_t k_end, float (&v)[kUnit]) const {
    if (!c.valid) {
      zero_unit(v);
      return;
    }
    if (vec && k + kUnit <= k_end) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(c.base + k));
      const float4 b = __ldg(reinterpret_cast<const float4*>(c.base + k) + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
      for (int i = 0; i < kUnit; ++i) v[i] = (k + i < k_end) ? __ldg(c.base + k + i) : 0.0f;
    }
  }
};

// op(r, k) = p[k * ld + r]   (the tile row index is contiguous: MN-major)
struct MNMajor {
  const float* p;
  int64_t rows, ld;
  struct Ctx {
    const float* base;
    bool valid;
  };
  __device__ Ctx row(int64_t r) const { return Ctx{p + r, r < rows}; }
  __device__ void load8(const Ctx& c, int64_t k, int64_t k_end, float (&v)[kUnit]) const {
    if (!c.valid) {
      zero_unit(v);
      return;
    }
#pragma unroll
    for (int i = 0; i < kUnit; ++i) v[i] = (k + i < k_end) ? __ldg(c.base + (k + i) * ld) : 0.0f;
  }
};

// --------------------------------------------------------------- problem

// How results leave the accumulator.
struct Epilogue {
  float* out;         // D, row-major, leading dimension ldo (or partials)
  int64_t ldo;
  const float* bias;  // optional per-column bias (direct mode only)
  bool partial;       // write split z to out + z * M * N (ld = N), no bias
};

template <class AV, class BV>
struct GemmProblem {
  AV a;
  BV b;
  int64_t M, N, K;
  int64_t k_per_split;  // multiple of BK
  int splits;
  Epilogue ep;
  WaitParams wait;  // set by launch_gemm
};

struct KernelSmem {
  int stages;
  int bn;
  size_t a_bytes, b_bytes, stage_bytes, bar_offset, total;
};

inline KernelSmem smem_plan(int bn, int stages) {
  KernelSmem s;
  s.stages = stages;
  s.bn = bn;
  s.a_bytes = (size_t)BM * BK * 4;
  s.b_bytes = (size_t)bn * BK * 4;
  s.stage_bytes = 2 * s.a_bytes + 2 * s.b_bytes;
  s.bar_offset = s.stage_bytes * stages;
  s.total = s.bar_offset + 8 * (2 * kMaxStages + 5) + 16 + 1024;  // + alignment slack
  return s;
}

struct TileCoord {
  int64_t m0, n0, k_begin, k_end;
  int z, nkb;
};

template <class P>
__device__ __forceinline__ TileCoord tile_coord(const P& p, int bn, int64_t t) {
  const int64_t nt = (p.N + bn - 1) / bn, mt = (p.M + BM - 1) / BM;
  TileCoord c;
  const int64_t n_idx = t % nt;
  const int64_t rest = t / nt;
  c.m0 = (rest % mt) * BM;
  c.z = (int)(rest / mt);
  c.n0 = n_idx * bn;
  c.k_begin = (int64_t)c.z * p.k_per_split;
  c.k_end = c.k_begin + p.k_per_split;
  if (c.k_end > p.K) c.k_end = p.K;
  c.nkb = c.k_end > c.k_begin ? (int)((c.k_end - c.k_begin + BK - 1) / BK) : 0;
  return c;
}

template <class P>
__global__ void __launch_bounds__(kThreads, 1) tc_gemm_kernel(const P p, const int bn, const int stages) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const size_t a_bytes = (size_t)BM * BK * 4;
  const size_t b_bytes = (size_t)bn * BK * 4;
  const size_t stage_bytes = 2 * a_bytes + 2 * b_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + stage_bytes * stages);
  uint64_t* empty = full + kMaxStages;
  uint64_t* chunk_full = empty + kMaxStages;  // [2]
  uint64_t* chunk_empty = chunk_full + 2;     // [2]
  uint64_t* mma_done = chunk_empty + 2;  // every MMA this CTA issued has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  __shared__ WaitState s_wait;
  WaitState* ws = &s_wait;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t nt = (p.N + bn - 1) / bn, mt = (p.M + BM - 1) / BM;
  const int64_t tiles = nt * mt * p.splits;
  const uint32_t acc_cols = (uint32_t)bn;
  const int need_cols = 3 * bn;  // P0, P1, S
  const uint32_t tmem_cols = need_cols <= 32 ? 32u : need_cols <= 64 ? 64u : need_cols <= 128 ? 128u
                             : need_cols <= 256 ? 256u : 512u;

  if (threadIdx.x == 0) {
    wait_state_init(ws, p.wait);
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], kProducerWarps * 32);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&chunk_full[a], 1);
      mbar_init(&chunk_empty[a], 128);
    }
    mbar_init(mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_base = *tmem_slot;

  if (warp < kProducerWarps) {
    // ---------------------------------------------------------- producers
    // Thread (warp w, lane l): rows 8w + (l & 7) (+64 per unit), k piece q = l >> 3.
    const int rsub = 8 * warp + (lane & 7);
    const int q = lane >> 3;
    uint32_t stage_cnt = 0;
    for (int64_t t = blockIdx.x; t < tiles && !aborted(ws); t += gridDim.x) {
      const TileCoord tc = tile_coord(p, bn, t);
      const auto ca0 = p.a.row(tc.m0 + rsub);
      const auto ca1 = p.a.row(tc.m0 + rsub + 64);
      typename decltype(p.b)::Ctx cb[3];
#pragma unroll
      for (int j = 0; j < 3; ++j) cb[j] = p.b.row(tc.n0 + rsub + 64 * j);
      for (int kb = 0; kb < tc.nkb; ++kb, ++stage_cnt) {
        const int s = (int)(stage_cnt % (uint32_t)stages);
        const uint32_t round = stage_cnt / (uint32_t)stages;
        // Issue every load of this k-block (2 A pieces, up to 3 B pieces)
        // before waiting for the stage or storing: one memory round trip per
        // k-block, overlapped with the wait for the slot.
        const int64_t k = tc.k_begin + (int64_t)kb * BK + q * kUnit;
        float va0[kUnit], va1[kUnit], vb[3][kUnit];
        p.a.load8(ca0, k, tc.k_end, va0);
        p.a.load8(ca1, k, tc.k_end, va1);
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          const int r = rsub + 64 * j;
          if (r < bn) {
            if (tc.n0 + r < p.N) p.b.load8(cb[j], k, tc.k_end, vb[j]); else zero_unit(vb[j]);
          }
        }
        if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1u, ws)) break;
        uint8_t* st = smem + (size_t)s * stage_bytes;
        store_unit_split(st, st + a_bytes, rsub, q, va0);
        store_unit_split(st, st + a_bytes, rsub + 64, q, va1);
        uint8_t* bhi = st + 2 * a_bytes;
        uint8_t* blo = bhi + b_bytes;
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          const int r = rsub + 64 * j;
          if (r < bn) store_unit_split(bhi, blo, r, q, vb[j]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(&full[s]);
      }
    }
  } else if (warp == kMmaWarp) {
    // -------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_tf32(bn);
      uint32_t stage_cnt = 0, g = 0;  // g counts chunks
      bool ok = true;
      for (int64_t t = blockIdx.x; t < tiles && ok && !aborted(ws); t += gridDim.x) {
        const TileCoord tc = tile_coord(p, bn, t);
        for (int kb0 = 0; kb0 < tc.nkb && ok; kb0 += kChunkKB, ++g) {
          const int a = (int)(g & 1u);
          const uint32_t use = g >> 1;
          if (use > 0 && !mbar_wait(&chunk_empty[a], (use - 1) & 1u, ws)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t d = tmem_base + (uint32_t)a * acc_cols;
          const int kb1 = kb0 + kChunkKB < tc.nkb ? kb0 + kChunkKB : tc.nkb;
          for (int kb = kb0; kb < kb1; ++kb, ++stage_cnt) {
            const int s = (int)(stage_cnt % (uint32_t)stages);
            if (!mbar_wait(&full[s], (stage_cnt / (uint32_t)stages) & 1u, ws)) {
              ok = false;
              break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t st = smem_u32(smem + (size_t)s * stage_bytes);
            const uint32_t a_hi = st, a_lo = st + (uint32_t)a_bytes;
            const uint32_t b_hi = st + 2u * (uint32_t)a_bytes, b_lo = b_hi + (uint32_t)b_bytes;
#pragma unroll
            for (int j = 0; j < BK / 8; ++j) {
              const uint32_t off = (uint32_t)j * 2u * kLBO;  // 8 tf32 = two core matrices along K
              mma_tf32(d, smem_desc(a_lo + off), smem_desc(b_hi + off), idesc, (kb > kb0 || j > 0) ? 1u : 0u);
              mma_tf32(d, smem_desc(a_hi + off), smem_desc(b_lo + off), idesc, 1u);
              mma_tf32(d, smem_desc(a_hi + off), smem_desc(b_hi + off), idesc, 1u);
            }
            mma_commit(&empty[s]);
          }
          mma_commit(&chunk_full[a]);
        }
      }
      // TMEM is freed at the end of the kernel: after an aborted pipeline the
      // epilogue may not have waited for the last MMAs, so wait for them here
      mma_commit(mma_done);
      mbar_wait_drain(mma_done, 0, ws->expired);
    }
  } else {
    // ----------------------------------------------------------- epilogue
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_addr = tmem_base + lane_off + 2u * acc_cols;
    uint32_t g = 0;
    bool ok = true;
    for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
      const TileCoord tc = tile_coord(p, bn, t);
      const int64_t m = tc.m0 + quarter * 32 + lane;
      const int64_t n_lim = p.N - tc.n0 < bn ? p.N - tc.n0 : bn;
      const int nch = (tc.nkb + kChunkKB - 1) / kChunkKB;
      for (int ch = 0; ch < (nch > 0 ? nch : 1); ++ch) {
        const bool first = ch == 0, last = ch + 1 >= nch;
        const int a = (int)(g & 1u);
        if (nch > 0) {
          if (!mbar_wait(&chunk_full[a], (g >> 1) & 1u, ws)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        }
        const uint32_t p_addr = tmem_base + lane_off + (uint32_t)a * acc_cols;
        for (int c = 0; c < bn; c += 16) {
          float v[16];
          if (nch > 0) {
            tmem_ld16(p_addr + (uint32_t)c, v);
            if (!first) {
              float sv[16];
              tmem_ld16(s_addr + (uint32_t)c, sv);
#pragma unroll
              for (int e = 0; e < 16; ++e) v[e] = __fadd_rn(sv[e], v[e]);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] = 0.0f;
          }
          if (!last) {
            tmem_st16(s_addr + (uint32_t)c, v);
            continue;
          }
          if (m >= p.M || c >= n_lim) continue;
          float* dst;
          const float* bias = nullptr;
          int64_t ld;
          if (p.ep.partial) {
            dst = p.ep.out + (int64_t)tc.z * p.M * p.N + m * p.N + tc.n0 + c;
            ld = p.N;
          } else {
            dst = p.ep.out + m * p.ep.ldo + tc.n0 + c;
            ld = p.ep.ldo;
            if (p.ep.bias) bias = p.ep.bias + tc.n0 + c;
          }
          if (bias) {
#pragma unroll
            for (int e = 0; e < 16; ++e)
              if (c + e < n_lim) v[e] += __ldg(bias + e);
          }
          if (c + 16 <= n_lim && ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0) && (ld % 4 == 0)) {
#pragma unroll
            for (int e = 0; e < 16; e += 4)
              *reinterpret_cast<float4*>(dst + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e)
              if (c + e < n_lim) dst[e] = v[e];
          }
        }
        if (nch > 0) {
          if (!last) asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          mbar_arrive(&chunk_empty[a]);  // P may be refilled
          ++g;
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols)
                 : "memory");
  }
}

// Sum split-K partials in split order and add the bias: D = sum_z P[z] + b.
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, int64_t M, int64_t N,
                                     const float* __restrict__ bias, float* __restrict__ out, int64_t ldo);

// Launch helpers (gemm_ops.cu).
int choose_bn(int64_t N);
int choose_stages(int bn, int max_smem);
int splits_for(int64_t tiles, int64_t K, int sm_count, int min_kb_per_split);

template <class P>
int launch_gemm(P prob, int bn, cudaStream_t s, const char* name) {
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  const int stages = choose_stages(bn, d->max_smem_optin);
  const KernelSmem plan = smem_plan(bn, stages);
  static SmemOptIn opt_in;  // per template instantiation
  B2_RETURN_IF_ERROR(opt_in.ensure(reinterpret_cast<const void*>(tc_gemm_kernel<P>), d->device, (int)plan.total));
  prob.wait = wait_params();
  const int64_t tiles = ceil_div(prob.N, bn) * ceil_div(prob.M, BM) * prob.splits;
  const int ctas = persistent_ctas(d);
  const int grid = (int)(tiles < ctas ? tiles : ctas);
  tc_gemm_kernel<P><<<grid, kThreads, plan.total, s>>>(prob, bn, stages);
  return check_launch(s, name);
}

}  // namespace tc
}  // namespace b2
