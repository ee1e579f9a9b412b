// tc_gemm.cuh -- 3xTF32 GEMM engine on the sm_100a tensor cores (tcgen05).
//
// Computes D[M,N] = sum_k A[m,k] * B[k,n] in fp32-class accuracy for every
// contraction on the hot path (Dense forward / backward, implicit-GEMM Conv2D
// forward / input grad / filter grad).  A "problem" object describes how to
// gather one tile row of A or B from global memory, so the same engine runs
// plain row-major matrices, transposed operands and im2col views.
//
// Per CTA: one 128 x BN output tile (BN a multiple of 16, <= 256), K walked in
// 32-element blocks through a ring of shared-memory stages.
//
//   warps 0-3  producers: each thread owns one tile row of A (and one or two
//              of B), loads its 32 fp32 values, splits each into
//              hi = tf32(x), lo = tf32(x - hi) (round to nearest) and stores
//              both into K-major, no-swizzle UMMA layouts; then
//              fence.proxy.async + mbarrier arrive on the stage's FULL barrier.
//   warp 4     allocates the TMEM accumulator; lane 0 waits FULL, issues
//              per 8-wide k step  D += Ahi*Bhi + Ahi*Blo + Alo*Bhi
//              (tcgen05.mma.cta_group::1.kind::tf32, M=128, N=BN) and
//              tcgen05.commit's the stage's EMPTY barrier; a final commit
//              arms the ACCUM barrier.
//   epilogue   warps 0-3 read their 32 TMEM lanes (tcgen05.ld 32x32b) and
//              write rows of D (optionally + bias), or fp32 partials for a
//              split-K reduction.
//
// Error-compensated 3xTF32 (the dropped lo*lo term is ~2^-22 relative) keeps
// fp32 accuracy; accumulation is fp32 in TMEM.
//
// Every mbarrier wait is bounded by a wall-clock limit; on expiry the thread
// records the failure in g_tc_timeouts and leaves its loop, the CTA still
// frees its TMEM, and the host reports B2_ERR_TIMEOUT when it checks.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "b2_internal.cuh"

namespace b2 {
namespace tc {

constexpr int BM = 128;             // UMMA M (cta_group::1)
constexpr int BK = 32;              // fp32 elements of K per stage (128 B rows)
constexpr int kProducerWarps = 4;
constexpr int kThreads = 32 * (kProducerWarps + 1);
constexpr int kMaxStages = 6;
constexpr uint64_t kWaitLimitNs = 10ull * 1000 * 1000 * 1000;  // 10 s

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

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for `parity` on `bar`; false (and a recorded timeout) if the
// phase did not complete within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0 && global_ns() - t0 > kWaitLimitNs) {
      atomicAdd(&g_tc_timeouts, 1u);
      return false;
    }
  }
}

__device__ __forceinline__ uint32_t tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// K-major, no-swizzle canonical layout ((8,n),2):((16B,SBO),LBO):
// core matrices of 8 rows x 16 B; LBO = 128 B between the core matrices that
// are adjacent along K, SBO = 1024 B between 8-row groups (8 core matrices
// cover one 32-element K block).  Element (r, k) of a tile lives at
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

// Split 32 values of tile row `r` into hi/lo tf32 and store them.
__device__ __forceinline__ void store_row_split(uint8_t* hi_tile, uint8_t* lo_tile, int r, const float (&v)[BK]) {
  const uint32_t row_off = (uint32_t)(r >> 3) * kSBO + (uint32_t)(r & 7) * 16u;
#pragma unroll
  for (int c = 0; c < BK / 4; ++c) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float x = v[c * 4 + j];
      h[j] = tf32_rna(x);
      l[j] = tf32_rna(x - __uint_as_float(h[j]));
    }
    *reinterpret_cast<uint4*>(hi_tile + row_off + c * kLBO) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo_tile + row_off + c * kLBO) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

__device__ __forceinline__ void zero_row(float (&v)[BK]) {
#pragma unroll
  for (int i = 0; i < BK; ++i) v[i] = 0.0f;
}

// --------------------------------------------------------- operand views
//
// A view exposes, for tile row r (an M index for A, an N index for B):
//   Ctx row(int r) const;                      per-row state, computed once
//   void load(const Ctx&, int k0, int k_end, float (&v)[32]) const;
// filling v[i] = op(r, k0 + i) for k0 + i < k_end, 0 otherwise (and 0 for
// rows outside the matrix).

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
  __device__ void load(const Ctx& c, int64_t k0, int64_t k_end, float (&v)[BK]) const {
    if (!c.valid) {
      zero_row(v);
      return;
    }
    if (vec && k0 + BK <= k_end) {
#pragma unroll
      for (int q = 0; q < BK / 4; ++q) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(c.base + k0) + q);
        v[4 * q] = t.x;
        v[4 * q + 1] = t.y;
        v[4 * q + 2] = t.z;
        v[4 * q + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < BK; ++i) v[i] = (k0 + i < k_end) ? __ldg(c.base + k0 + i) : 0.0f;
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
  __device__ void load(const Ctx& c, int64_t k0, int64_t k_end, float (&v)[BK]) const {
    if (!c.valid) {
      zero_row(v);
      return;
    }
#pragma unroll
    for (int i = 0; i < BK; ++i) v[i] = (k0 + i < k_end) ? __ldg(c.base + (k0 + i) * ld) : 0.0f;
  }
};

// --------------------------------------------------------------- problem

// How results leave the accumulator.
struct Epilogue {
  float* out;          // D, row-major, leading dimension ldo (or partials)
  int64_t ldo;
  const float* bias;   // optional per-column bias (direct mode only)
  bool partial;        // write split z to out + z * M * N (ld = N), no bias
};

template <class AV, class BV>
struct GemmProblem {
  AV a;
  BV b;
  int64_t M, N, K;
  int64_t k_per_split;  // multiple of BK
  Epilogue ep;
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
  s.total = s.bar_offset + 8 * (2 * kMaxStages + 1) + 16 + 1024;  // + alignment slack
  return s;
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
  uint64_t* accum = empty + kMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t n0 = (int64_t)blockIdx.x * bn;
  const int64_t m0 = (int64_t)blockIdx.y * BM;
  const int64_t k_begin = (int64_t)blockIdx.z * p.k_per_split;
  int64_t k_end = k_begin + p.k_per_split;
  if (k_end > p.K) k_end = p.K;
  const int nkb = k_end > k_begin ? (int)((k_end - k_begin + BK - 1) / BK) : 0;
  const uint32_t tmem_cols = bn <= 32 ? 32u : bn <= 64 ? 64u : bn <= 128 ? 128u : 256u;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], kProducerWarps * 32);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kProducerWarps) {
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
    const int t = threadIdx.x;
    const auto ca = p.a.row(m0 + t);
    const auto cb0 = p.b.row(n0 + t);
    const auto cb1 = p.b.row(n0 + t + 128);
    float v[BK];
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % stages;
      const uint32_t ph = (uint32_t)(kb / stages) & 1u;
      if (kb >= stages && !mbar_wait(&empty[s], ph ^ 1u)) {
        s_abort = 1;
        break;
      }
      if (s_abort) break;
      uint8_t* st = smem + (size_t)s * stage_bytes;
      const int64_t k0 = k_begin + (int64_t)kb * BK;
      p.a.load(ca, k0, k_end, v);
      store_row_split(st, st + a_bytes, t, v);
      if (t < bn) {
        if (n0 + t < p.N) p.b.load(cb0, k0, k_end, v); else zero_row(v);
        store_row_split(st + 2 * a_bytes, st + 2 * a_bytes + b_bytes, t, v);
      }
      if (t + 128 < bn) {
        if (n0 + t + 128 < p.N) p.b.load(cb1, k0, k_end, v); else zero_row(v);
        store_row_split(st + 2 * a_bytes, st + 2 * a_bytes + b_bytes, t + 128, v);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&full[s]);
    }
  } else if (lane == 0) {
    // -------------------------------------------------------- MMA issuer
    const uint32_t idesc = idesc_tf32(bn);
    bool ok = true;
    for (int kb = 0; kb < nkb && ok; ++kb) {
      const int s = kb % stages;
      const uint32_t ph = (uint32_t)(kb / stages) & 1u;
      if (!mbar_wait(&full[s], ph)) {
        s_abort = 1;
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
        mma_tf32(tmem_base, smem_desc(a_lo + off), smem_desc(b_hi + off), idesc, (kb > 0 || j > 0) ? 1u : 0u);
        mma_tf32(tmem_base, smem_desc(a_hi + off), smem_desc(b_lo + off), idesc, 1u);
        mma_tf32(tmem_base, smem_desc(a_hi + off), smem_desc(b_hi + off), idesc, 1u);
      }
      mma_commit(&empty[s]);
    }
    mma_commit(accum);
  }

  // ------------------------------------------------------------- epilogue
  if (warp < kProducerWarps) {
    const int64_t m = m0 + warp * 32 + lane;
    bool have_acc = nkb > 0;
    if (have_acc && !mbar_wait(accum, 0)) {
      s_abort = 1;
      have_acc = false;
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int64_t n_lim = p.N - n0 < bn ? p.N - n0 : bn;
    for (int c = 0; c < bn; c += 16) {
      float v[16];
      if (have_acc) {
        tmem_ld16(tmem_base + ((uint32_t)(warp * 32) << 16) + (uint32_t)c, v);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.0f;
      }
      if (m >= p.M || c >= n_lim) continue;
      if (p.ep.partial) {
        float* dst = p.ep.out + (int64_t)blockIdx.z * p.M * p.N + m * p.N + n0 + c;
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (c + i < n_lim) dst[i] = v[i];
      } else {
        float* dst = p.ep.out + m * p.ep.ldo + n0 + c;
        const float* bias = p.ep.bias ? p.ep.bias + n0 + c : nullptr;
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (c + i < n_lim) dst[i] = bias ? v[i] + __ldg(bias + i) : v[i];
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == kProducerWarps) {
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols)
                 : "memory");
  }
}

// Sum split-K partials in split order and add the bias: D = sum_z P[z] + b.
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, int64_t M, int64_t N,
                                     const float* __restrict__ bias, float* __restrict__ out, int64_t ldo);

// Launch helpers (tc_gemm.cu).
int choose_bn(int64_t N);
int choose_stages(int bn, int max_smem);
int splits_for(int64_t tiles, int64_t K, int sm_count, int min_kb_per_split);

template <class P>
int launch_gemm(P prob, int bn, int splits, cudaStream_t s, const char* name) {
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  const int stages = choose_stages(bn, d->max_smem_optin);
  const KernelSmem plan = smem_plan(bn, stages);
  static int configured_bytes = 0;  // per template instantiation
  if ((int)plan.total > configured_bytes) {
    B2_CUDA_OR_RETURN(
        cudaFuncSetAttribute(tc_gemm_kernel<P>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan.total));
    configured_bytes = (int)plan.total;
  }
  dim3 grid((unsigned)ceil_div(prob.N, bn), (unsigned)ceil_div(prob.M, BM), (unsigned)splits);
  tc_gemm_kernel<P><<<grid, kThreads, plan.total, s>>>(prob, bn, stages);
  return check_launch(s, name);
}

}  // namespace tc
}  // namespace b2
