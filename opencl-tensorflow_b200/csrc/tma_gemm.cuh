// tma_gemm.cuh -- 3xTF32 GEMM engine fed by the Tensor Memory Accelerator,
// for contractions whose operands are plain row-major matrices (Dense forward
// and backward, 1x1 / stride-1 / unpadded Conv2D forward and gradients).
//
// Each operand is K-major (op(r, k) = p[r*ld + k]) or MN-major
// (op(r, k) = p[k*ld + r]); both are loaded as 128-byte-swizzled tiles that
// the tensor core reads directly in that major-ness, so no thread ever
// gathers or transposes operand data:
//
//   K-major  tile [R rows][32 k]          one TMA box {32, R}; UMMA K-major
//            SWIZZLE_128B, SBO = 1024 B (8-row groups), k step = +32 B.
//   MN-major tile [R/32][32 k][32 rows]   R/32 TMA boxes {32, 32} with the
//            128-byte swizzle of 32-byte atoms (the only MN-major smem
//            layout tf32 UMMA accepts); UMMA MN-major SWIZZLE_128B_BASE32B,
//            LBO = 4096 B (32-row blocks), SBO = 512 B (4-k groups),
//            k step = +1024 B.
//
// Out-of-range rows and k are zero-filled by the TMA unit.  One CTA per SM
// loops over output tiles 128 x BN (BN a multiple of 32, <= 128) and split-K
// slices, with four warp roles:
//
//   warp 0       lane 0 waits for a free stage (EMPTY), posts the stage's
//                byte count on RAW_FULL and issues the TMA loads of A and B.
//   warp 1       allocates TMEM (chunk accumulators P0, P1 and running sum
//                S); lane 0 waits CONV_FULL and issues, per 8-wide k step,
//                P += Alo*Bhi + Ahi*Blo + Ahi*Bhi, commits EMPTY per stage and
//                CHUNK_FULL per chunk (at most kChunkKB k-blocks).
//   warps 2-9    converters: wait RAW_FULL, split every fp32 word of the
//                landed tiles in place, x -> hi = tf32_rna(x) (kept where x
//                was) and lo = tf32_rna(x - hi) (same offset in the stage's lo
//                tile, so the swizzle carries over), fence.proxy.async, arrive
//                CONV_FULL.  Linear 16-byte accesses: no bank conflicts.
//   warps 10-13  epilogue: per chunk fold P into S with round-to-nearest fp32
//                adds (as the register-fed engine does); after the tile's last
//                chunk, add the bias, write 32 x 32 blocks into 128-byte-
//                swizzled shared buffers (double-buffered per warp) and store
//                them with TMA (clipped to the output), so every row leaves
//                as whole 128-byte lines.
//
// Every mbarrier wait is bounded; on expiry the CTA raises its abort flag,
// lets TMA loads already issued land, waits for its own TMA stores, frees its
// TMEM and exits, and the expiry is counted in g_tc_timeouts.
#pragma once

#include <cuda.h>

#include "tc_gemm.cuh"

namespace b2 {
namespace tc {

constexpr int kTmaWarp = 0;
constexpr int kTmaMmaWarp = 1;
constexpr int kConvWarp0 = 2;
constexpr int kConvWarps = 8;
constexpr int kTmaEpiWarp0 = kConvWarp0 + kConvWarps;  // 10 .. 13: lane quarters 2, 3, 0, 1
constexpr int kTmaThreads = 32 * (kTmaEpiWarp0 + 4);
constexpr int kTmaMaxStages = 8;
constexpr int kTmaMaxBN = 128;
constexpr uint32_t kEpiBuf = 32 * 128;  // one 32 x 32 fp32 output block

struct TmaProblem {
  int64_t M, N, K;
  int64_t k_per_split;  // multiple of BK
  int splits;
  int bn;
  const float* bias;  // per-column bias, direct mode only
  bool partial;       // out is [splits][M][N] partials (3-D store map)
};

struct TmaSmem {
  int stages;
  uint32_t a_bytes, b_bytes, stage_bytes, epi_offset, bar_offset, total;
};

__host__ __device__ inline TmaSmem tma_smem_plan(int bn, int stages) {
  TmaSmem s;
  s.stages = stages;
  s.a_bytes = (uint32_t)BM * BK * 4;
  s.b_bytes = (uint32_t)bn * BK * 4;
  s.stage_bytes = 2 * s.a_bytes + 2 * s.b_bytes;
  s.epi_offset = s.stage_bytes * (uint32_t)stages;
  s.bar_offset = s.epi_offset + 4 * 2 * kEpiBuf;
  s.total = s.bar_offset + 8 * (3 * kTmaMaxStages + 4) + 16 + 1024;  // + alignment slack
  return s;
}

// ------------------------------------------------------------ PTX helpers

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Wait bounded by time only (used while draining, after an abort).
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > kWaitLimitNs) {
      atomicAdd(&g_tc_timeouts, 1u);
      return;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(src)
               : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, int x, int y, int z, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z), "r"(src)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// UMMA shared-memory descriptor with a swizzled layout: type 2 = 128-byte
// swizzle of 16-byte atoms, type 1 = 128-byte swizzle of 32-byte atoms.
__device__ __forceinline__ uint64_t smem_desc_swz(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t type) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)type << 61);
}

// Instruction descriptor: D fp32, A/B tf32, M = 128, N = n; a_mn / b_mn set
// the MN-major bits (15 / 16).
__host__ __device__ constexpr uint32_t idesc_tf32_major(int n, bool a_mn, bool b_mn) {
  return idesc_tf32(n) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16);
}

template <bool kAK>
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int j) {
  if constexpr (kAK) return smem_desc_swz(base + (uint32_t)j * 32u, 16u, 1024u, 2u);
  else return smem_desc_swz(base + (uint32_t)j * 1024u, 4096u, 512u, 1u);
}

// Split the 16-byte words [i0, n) step `step` of a landed tile in place.
__device__ __forceinline__ void split_words(uint8_t* hi, uint8_t* lo, int n, int i0, int step) {
  for (int i = i0; i < n; i += step) {
    const uint4 w = *reinterpret_cast<const uint4*>(hi + 16 * i);
    const uint32_t h0 = tf32_rna(__uint_as_float(w.x)), h1 = tf32_rna(__uint_as_float(w.y));
    const uint32_t h2 = tf32_rna(__uint_as_float(w.z)), h3 = tf32_rna(__uint_as_float(w.w));
    const uint4 l = make_uint4(tf32_rna(__uint_as_float(w.x) - __uint_as_float(h0)),
                               tf32_rna(__uint_as_float(w.y) - __uint_as_float(h1)),
                               tf32_rna(__uint_as_float(w.z) - __uint_as_float(h2)),
                               tf32_rna(__uint_as_float(w.w) - __uint_as_float(h3)));
    *reinterpret_cast<uint4*>(hi + 16 * i) = make_uint4(h0, h1, h2, h3);
    *reinterpret_cast<uint4*>(lo + 16 * i) = l;
  }
}

struct TmaTile {
  int64_t m0, n0, k_begin, k_end;
  int z, nkb;
};

__device__ __forceinline__ TmaTile tma_tile(const TmaProblem& p, int64_t t) {
  const int64_t nt = (p.N + p.bn - 1) / p.bn, mt = (p.M + BM - 1) / BM;
  TmaTile c;
  const int64_t n_idx = t % nt;
  const int64_t rest = t / nt;
  c.m0 = (rest % mt) * BM;
  c.z = (int)(rest / mt);
  c.n0 = n_idx * p.bn;
  c.k_begin = (int64_t)c.z * p.k_per_split;
  c.k_end = c.k_begin + p.k_per_split;
  if (c.k_end > p.K) c.k_end = p.K;
  c.nkb = c.k_end > c.k_begin ? (int)((c.k_end - c.k_begin + BK - 1) / BK) : 0;
  return c;
}

template <bool kAK, bool kBK>
__global__ void __launch_bounds__(kTmaThreads, 1)
    tma_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                    const __grid_constant__ CUtensorMap map_d, const TmaProblem p, const int stages) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int bn = p.bn;
  const TmaSmem plan = tma_smem_plan(bn, stages);
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(smem + plan.bar_offset);
  uint64_t* conv_full = raw_full + kTmaMaxStages;
  uint64_t* empty = conv_full + kTmaMaxStages;
  uint64_t* chunk_full = empty + kTmaMaxStages;  // [2]
  uint64_t* chunk_empty = chunk_full + 2;        // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(chunk_empty + 2);
  __shared__ int s_abort;
  volatile int* abort_flag = &s_abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t nt = (p.N + bn - 1) / bn, mt = (p.M + BM - 1) / BM;
  const int64_t tiles = nt * mt * p.splits;
  const uint32_t acc_cols = (uint32_t)bn;
  const int need_cols = 3 * bn;  // P0, P1, S
  const uint32_t tmem_cols = need_cols <= 32 ? 32u : need_cols <= 64 ? 64u : need_cols <= 128 ? 128u
                             : need_cols <= 256 ? 256u : 512u;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < stages; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&conv_full[s], kConvWarps * 32);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&chunk_full[a], 1);
      mbar_init(&chunk_empty[a], 128);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kTmaMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_base = *tmem_slot;

  if (warp == kTmaWarp) {
    // ---------------------------------------------------------- TMA issue
    if (lane == 0) {
      const uint32_t tx = plan.a_bytes + plan.b_bytes;
      uint32_t it = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const TmaTile tc = tma_tile(p, t);
        for (int kb = 0; kb < tc.nkb; ++kb, ++it) {
          const int s = (int)(it % (uint32_t)stages);
          const uint32_t round = it / (uint32_t)stages;
          if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t st = smem_u32(smem + (size_t)s * plan.stage_bytes);
          const uint32_t a_hi = st, b_hi = st + 2u * plan.a_bytes;
          const int k0 = (int)(tc.k_begin + (int64_t)kb * BK);
          mbar_expect_tx(&raw_full[s], tx);
          if constexpr (kAK) {
            tma_load_2d(a_hi, &map_a, k0, (int)tc.m0, &raw_full[s]);
          } else {
#pragma unroll
            for (int b = 0; b < BM / 32; ++b) tma_load_2d(a_hi + 4096u * b, &map_a, (int)tc.m0 + 32 * b, k0, &raw_full[s]);
          }
          if constexpr (kBK) {
            tma_load_2d(b_hi, &map_b, k0, (int)tc.n0, &raw_full[s]);
          } else {
            for (int b = 0; b < bn / 32; ++b) tma_load_2d(b_hi + 4096u * b, &map_b, (int)tc.n0 + 32 * b, k0, &raw_full[s]);
          }
        }
      }
      // Let every issued load land before the CTA can exit.
      const uint32_t n = it < (uint32_t)stages ? it : (uint32_t)stages;
      for (uint32_t i = it - n; i < it; ++i) mbar_wait_drain(&raw_full[i % (uint32_t)stages], (i / (uint32_t)stages) & 1u);
    }
  } else if (warp >= kConvWarp0 && warp < kTmaEpiWarp0) {
    // ---------------------------------------------------------- converters
    const int ct = threadIdx.x - 32 * kConvWarp0;
    constexpr int nct = kConvWarps * 32;
    const int a_words = (int)(plan.a_bytes / 16), b_words = (int)(plan.b_bytes / 16);
    uint32_t it = 0;
    bool ok = true;
    for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
      const TmaTile tc = tma_tile(p, t);
      for (int kb = 0; kb < tc.nkb; ++kb, ++it) {
        const int s = (int)(it % (uint32_t)stages);
        if (!mbar_wait(&raw_full[s], (it / (uint32_t)stages) & 1u, abort_flag)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + (size_t)s * plan.stage_bytes;
        split_words(st, st + plan.a_bytes, a_words, ct, nct);
        uint8_t* bh = st + 2 * plan.a_bytes;
        split_words(bh, bh + plan.b_bytes, b_words, ct, nct);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(&conv_full[s]);
      }
    }
  } else if (warp == kTmaMmaWarp) {
    // -------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_tf32_major(bn, !kAK, !kBK);
      uint32_t it = 0, g = 0;  // g counts chunks
      bool ok = true;
      for (int64_t t = blockIdx.x; t < tiles && ok && !*abort_flag; t += gridDim.x) {
        const TmaTile tc = tma_tile(p, t);
        for (int kb0 = 0; kb0 < tc.nkb && ok; kb0 += kChunkKB, ++g) {
          const int a = (int)(g & 1u);
          const uint32_t use = g >> 1;
          if (use > 0 && !mbar_wait(&chunk_empty[a], (use - 1) & 1u, abort_flag)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t d = tmem_base + (uint32_t)a * acc_cols;
          const int kb1 = kb0 + kChunkKB < tc.nkb ? kb0 + kChunkKB : tc.nkb;
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s = (int)(it % (uint32_t)stages);
            if (!mbar_wait(&conv_full[s], (it / (uint32_t)stages) & 1u, abort_flag)) {
              ok = false;
              break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t st = smem_u32(smem + (size_t)s * plan.stage_bytes);
            const uint32_t a_hi = st, a_lo = st + plan.a_bytes;
            const uint32_t b_hi = st + 2u * plan.a_bytes, b_lo = b_hi + plan.b_bytes;
#pragma unroll
            for (int j = 0; j < BK / 8; ++j) {
              mma_tf32(d, operand_desc<kAK>(a_lo, j), operand_desc<kBK>(b_hi, j), idesc,
                       (kb > kb0 || j > 0) ? 1u : 0u);
              mma_tf32(d, operand_desc<kAK>(a_hi, j), operand_desc<kBK>(b_lo, j), idesc, 1u);
              mma_tf32(d, operand_desc<kAK>(a_hi, j), operand_desc<kBK>(b_hi, j), idesc, 1u);
            }
            mma_commit(&empty[s]);
          }
          mma_commit(&chunk_full[a]);
        }
      }
    }
  } else {
    // ----------------------------------------------------------- epilogue
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_addr = tmem_base + lane_off + 2u * acc_cols;
    uint8_t* ebuf = smem + plan.epi_offset + (size_t)(warp - kTmaEpiWarp0) * 2 * kEpiBuf;
    uint32_t g = 0, nstore = 0;
    bool ok = true;
    for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
      const TmaTile tc = tma_tile(p, t);
      const int nch = (tc.nkb + kChunkKB - 1) / kChunkKB;
      const int row0 = (int)tc.m0 + quarter * 32;
      for (int ch = 0; ch < (nch > 0 ? nch : 1); ++ch) {
        const bool first = ch == 0, last = ch + 1 >= nch;
        const int a = (int)(g & 1u);
        if (nch > 0) {
          if (!mbar_wait(&chunk_full[a], (g >> 1) & 1u, abort_flag)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        }
        const uint32_t p_addr = tmem_base + lane_off + (uint32_t)a * acc_cols;
        for (int c = 0; c < bn; c += 32) {
          float v[32];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float* vh = v + 16 * h;
            if (nch > 0) {
              float pv[16];
              tmem_ld16(p_addr + (uint32_t)(c + 16 * h), pv);
              if (!first) {
                float sv[16];
                tmem_ld16(s_addr + (uint32_t)(c + 16 * h), sv);
#pragma unroll
                for (int e = 0; e < 16; ++e) pv[e] = __fadd_rn(sv[e], pv[e]);
              }
              if (!last) tmem_st16(s_addr + (uint32_t)(c + 16 * h), pv);
#pragma unroll
              for (int e = 0; e < 16; ++e) vh[e] = pv[e];
            } else {
#pragma unroll
              for (int e = 0; e < 16; ++e) vh[e] = 0.0f;
            }
          }
          if (!last) continue;
          if (p.bias) {
            const int64_t n = tc.n0 + c;
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (n + e < p.N) v[e] += __ldg(p.bias + n + e);
          }
          if (row0 >= p.M || tc.n0 + c >= p.N) continue;  // block wholly outside D
          // 32 x 32 block -> swizzled buffer -> TMA store
          const uint32_t b = nstore & 1u;
          if (nstore >= 2) {
            if (lane == 0) bulk_wait_read1();
            __syncwarp();
          }
          uint8_t* buf = ebuf + b * kEpiBuf;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(buf + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            if (p.partial) tma_store_3d(&map_d, (int)tc.n0 + c, row0, tc.z, smem_u32(buf));
            else tma_store_2d(&map_d, (int)tc.n0 + c, row0, smem_u32(buf));
            bulk_commit();
          }
          ++nstore;
        }
        if (nch > 0) {
          if (!last) asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          mbar_arrive(&chunk_empty[a]);  // P may be refilled
          ++g;
        }
      }
    }
    if (lane == 0) bulk_wait_all();
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == kTmaMmaWarp) {
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols)
                 : "memory");
  }
}

}  // namespace tc
}  // namespace b2
