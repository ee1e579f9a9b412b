// tma_gemm.cuh -- 3xTF32 GEMM engine fed by the Tensor Memory Accelerator.
//
// D[M,N] = sum_k A[m,k] B[k,n] for Dense forward / backward, 1x1 Conv2D and
// the Conv2D forward / filter gradient of inputs with short rows (the README
// stem).  Per 32-wide k-block:
//
//   A  TMA loads raw fp32 data into a raw stage: a K-major matrix tile (one
//      box {32, 128}, 128-byte swizzle, so the converters' row reads are
//      conflict-free), an MN-major tile (four unswizzled boxes {32 rows,
//      32 k}), or, for the im2col kinds, every NHWC input row the k-block
//      touches (one box of whole rows, zero-filled outside the image).  The
//      converter warps read their row of A (gathering im2col elements from
//      the staged rows), split each element into x = hi + lo (tf32_hi_bits)
//      and write both into a tensor-memory slot (128 lanes = rows, 32 + 32
//      columns) from which the MMA reads A.
//   B  TMA loads the tile in a layout UMMA reads directly (K-major: box
//      {32, BN}, 128-byte swizzle, SBO = 1024 B, k step +32 B; MN-major: BN/32
//      boxes {32, 32} with the 128-byte swizzle of 32-byte atoms, the only
//      MN-major smem layout tf32 UMMA accepts, LBO = 4096 B, SBO = 512 B,
//      k step +1024 B); the converters write hi and lo at the same offsets
//      of an operand stage, so the swizzle carries over.
//
// Out-of-range rows and k are zero-filled by the TMA unit.  One CTA per SM
// loops over output tiles 128 x BN (BN a multiple of 32, <= 96) and split-K
// slices.  Two rings decouple the memory latency from the tensor work: raw
// stages (TMA -> converters) and operand stages (converters -> MMA: B hi/lo
// in shared memory, A hi/lo in TMEM).  Warp roles:
//
//   warp 0       lane 0 waits for a free raw stage (RAW_EMPTY), posts its
//                byte count on RAW_FULL and issues the TMA loads; the first
//                round is issued before the block-wide barrier, overlapping
//                the TMEM allocation.
//   warp 1       allocates all 512 TMEM columns: chunk accumulators P0, P1,
//                the running sum S (only when a tile spans several chunks)
//                and one A slot per operand stage.  Lane 0 waits OP_FULL and
//                issues, per 8-wide k step, P += Alo*Bhi + Ahi*Blo + Ahi*Bhi
//                (tcgen05.mma kind::tf32, A from TMEM, B from shared memory),
//                commits OP_EMPTY per operand stage and CHUNK_FULL per chunk
//                (at most kChunkKB k-blocks).
//   warps 2-9    converters, two groups of four warps (one per TMEM lane
//                quarter) on alternate k-blocks: wait RAW_FULL, read their
//                row of A and a share of B, release the raw stage, wait for a
//                free operand stage, write A into its TMEM slot (tcgen05.st)
//                and B hi / lo into its shared-memory tiles, fence both
//                proxies, arrive OP_FULL.
//   warps 10-13  epilogue: per chunk fold P into S with round-to-nearest fp32
//                adds; after the tile's last chunk, add the bias, write the
//                warp's 32 x BN block as 128-byte-swizzled 32 x 32 pieces into
//                its shared buffer and store them with TMA (clipped to D), so
//                every row leaves as whole 128-byte lines; the buffer is
//                rewritten only after those stores have read it.
//
// Why chunks: the tensor core's fp32 accumulation rounds on every update, so
// long reductions fold every 256 k into S (round-to-nearest fp32 adds), as the
// register-fed engine does.
//
// Every mbarrier wait is bounded (the limit is a launch parameter); on expiry
// the CTA raises its abort flag, lets TMA loads already issued land, waits for
// its own TMA stores and for the MMAs it issued, frees its TMEM and exits; the
// expiry is counted in g_tc_timeouts and set in the host-mapped expiry word,
// so the op calls that follow return B2_ERR_TIMEOUT.
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
constexpr int kTmaMaxStages = 8;    // raw (TMA) stages
constexpr int kTmaMaxOpStages = 4;  // operand stages (B hi/lo in smem + A hi/lo in TMEM)
constexpr int kTmaMaxBN = 96;
constexpr int kTmaMaxResKB = 5;                 // resident B: at most this many k-blocks (K <= 160)
constexpr int64_t kTmaMaxResBytes = 120 << 10;  // and at most this much shared memory
constexpr uint32_t kEpiBuf = 32 * 128;  // one 32 x 32 fp32 output block
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kASlotCols = 2 * BK;  // A hi and lo of one k-block

// How the A tile of a k-block is produced.
enum AKind : int {
  kAMN = 0,         // MN-major matrix: op(r, k) = p[k*ld + r]
  kAK = 1,          // K-major matrix: op(r, k) = p[r*ld + k]
  kAFpropRows = 2,  // Conv2D forward im2col: rows = output pixels, k = (kh, kw, ci)
  kAWgradRows = 3,  // Conv2D filter-grad im2col^T: rows = (kh, kw, ci), k = output pixels
};

// NHWC input geometry for the im2col kinds.  The TMA stages `span` input
// rows covering every output row the k-block touches, each widened to `wcp`
// floats: `xpad` zeros (>= pW*Ci, a multiple of 4) before the row's W*Ci
// values and zeros after them past the right padding, so that every tap of
// every output pixel lands inside the staged row and the converters gather
// without bounds checks; rows outside the image are zero-filled too.
struct ConvRows {
  int H, W, Ci, kW, sH, sW, pH, pW, Ho, Wo;
  int span;  // input rows staged per k-block
  int xpad;  // zeros staged before each row (floats)
  int wcp;   // staged row width (floats, multiple of 4, <= 256)
};

// Division by a divisor fixed at launch, for 32-bit dividends: q = (hi32(n *
// mul) + n) >> shift with mul, shift chosen on the host (Granlund and
// Montgomery, "Division by invariant integers using multiplication", PLDI
// 1994) -- a multiply-high, an add and a shift instead of a division routine
// on the per-tile critical path of every warp role.
struct FastDiv {
  uint32_t d, mul, shift;
  __host__ __device__ FastDiv() : d(1), mul(1), shift(0) {}
  __host__ explicit FastDiv(uint32_t div) : d(div), mul(1), shift(0) {
    while ((1ull << shift) < div) ++shift;
    mul = (uint32_t)(((1ull << 32) * ((1ull << shift) - div)) / div + 1);
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    return (uint32_t)(((uint64_t)__umulhi(n, mul) + n) >> shift);
  }
};

struct TmaProblem {
  ConvRows cr;
  int64_t M, N, K;
  int64_t k_per_split;  // multiple of BK
  int splits;
  int bn;
  const float* bias;  // per-column bias, direct mode only
  bool partial;       // out is [splits][M][N] partials (3-D store map)
  bool use_s;         // some tile spans several chunks: keep a running sum S
  uint32_t a_tx;      // bytes of the raw A load per k-block (<= 16 KB)
  bool relu;          // direct mode: the output is relu(sum + bias)
  int b_res_kb;       // > 0: every tile of a CTA shares one B tile of this many
                      // k-blocks, loaded and split once and kept in shared memory
  FastDiv nt_div, mt_div;  // N tiles, M tiles (tile indices < 2^31)
  FastDiv wo_div, ho_div, kwc_div;  // conv kinds: Wo, Ho and kW * Ci
  WaitParams wait;                  // limit of each pipeline wait, expiry word
};

// TMEM columns used by the accumulators (P0, P1 and, when needed, S).
__host__ __device__ inline uint32_t tma_acc_cols(int bn, bool use_s) { return (uint32_t)bn * (use_s ? 3u : 2u); }

struct TmaSmem {
  int raw_stages, op_stages;
  uint32_t a_bytes, b_bytes, raw_bytes, op_bytes, op_offset, epi_offset, bar_offset, table_offset, total;
};

// Conv2D-forward im2col: staged-row offset of each k = (kh, kw, ci), one int
// per k, at most this many (K = kH*kW*Ci).  The table is padded with zero
// offsets to a multiple of 32 entries so a k-block reads it four at a time.
constexpr int kMaxImTable = 1024;
__host__ __device__ inline int im_table_entries(int64_t K) { return (int)((K + 31) / 32 * 32); }

// Shared memory: a ring of raw stages (TMA destinations: raw A tile + raw B
// tile), a ring of operand stages (B hi tile + B lo tile, read by the MMA),
// the epilogue buffers and the barriers.  With a resident B (b_res_kb > 0)
// the raw stages hold A only and the operand area holds B hi / lo of every
// k-block of the CTA's B tile, indexed by k-block.
__host__ __device__ inline TmaSmem tma_smem_plan(int bn, int raw_stages, int op_stages, int table_entries,
                                                 int b_res_kb = 0) {
  TmaSmem s;
  s.raw_stages = raw_stages;
  s.op_stages = op_stages;
  s.a_bytes = (uint32_t)BM * BK * 4;
  s.b_bytes = (uint32_t)bn * BK * 4;
  s.raw_bytes = s.a_bytes + (b_res_kb > 0 ? 0u : s.b_bytes);
  s.op_bytes = 2 * s.b_bytes;
  s.op_offset = s.raw_bytes * (uint32_t)raw_stages;
  s.epi_offset = s.op_offset + s.op_bytes * (uint32_t)(b_res_kb > 0 ? b_res_kb : op_stages);
  s.bar_offset = s.epi_offset + 4 * (uint32_t)(bn / 32) * kEpiBuf;  // a 32 x BN block per epilogue warp
  // the offset table is read as int4: keep it 16-byte aligned
  s.table_offset = (s.bar_offset + 8 * (2 * kTmaMaxStages + 2 * kTmaMaxOpStages + 4 + 3) + 16 + 15) & ~15u;
  s.total = s.table_offset + 4 * (uint32_t)table_entries + 1024;  // + alignment slack
  return s;
}

// ------------------------------------------------------------ PTX helpers

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
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
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 32 consecutive TMEM columns of this warp's 32 lanes; pair with tmem_wait_ld.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 3xTF32 operand split: x = hi + lo with hi = tf32(x) rounded to nearest,
// ties away from zero (one `cvt.rna.tf32.f32`, the same bits as adding half a
// tf32 ulp to the magnitude and clearing the 13 dropped bits; Inf stays Inf,
// NaN stays NaN) and lo = x - hi, exact in fp32.  The tensor core reads the
// top 19 bits of each element, so lo enters truncated to tf32; since lo has
// either sign that error is unbiased, and hi + lo carries x to within
// 2^-21 |x| (typically ~2^-23).
__device__ __forceinline__ uint32_t tf32_hi_bits(uint32_t u) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(__uint_as_float(u)));
  return r;
}

__device__ __forceinline__ uint32_t tf32_lo_bits(uint32_t u, uint32_t hi) {
  return __float_as_uint(__uint_as_float(u) - __uint_as_float(hi));
}

__device__ __forceinline__ void split_word(uint4 w, uint4& h, uint4& l) {
  h.x = tf32_hi_bits(w.x);
  h.y = tf32_hi_bits(w.y);
  h.z = tf32_hi_bits(w.z);
  h.w = tf32_hi_bits(w.w);
  l.x = tf32_lo_bits(w.x, h.x);
  l.y = tf32_lo_bits(w.y, h.y);
  l.z = tf32_lo_bits(w.z, h.z);
  l.w = tf32_lo_bits(w.w, h.w);
}

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

// D (+)= A * B with A read from tensor memory at column address a_tmem.
__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

template <bool kKMajor>
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int j) {
  if constexpr (kKMajor) return smem_desc_swz(base + (uint32_t)j * 32u, 16u, 1024u, 2u);
  else return smem_desc_swz(base + (uint32_t)j * 1024u, 4096u, 512u, 1u);
}

// Split the landed words i0, i0 + step, ... (at most N of them, below n) of a
// tile in place; all loads are issued before the first store.
template <int N>
__device__ __forceinline__ void split_words(uint8_t* hi, uint8_t* lo, int n, int i0, int step) {
  uint4 w[N];
#pragma unroll
  for (int j = 0; j < N; ++j)
    if (i0 + j * step < n) w[j] = *reinterpret_cast<const uint4*>(hi + 16 * (i0 + j * step));
#pragma unroll
  for (int j = 0; j < N; ++j)
    if (i0 + j * step < n) {
      uint4 h, l;
      split_word(w[j], h, l);
      *reinterpret_cast<uint4*>(hi + 16 * (i0 + j * step)) = h;
      *reinterpret_cast<uint4*>(lo + 16 * (i0 + j * step)) = l;
    }
}

struct TmaTile {
  int64_t m0, n0, k_begin, k_end;
  int z, nkb;
};

__device__ __forceinline__ TmaTile tma_tile(const TmaProblem& p, int64_t t) {
  TmaTile c;
  const uint32_t t32 = (uint32_t)t;
  const uint32_t rest = p.nt_div.div(t32);
  const uint32_t n_idx = t32 - rest * p.nt_div.d;
  const uint32_t z = p.mt_div.div(rest);
  c.m0 = (int64_t)(rest - z * p.mt_div.d) * BM;
  c.z = (int)z;
  c.n0 = (int64_t)n_idx * p.bn;
  c.k_begin = (int64_t)c.z * p.k_per_split;
  c.k_end = c.k_begin + p.k_per_split;
  if (c.k_end > p.K) c.k_end = p.K;
  c.nkb = c.k_end > c.k_begin ? (int)((c.k_end - c.k_begin + BK - 1) / BK) : 0;
  return c;
}

// First output row (n * Ho + ho) of the pixels [p0, ...) and the input row
// its staging starts at.
__device__ __forceinline__ void staged_rows(const TmaProblem& p, int64_t p0, int* n, int* hi_first) {
  const ConvRows& cr = p.cr;
  const int ro = (int)p.wo_div.div((uint32_t)p0);  // pixel indices < 2^31 on these paths
  *n = (int)p.ho_div.div((uint32_t)ro);
  *hi_first = (ro - *n * cr.Ho) * cr.sH - cr.pH;
}

// Loads of one k-block (raw A: tile or staged input rows; raw B tile
// BN x 32) into a raw stage.
template <int AK, bool kBK>
__device__ __forceinline__ void issue_b(const CUtensorMap* map_b, uint32_t dst, uint64_t* bar, int bn, int64_t n0,
                                        int k0) {
  if constexpr (kBK) {
    tma_load_2d(dst, map_b, k0, (int)n0, bar);
  } else {
    for (int b = 0; b < bn / 32; ++b) tma_load_2d(dst + 4096u * b, map_b, (int)n0 + 32 * b, k0, bar);
  }
}

template <int AK, bool kBK>
__device__ __forceinline__ void issue_stage(const CUtensorMap* map_a, const CUtensorMap* map_b, uint32_t st,
                                            uint32_t a_bytes, uint64_t* bar, uint32_t tx, const TmaProblem& p,
                                            const TmaTile& tc, int kb) {
  const uint32_t b_raw = st + a_bytes;
  const int k0 = (int)(tc.k_begin + (int64_t)kb * BK);
  mbar_expect_tx(bar, tx);
  if constexpr (AK == kAK) {
    tma_load_2d(st, map_a, k0, (int)tc.m0, bar);
  } else if constexpr (AK == kAMN) {
#pragma unroll
    for (int b = 0; b < BM / 32; ++b) tma_load_2d(st + 4096u * b, map_a, (int)tc.m0 + 32 * b, k0, bar);
  } else {
    int n, hi_first;
    staged_rows(p, AK == kAFpropRows ? tc.m0 : (int64_t)k0, &n, &hi_first);
    tma_load_3d(st, map_a, -p.cr.xpad, hi_first, n, bar);
  }
  if (p.b_res_kb == 0) issue_b<AK, kBK>(map_b, b_raw, bar, p.bn, tc.n0, k0);
}

// Row r, k = k0 + 16h .. +15 of A, from a landed raw stage.
template <int AK>
__device__ __forceinline__ void read_a_row(const uint8_t* raw, int r, int h, float (&v)[16]) {
  if constexpr (AK == kAK) {
    // [128 rows][128 B], 16-byte chunk j of row r at chunk position j ^ (r & 7)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 q = *reinterpret_cast<const float4*>(raw + r * 128 + (((4 * h + j) ^ (r & 7)) << 4));
      v[4 * j] = q.x;
      v[4 * j + 1] = q.y;
      v[4 * j + 2] = q.z;
      v[4 * j + 3] = q.w;
    }
  } else {
    // [4 blocks][32 k][32 rows]
    const float* col = reinterpret_cast<const float*>(raw + (r >> 5) * 4096) + (r & 31);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = col[(16 * h + i) * 32];
  }
}

// Per-tile part of a converter thread's im2col gather (the row kinds): the
// staged-row offset of its A row, computed once per tile so a k-block costs
// one offset step per element.
struct RowGather {
  int base;  // offset into the staged rows of the row's first element
};

template <int AK>
__device__ __forceinline__ RowGather row_gather(const TmaProblem& p, const TmaTile& tc, int r) {
  const ConvRows& cr = p.cr;
  RowGather g;
  if constexpr (AK == kAFpropRows) {
    // row = output pixel m; its k = (kh, kw, ci) element sits at imtab[k]
    // from the pixel's base (rows m >= M read in-bounds values and are never
    // stored)
    const int m = (int)tc.m0 + r;
    const int ro = (int)p.wo_div.div((uint32_t)m), wo = m - ro * cr.Wo;
    const int j = ro - (int)p.wo_div.div((uint32_t)tc.m0);
    g.base = j * cr.sH * cr.wcp + wo * cr.sW * cr.Ci + (cr.xpad - cr.pW * cr.Ci);
  } else {
    // row = filter element m = (kh, kw, ci); rows m >= M gather element 0's
    // values (never stored)
    int m = (int)tc.m0 + r;
    if (m >= (int)p.M) m = 0;
    const int kwc = cr.kW * cr.Ci;
    const int kh = (int)p.kwc_div.div((uint32_t)m), kwci = m - kh * kwc;
    g.base = kh * cr.wcp + kwci + (cr.xpad - cr.pW * cr.Ci);
  }
  return g;
}

// Both 16-element halves of this thread's A row for the k-block at k0.
template <int AK>
__device__ __forceinline__ void read_a_rows(const uint8_t* raw, const TmaProblem& p, const RowGather& g, int k0,
                                            const int* imtab, float (&v)[2][16]) {
  const ConvRows& cr = p.cr;
  const float* xs = reinterpret_cast<const float*>(raw) + g.base;  // [span][wcp], column c at c + xpad
  if constexpr (AK == kAFpropRows) {
    const int K = (int)p.K;  // < 2^31 on this path (checked on the host)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int k = k0 + 16 * h;
      const int4* t4 = reinterpret_cast<const int4*>(imtab + k);  // padded table: always in bounds
      int off[16];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int4 o = t4[q];
        off[4 * q] = o.x;
        off[4 * q + 1] = o.y;
        off[4 * q + 2] = o.z;
        off[4 * q + 3] = o.w;
      }
      if (k + 16 <= K) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[h][i] = xs[off[i]];
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[h][i] = k + i < K ? xs[off[i]] : 0.0f;
      }
    }
  } else {
    // k = output pixel (ro, wo) at staged offset (ro - ro0)*sH*wcp + wo*sW*Ci,
    // ro0 the k-block's first output row (K is a multiple of 32 on this path)
    const int ro0 = (int)p.wo_div.div((uint32_t)k0);
    const int wo0 = k0 - ro0 * cr.Wo;
    const int step = cr.sW * cr.Ci, wrap = cr.sH * cr.wcp - (cr.Wo - 1) * step;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      int wo = wo0 + 16 * h, b = 0;
      while (wo >= cr.Wo) {  // at most 16 / Wo + 1 times
        wo -= cr.Wo;
        b += cr.sH * cr.wcp;
      }
      b += wo * step;
      const int n1 = cr.Wo - wo;  // pixels left in this output row
      const float* xb = xs + b;
      if (n1 >= 16) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[h][i] = xb[i * step];
      } else if (cr.Wo >= 16) {
        // one row change: every offset is independent of the previous one
#pragma unroll
        for (int i = 0; i < 16; ++i) v[h][i] = xb[i * step + (i >= n1 ? wrap - step : 0)];
      } else {
        int c = 0;
        wo = cr.Wo - n1;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          v[h][i] = xb[c];
          if (++wo == cr.Wo) {
            wo = 0;
            c += wrap;
          } else {
            c += step;
          }
        }
      }
    }
  }
}

__device__ __forceinline__ void split16(const float (&v)[16], uint32_t (&hv)[16], uint32_t (&lv)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    hv[i] = tf32_hi_bits(__float_as_uint(v[i]));
    lv[i] = tf32_lo_bits(__float_as_uint(v[i]), hv[i]);
  }
}

constexpr int kGroupThreads = 128;  // one converter group: a warp per TMEM lane quarter
constexpr int kMaxBWords = kTmaMaxBN * BK * 4 / 16 / kGroupThreads;  // 16-byte B words per thread

template <int AK, bool kBK>
__global__ void __launch_bounds__(kTmaThreads, 1)
    tma_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                    const __grid_constant__ CUtensorMap map_d, const TmaProblem p, const int raw_stages,
                    const int op_stages) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int bn = p.bn;
  const int table_entries = AK == kAFpropRows ? im_table_entries(p.K) : 0;
  const bool bres = p.b_res_kb > 0;
  const TmaSmem plan = tma_smem_plan(bn, raw_stages, op_stages, table_entries, p.b_res_kb);
  int* imtab = reinterpret_cast<int*>(smem + plan.table_offset);
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(smem + plan.bar_offset);
  uint64_t* raw_empty = raw_full + kTmaMaxStages;
  uint64_t* op_full = raw_empty + kTmaMaxStages;
  uint64_t* op_empty = op_full + kTmaMaxOpStages;
  uint64_t* chunk_full = op_empty + kTmaMaxOpStages;  // [2]
  uint64_t* chunk_empty = chunk_full + 2;             // [2]
  uint64_t* b_full = chunk_empty + 2;                 // resident B landed
  uint64_t* b_ready = b_full + 1;                     // resident B split (one arrival per converter warp)
  uint64_t* mma_done = b_ready + 1;                   // every MMA this CTA issued has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  __shared__ WaitState s_wait;
  WaitState* ws = &s_wait;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t nt = (p.N + bn - 1) / bn, mt = (p.M + BM - 1) / BM;
  const int64_t tiles = nt * mt * p.splits;
  const uint32_t acc_cols = (uint32_t)bn;
  const uint32_t a_col0 = tma_acc_cols(bn, p.use_s);  // first A slot column
  const uint32_t tx = p.a_tx + (bres ? 0u : plan.b_bytes);  // bytes the TMA delivers per k-block
  const uint32_t R = (uint32_t)raw_stages, Q = (uint32_t)op_stages;

  // TMA issue cursor (lane 0 of warp 0): tile t, k-block kb, raw stage use it.
  int64_t t_iss = blockIdx.x;
  int kb_iss = 0;
  uint32_t it_iss = 0;
  TmaTile tc_iss{};
  if (threadIdx.x == 0) {
    wait_state_init(ws, p.wait);
    for (int s = 0; s < raw_stages; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], 4);
    }
    for (int s = 0; s < op_stages; ++s) {
      mbar_init(&op_full[s], 4);
      mbar_init(&op_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&chunk_full[a], 1);
      mbar_init(&chunk_empty[a], 128);
    }
    mbar_init(b_full, 1);
    mbar_init(b_ready, kConvWarps);
    mbar_init(mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_map(&map_a);
    prefetch_map(&map_b);
    prefetch_map(&map_d);
    if (bres && blockIdx.x < tiles) {
      // every tile of this CTA has n-tile blockIdx.x % nt (the grid is a multiple of nt)
      mbar_expect_tx(b_full, (uint32_t)p.b_res_kb * plan.b_bytes);
      for (int kb = 0; kb < p.b_res_kb; ++kb)
        issue_b<AK, kBK>(&map_b, smem_u32(smem + plan.op_offset + (size_t)kb * plan.op_bytes), b_full, bn,
                         (blockIdx.x % nt) * bn, kb * BK);
    }
    // The first round of raw stages needs no EMPTY wait: issue it before the
    // block-wide barrier so the loads overlap the TMEM allocation.
    if (t_iss < tiles) tc_iss = tma_tile(p, t_iss);
    while (t_iss < tiles && it_iss < R) {
      issue_stage<AK, kBK>(&map_a, &map_b, smem_u32(smem + (size_t)it_iss * plan.raw_bytes), plan.a_bytes,
                           &raw_full[it_iss], tx, p, tc_iss, kb_iss);
      ++it_iss;
      if (++kb_iss == tc_iss.nkb) {
        kb_iss = 0;
        t_iss += gridDim.x;
        if (t_iss < tiles) tc_iss = tma_tile(p, t_iss);
      }
    }
  }
  if constexpr (AK == kAFpropRows) {
    const int kwc = p.cr.kW * p.cr.Ci;
    for (int k = threadIdx.x; k < table_entries; k += blockDim.x)
      imtab[k] = k < (int)p.K ? (k / kwc) * p.cr.wcp + k % kwc : 0;
  }
  if (warp == kTmaMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
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
      uint32_t s = 0, lap = 1;  // it_iss = lap * R + s (it_iss == R here unless the work ran out)
      while (t_iss < tiles) {
        if (!mbar_wait(&raw_empty[s], (lap - 1) & 1u, ws)) break;
        issue_stage<AK, kBK>(&map_a, &map_b, smem_u32(smem + (size_t)s * plan.raw_bytes), plan.a_bytes,
                             &raw_full[s], tx, p, tc_iss, kb_iss);
        ++it_iss;
        if (++s == R) {
          s = 0;
          ++lap;
        }
        if (++kb_iss == tc_iss.nkb) {
          kb_iss = 0;
          t_iss += gridDim.x;
          if (t_iss < tiles) tc_iss = tma_tile(p, t_iss);
        }
      }
      // Let every issued load land before the CTA can exit.
      const uint32_t n = it_iss < R ? it_iss : R;
      for (uint32_t i = it_iss - n; i < it_iss; ++i) mbar_wait_drain(&raw_full[i % R], (i / R) & 1u, ws->expired);
      if (bres && blockIdx.x < tiles) mbar_wait_drain(b_full, 0, ws->expired);
    }
  } else if (warp >= kConvWarp0 && warp < kTmaEpiWarp0) {
    // ---------------------------------------------------------- converters
    // Two groups of four warps take alternate k-blocks; in a group, the warp
    // of lane quarter q converts rows 32q .. 32q+31 of A (one row a thread)
    // and a share of B's 16-byte words.
    const int group = (warp - kConvWarp0) >> 2;
    const int quarter = warp & 3;
    const int gt = ((warp - kConvWarp0) & 3) * 32 + lane;
    const int row = quarter * 32 + lane;
    const uint32_t a_taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + a_col0;
    const int b_words = bn * BK * 4 / 16;
    uint32_t i = 0;  // k-block sequence number
    uint32_t sr = 0, lap_r = 0, sq = 0, lap_q = 0;  // i = lap_r * R + sr = lap_q * Q + sq
    bool ok = true;
    if (bres && blockIdx.x < tiles) {
      // split the resident B tile in place, all converter warps together
      ok = mbar_wait(b_full, 0, ws);
      if (ok) {
        const int ct = (warp - kConvWarp0) * 32 + lane;
        const int words = p.b_res_kb * b_words;
        for (int w = ct; w < words; w += kConvWarps * 32) {
          const int kbw = w / b_words, wi = w - kbw * b_words;
          uint8_t* hi = smem + plan.op_offset + (size_t)kbw * plan.op_bytes + 16 * wi;
          uint4 h, l;
          split_word(*reinterpret_cast<const uint4*>(hi), h, l);
          *reinterpret_cast<uint4*>(hi) = h;
          *reinterpret_cast<uint4*>(hi + plan.b_bytes) = l;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(b_ready);
    }
    for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
      const TmaTile tc = tma_tile(p, t);
      RowGather rg{};
      if constexpr (AK == kAFpropRows || AK == kAWgradRows) rg = row_gather<AK>(p, tc, row);
      for (int kb = 0; kb < tc.nkb; ++kb, ++i) {
        const uint32_t cur_sr = sr, cur_lr = lap_r, cur_sq = sq, cur_lq = lap_q;
        if (++sr == R) {
          sr = 0;
          ++lap_r;
        }
        if (++sq == Q) {
          sq = 0;
          ++lap_q;
        }
        if ((int)(i & 1u) != group) continue;
        const uint32_t sr = cur_sr, sq = cur_sq;
        if (!mbar_wait(&raw_full[sr], cur_lr & 1u, ws)) {
          ok = false;
          break;
        }
        const uint8_t* raw = smem + (size_t)sr * plan.raw_bytes;
        float va[2][16];
        const int k0 = (int)(tc.k_begin + (int64_t)kb * BK);
        if constexpr (AK == kAFpropRows || AK == kAWgradRows) {
          read_a_rows<AK>(raw, p, rg, k0, imtab, va);
        } else {
          read_a_row<AK>(raw, row, 0, va[0]);
          read_a_row<AK>(raw, row, 1, va[1]);
        }
        uint4 wb[kMaxBWords];
#pragma unroll
        for (int j = 0; j < kMaxBWords; ++j)
          if (!bres && gt + j * kGroupThreads < b_words)
            wb[j] = *reinterpret_cast<const uint4*>(raw + plan.a_bytes + 16 * (gt + j * kGroupThreads));
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[sr]);  // this warp has read the raw stage
        if (cur_lq > 0 && !mbar_wait(&op_empty[sq], (cur_lq - 1) & 1u, ws)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t slot = a_taddr + sq * kASlotCols;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t hv[16], lv[16];
          split16(va[h], hv, lv);
          tmem_st16u(slot + 16u * h, hv);
          tmem_st16u(slot + BK + 16u * h, lv);
        }
        uint8_t* bh = smem + plan.op_offset + (size_t)sq * plan.op_bytes;
#pragma unroll
        for (int j = 0; j < kMaxBWords; ++j)
          if (!bres && gt + j * kGroupThreads < b_words) {
            uint4 h, l;
            split_word(wb[j], h, l);
            *reinterpret_cast<uint4*>(bh + 16 * (gt + j * kGroupThreads)) = h;
            *reinterpret_cast<uint4*>(bh + plan.b_bytes + 16 * (gt + j * kGroupThreads)) = l;
          }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&op_full[sq]);
      }
    }
  } else if (warp == kTmaMmaWarp) {
    // -------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_tf32_major(bn, false, !kBK);
      uint32_t it = 0, g = 0;  // g counts chunks
      uint32_t sq = 0, lap_q = 0;  // it = lap_q * Q + sq
      bool ok = !(bres && blockIdx.x < tiles) || mbar_wait(b_ready, 0, ws);
      // With one split every tile has the same k-blocks: no tile decomposition
      // on this thread's path (an abort is seen by the waits, which check it).
      const int nkb_all = p.splits == 1 ? (int)((p.K + BK - 1) / BK) : -1;
      for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int tile_nkb = nkb_all >= 0 ? nkb_all : tma_tile(p, t).nkb;
        for (int kb0 = 0; kb0 < tile_nkb && ok; kb0 += kChunkKB, ++g) {
          const int a = (int)(g & 1u);
          const uint32_t use = g >> 1;
          const int kb1 = kb0 + kChunkKB < tile_nkb ? kb0 + kChunkKB : tile_nkb;
          // Every barrier operation of this thread queues behind the other
          // warps' shared-memory traffic, so the accumulator and the next two
          // operand stages are probed together (their round trips overlap);
          // only what is not complete yet is waited for.  A stage's previous
          // phase is one this thread consumed, so a completed parity can only
          // mean the current use.
          uint32_t sq1 = sq + 1 == Q ? 0u : sq + 1, lap1 = sq + 1 == Q ? lap_q + 1 : lap_q;
          uint32_t ready = mbar_probe3(&chunk_empty[a], (use - 1) & 1u, &op_full[sq], lap_q & 1u, &op_full[sq1],
                                       lap1 & 1u);
          if (use > 0 && !(ready & 1u) && !mbar_wait(&chunk_empty[a], (use - 1) & 1u, ws)) {
            ok = false;
            break;
          }
          const uint32_t d = tmem_base + (uint32_t)a * acc_cols;
          bool first = true;
          for (int kb = kb0; kb < kb1 && ok;) {
            // One wait and one thread-sync fence (which also covers the
            // accumulator's release at a chunk's start) for a pair of
            // k-blocks when the second stage is ready too.
            if (!first) {
              sq1 = sq + 1 == Q ? 0u : sq + 1;
              lap1 = sq + 1 == Q ? lap_q + 1 : lap_q;
              // bits 1 and 2 as at the chunk's start (bit 0 repeats bit 1)
              ready = mbar_probe3(&op_full[sq], lap_q & 1u, &op_full[sq], lap_q & 1u, &op_full[sq1], lap1 & 1u);
            }
            first = false;
            if (!(ready & 2u) && !mbar_wait(&op_full[sq], lap_q & 1u, ws)) {
              ok = false;
              break;
            }
            const int nkb = (kb + 1 < kb1 && (ready & 4u)) ? 2 : 1;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            for (int u = 0; u < nkb; ++u, ++kb, ++it) {
              const uint32_t a_hi = tmem_base + a_col0 + sq * kASlotCols, a_lo = a_hi + BK;
              const uint32_t b_hi =
                  smem_u32(smem + plan.op_offset + (size_t)(bres ? (uint32_t)kb : sq) * plan.op_bytes);
              // descriptors of the 8-wide k steps differ only in the start
              // address field: +32 B (K-major) or +1024 B (MN-major) a step
              const uint64_t dh = operand_desc<kBK>(b_hi, 0), dl = operand_desc<kBK>(b_hi + plan.b_bytes, 0);
              constexpr uint64_t kStep = kBK ? 2u : 64u;  // in the descriptor's 16-byte units
#pragma unroll
              for (int j = 0; j < BK / 8; ++j) {
                mma_tf32_ts(d, a_lo + 8u * j, dh + kStep * j, idesc, (kb > kb0 || j > 0) ? 1u : 0u);
                mma_tf32_ts(d, a_hi + 8u * j, dl + kStep * j, idesc, 1u);
                mma_tf32_ts(d, a_hi + 8u * j, dh + kStep * j, idesc, 1u);
              }
              mma_commit(&op_empty[sq]);
              if (++sq == Q) {
                sq = 0;
                ++lap_q;
              }
            }
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
    uint8_t* ebuf = smem + plan.epi_offset + (size_t)(warp - kTmaEpiWarp0) * (bn / 32) * kEpiBuf;
    uint32_t g = 0;
    bool ok = true, pending = false;
    for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
      const TmaTile tc = tma_tile(p, t);
      const int nch = (tc.nkb + kChunkKB - 1) / kChunkKB;
      const int row0 = (int)tc.m0 + quarter * 32;
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
        if (last && pending) {  // the previous tile's stores must have read the buffer
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
          pending = false;
        }
        const uint32_t p_addr = tmem_base + lane_off + (uint32_t)a * acc_cols;
        for (int c = 0; c < bn; c += 32) {
          float v[32];
          if (nch > 0) {
            uint32_t pv[32];
            tmem_ld32(p_addr + (uint32_t)c, pv);
            if (!first) {
              uint32_t sv[32];
              tmem_ld32(s_addr + (uint32_t)c, sv);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 32; ++e) v[e] = __fadd_rn(__uint_as_float(sv[e]), __uint_as_float(pv[e]));
            } else {
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(pv[e]);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = 0.0f;
          }
          if (!last) {
            tmem_st16(s_addr + (uint32_t)c, *reinterpret_cast<const float(*)[16]>(v));
            tmem_st16(s_addr + (uint32_t)c + 16u, *reinterpret_cast<const float(*)[16]>(v + 16));
            continue;
          }
          if (p.bias) {
            const int64_t n = tc.n0 + c;
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (n + e < p.N) v[e] += __ldg(p.bias + n + e);
          }
          if (p.relu) {
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = v[e] > 0.0f ? v[e] : 0.0f;  // fmax(v, 0): NaN -> 0, -0 -> +0
          }
          uint8_t* buf = ebuf + (c / 32) * kEpiBuf;  // 32 x 32 block, 128-byte swizzled rows
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(buf + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
        if (nch > 0) {
          if (!last) asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          mbar_arrive(&chunk_empty[a]);  // P may be refilled
          ++g;
        }
        if (last) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0 && row0 < p.M) {
            for (int c = 0; c < bn && tc.n0 + c < p.N; c += 32) {
              const uint32_t src = smem_u32(ebuf + (c / 32) * kEpiBuf);
              if (p.partial) tma_store_3d(&map_d, (int)tc.n0 + c, row0, tc.z, src);
              else tma_store_2d(&map_d, (int)tc.n0 + c, row0, src);
            }
            bulk_commit();
          }
          pending = true;
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
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                 : "memory");
  }
}

}  // namespace tc
}  // namespace b2
