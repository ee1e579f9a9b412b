// conv_wgrad.cu -- Conv2D filter gradient for inputs with few channels (the
// README network's stem: a 3x7 filter over 3 input channels, strides (1, 2)),
// on the CUDA cores, optionally fused with the BatchNorm -> ReLU backward that
// produces its output gradient.
//
// Reference: kernels/conv2d_kernels.cl:123-158 (conv2d_backprop_filter: one
// work-item per filter element, a serial fp32 loop over every output pixel).
//
//   dW[kh, kw, ci, co] = sum over (n, ho, wo) of
//                        x[n, ho*sH - pH + kh, wo*sW - pW + kw, ci] * dy[n, ho, wo, co]
//
// Why the CUDA cores: per output pixel the work is, for each filter row kh, an
// outer product of the input window (kW*Ci = 21 contiguous floats of one NHWC
// input row) with the Co output-gradient values.  As a GEMM its M = kH*kW*Ci =
// 63 fills half of a 128-row MMA, and its im2col^T operand has to be
// transposed element by element by converter warps; here each thread keeps the
// window in registers instead: a thread owns (kh, CPT = 3 or 4 output
// channels) and accumulates 21 x CPT sums over WPT = 4 adjacent output
// columns, whose windows overlap (stride 2: each column adds 2 pixels).
//
// Work unit: R output rows (n, ho..ho+R-1), or, when a row's dy does not fit a
// slot, a chunk of Wc of one row's columns.  A CTA (one per SM) walks a
// contiguous range of units through a ring of shared-memory slots with three
// warp roles and no block-wide barrier:
//
//   warp 0        lane 0 stages a unit with two or three 1-D bulk copies
//                 (cp.async.bulk, completion on the slot's FULL mbarrier): the
//                 unit's dy block (contiguous in NHWC), FUSED also the BatchNorm
//                 input block, and the contiguous run of input rows the unit
//                 reads (clipped to the image); its unit bookkeeping is
//                 incremental, without divisions, so it keeps ahead;
//   warps 1..2    (FUSED) compute dy = the BatchNorm -> ReLU backward of the
//                 staged dz and y, with the per-channel constants in
//                 registers, into the slot, and arrive on DX_READY;
//   12 warps      consumers, three per scheduler: teams of kH * Co/CPT threads
//                 split the unit's column groups; a thread loads its input
//                 window (input columns outside the image read as zero), its
//                 WPT x CPT dy values and issues the FMAs; each warp arrives on
//                 EMPTY.
//
// Every wait is bounded.  At the end the CTA folds its teams in team order
// and writes one partial per filter element; a second kernel adds the CTA
// partials in block order, so results are deterministic.
//
// FUSED: dy is not read but computed in shared memory from the BatchNorm ->
// ReLU backward's inputs (dz and the BN input y) and its per-channel
// constants, with the same arithmetic as the BatchNorm dx pass (so the filter
// gradient equals the unfused sequence's bit for bit), and never written to
// HBM.
#include <climits>

#include "bn_common.cuh"
#include "conv_common.cuh"

namespace b2 {

static __device__ unsigned int g_wg_timeouts = 0;

namespace {

constexpr int kWgConsumerWarps = 12;  // three per scheduler
constexpr int kWgConsumers = 32 * kWgConsumerWarps;
constexpr int kWgDxWarps = 2;         // FUSED: dx warps
constexpr int kWgWpt = 4;             // output columns per consumer thread per group
constexpr int kWgMaxStages = 8;
constexpr int kWgMargin = 64;         // floats before / after the staged input rows
constexpr int kWgSlotBudget = 40 * 1024;  // target bytes of one slot

__host__ __device__ constexpr int wg_threads(bool fused) {
  return 32 * (1 + (fused ? kWgDxWarps : 0) + kWgConsumerWarps);
}

struct WgGeom {
  int N, H, W, Co, kH, sH, pH, pW, Ho, Wo;
  int cpt;      // output channels per consumer thread (3 or 4)
  int combos;   // threads per team: kH * Co / cpt
  int teams;    // consumer teams
  int R;        // output rows per unit (1 when chunks > 1)
  int Wc;       // output columns per unit (Wo when chunks == 1)
  int chunks;   // units per block of R rows
  int xrows;    // input rows staged per unit: (R - 1) * sH + kH
  int slot;     // floats per slot
  int stages;   // slots
  int units;    // (N * Ho / R) * chunks
  int upb;      // units per CTA
  WaitParams wait;
};

struct BnDx {
  const float *mean, *inv_std, *k1, *grad_beta, *grad_gamma, *gamma, *beta;
  float nhw_f;
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(b)), "r"(count) : "memory");
}

__device__ __forceinline__ void bar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(b)) : "memory");
}

__device__ __forceinline__ void bar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(b)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool bar_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(b)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for the phase of parity `parity`, at most limit_ns (or until another
// wait of the CTA gave up: *abort); an expiry is counted, raises *abort and
// sets the library's host-mapped expiry word.
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t parity, const WaitParams& wp, volatile int* abort) {
  if (bar_try_wait(b, parity)) return true;
  const uint64_t t0 = now_ns();
  for (uint32_t it = 0;; ++it) {
    if (bar_try_wait(b, parity)) return true;
    if ((it & 255u) == 0) {
      if (*abort) return false;
      if (now_ns() - t0 > wp.limit_ns) {
        atomicAdd(&g_wg_timeouts, 1u);
        *abort = 1;
        if (wp.expired) {
          *reinterpret_cast<volatile unsigned int*>(wp.expired) = 1u;
          __threadfence_system();
        }
        return false;
      }
    }
  }
}

__device__ __forceinline__ void bulk_g2s(float* dst, const float* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

// Where a unit is: output rows ho .. ho + R - 1 of image n, columns wo0 ..
// wo0 + Wc - 1; advanced one unit at a time without dividing.
struct UnitPos {
  int n, ho, c;
  __device__ void start(const WgGeom& g, int u) {
    const int rb = u / g.chunks;
    c = u - rb * g.chunks;
    const int row = rb * g.R;
    n = row / g.Ho;
    ho = row - n * g.Ho;
  }
  __device__ void next(const WgGeom& g) {
    if (++c == g.chunks) {
      c = 0;
      ho += g.R;
      if (ho == g.Ho) {
        ho = 0;
        ++n;
      }
    }
  }
};

// Slot layout (floats): dy (or dz) block [R][Wc][Co]; FUSED: BN-input block
// and the computed dy block, same shape; then kWgMargin, the input rows
// [xrows][W*Ci], kWgMargin.
__host__ __device__ inline int wg_block(const WgGeom& g) { return g.R * g.Wc * g.Co; }
__host__ __device__ inline int wg_xoff(const WgGeom& g, bool fused) {
  return wg_block(g) * (fused ? 3 : 1) + kWgMargin;
}
__host__ __device__ inline int wg_slot_floats(const WgGeom& g, bool fused) {
  return wg_xoff(g, fused) + g.xrows * g.W * 3 + kWgMargin;
}

// Dynamic shared memory: max(ring, team fold) + barriers.
template <int KWC>
__host__ __device__ inline int wg_smem_bytes(const WgGeom& g) {
  const int ring = g.stages * g.slot;
  const int fold = g.teams * g.combos * KWC * g.cpt;
  const int body = (ring > fold ? ring : fold) * 4;
  return body + 8 * 3 * kWgMaxStages + 16;
}

template <int KW, int CI, int SW, int CPT, bool FUSED>
__global__ void __launch_bounds__(wg_threads(FUSED), 1)
    conv_wgrad_rows_kernel(const float* __restrict__ x, const float* __restrict__ dy,
                           const float* __restrict__ ybn, BnDx bn, WgGeom g, float* __restrict__ partial) {
  constexpr int KWC = KW * CI;
  constexpr int STEP = SW * CI;                    // window shift per output column
  constexpr int NWIN = (kWgWpt - 1) * STEP + KWC;  // floats of x a thread's columns read per filter row
  constexpr int kConsumer0 = 32 * (1 + (FUSED ? kWgDxWarps : 0));
  extern __shared__ __align__(16) float wsm[];
  const int S = g.stages, Co = g.Co, blk = wg_block(g), xoff = wg_xoff(g, FUSED), WCI = g.W * CI;
  const int fold_floats = g.teams * g.combos * KWC * CPT;
  const int body = S * g.slot > fold_floats ? S * g.slot : fold_floats;
  uint64_t* full = reinterpret_cast<uint64_t*>(wsm + body);
  uint64_t* dxr = full + kWgMaxStages;
  uint64_t* empty = dxr + kWgMaxStages;
  __shared__ int s_abort;
  volatile int* abort = &s_abort;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int u_begin = blockIdx.x * g.upb;
  const int nu = (u_begin + g.upb < g.units ? u_begin + g.upb : g.units) - u_begin;

  // the margins around the input rows are never written by the copies
  for (int i = tid; i < S * g.slot; i += blockDim.x) wsm[i] = 0.0f;
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (tid == 0) {
    s_abort = 0;
    for (int i = 0; i < S; ++i) {
      bar_init(&full[i], 1);
      bar_init(&dxr[i], kWgDxWarps);
      bar_init(&empty[i], kWgConsumerWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  float acc[KWC][CPT];
#pragma unroll
  for (int k = 0; k < KWC; ++k)
#pragma unroll
    for (int c = 0; c < CPT; ++c) acc[k][c] = 0.0f;
  const int ct = tid - kConsumer0;
  const int ng = g.Co / CPT;  // channel groups
  const int team = ct >= 0 ? ct / g.combos : g.teams, r = ct >= 0 ? ct - team * g.combos : 0;
  const int kh = r / ng, cgrp = r - kh * ng;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int issued = 0;
      UnitPos up;
      up.start(g, u_begin);
      for (int i = 0; i < nu; ++i, ++issued, up.next(g)) {
        const int sl = i % S;
        if (i >= S && !bar_wait(&empty[sl], (uint32_t)(i / S - 1) & 1u, g.wait, abort)) break;
        float* base = wsm + (size_t)sl * g.slot;
        const int wo0 = up.c * g.Wc;
        const int nv = g.Wo - wo0 < g.Wc ? g.Wo - wo0 : g.Wc;
        // input rows (R - 1) * sH + kH from ho * sH - pH, clipped to the image
        int h0 = up.ho * g.sH - g.pH, h1 = h0 + g.xrows;
        const int c0 = h0 < 0 ? 0 : h0, c1 = h1 > g.H ? g.H : h1;
        const uint32_t dbytes = (uint32_t)(g.R * nv * Co * 4);
        const uint32_t xbytes = c1 > c0 ? (uint32_t)((c1 - c0) * WCI * 4) : 0u;
        bar_expect_tx(&full[sl], dbytes * (FUSED ? 2u : 1u) + xbytes);
        const int64_t d0 = (((int64_t)up.n * g.Ho + up.ho) * g.Wo + wo0) * Co;
        bulk_g2s(base, dy + d0, dbytes, &full[sl]);
        if (FUSED) bulk_g2s(base + blk, ybn + d0, dbytes, &full[sl]);
        if (xbytes)
          bulk_g2s(base + xoff + (c0 - h0) * WCI, x + ((int64_t)up.n * g.H + c0) * WCI, xbytes, &full[sl]);
      }
      // let every issued copy land before the CTA can leave its ring
      const int first = issued > S ? issued - S : 0;
      WaitParams drain = g.wait;
      drain.limit_ns = kDefaultWaitLimitNs;
      int no_abort = 0;
      for (int i = first; i < issued; ++i)
        bar_wait(&full[i % S], (uint32_t)(i / S) & 1u, drain, &no_abort);
    }
  } else if (FUSED && warp <= kWgDxWarps) {
    // ------------------------------------------------------- dx (FUSED)
    // thread t: channel quad t % cq of columns t / cq, t / cq + per, ...
    const int cq = Co / 4;
    const int t = tid - 32, per = (32 * kWgDxWarps) / cq;
    const bool active = t < per * cq;
    const int dcq = active ? t % cq : 0, wl0 = t / cq;
    float m[4], iv[4], k1[4], gb[4], gg[4], ga[4], be[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int ch = 4 * dcq + j;
      m[j] = bn.mean[ch];
      iv[j] = bn.inv_std[ch];
      k1[j] = bn.k1[ch];
      gb[j] = bn.grad_beta[ch];
      gg[j] = bn.grad_gamma[ch];
      ga[j] = bn.gamma[ch];
      be[j] = bn.beta[ch];
    }
    UnitPos up;
    up.start(g, u_begin);
    for (int i = 0; i < nu; ++i, up.next(g)) {
      const int sl = i % S;
      if (!bar_wait(&full[sl], (uint32_t)(i / S) & 1u, g.wait, abort)) break;
      const int wo0 = up.c * g.Wc;
      const int nv = g.Wo - wo0 < g.Wc ? g.Wo - wo0 : g.Wc;
      float* base = wsm + (size_t)sl * g.slot;
      if (active) {
        for (int rr = 0; rr < g.R; ++rr) {
#pragma unroll 2
          for (int wl = wl0; wl < nv; wl += per) {
            const int e = (rr * g.Wc + wl) * Co + 4 * dcq;
            const float4 z4 = *reinterpret_cast<const float4*>(base + e);
            const float4 y4 = *reinterpret_cast<const float4*>(base + blk + e);
            float4 o;
            o.x = bn_grad_dx_value<true>(y4.x, z4.x, m[0], iv[0], k1[0], gb[0], gg[0], ga[0], be[0], bn.nhw_f);
            o.y = bn_grad_dx_value<true>(y4.y, z4.y, m[1], iv[1], k1[1], gb[1], gg[1], ga[1], be[1], bn.nhw_f);
            o.z = bn_grad_dx_value<true>(y4.z, z4.z, m[2], iv[2], k1[2], gb[2], gg[2], ga[2], be[2], bn.nhw_f);
            o.w = bn_grad_dx_value<true>(y4.w, z4.w, m[3], iv[3], k1[3], gb[3], gg[3], ga[3], be[3], bn.nhw_f);
            *reinterpret_cast<float4*>(base + 2 * blk + e) = o;
          }
        }
      }
      __syncwarp();
      if (lane == 0) bar_arrive(&dxr[sl]);
    }
  } else if (ct >= 0) {
    // ----------------------------------------------------------- consumers
    const bool active = team < g.teams;
    const int groups = (g.Wc + kWgWpt - 1) / kWgWpt;  // column groups of a unit row
    UnitPos up;
    up.start(g, u_begin);
    for (int i = 0; i < nu; ++i, up.next(g)) {
      const int sl = i % S;
      // FULL (the staged input rows; in the fused kernel it has completed
      // before DX_READY, but waiting on it makes the bulk copies' writes
      // visible to this thread directly) then, fused, DX_READY
      if (!bar_wait(&full[sl], (uint32_t)(i / S) & 1u, g.wait, abort)) break;
      if (FUSED && !bar_wait(&dxr[sl], (uint32_t)(i / S) & 1u, g.wait, abort)) break;
      const int wo0 = up.c * g.Wc;
      const int nv = g.Wo - wo0 < g.Wc ? g.Wo - wo0 : g.Wc;
      const float* base = wsm + (size_t)sl * g.slot;
      const float* dsrc0 = base + (FUSED ? 2 * blk : 0) + CPT * cgrp;
      const int h_base = up.ho * g.sH - g.pH;  // first staged input row (may be outside the image)
      if (active) {
        for (int rr = 0; rr < g.R; ++rr) {
          const int hi = h_base + rr * g.sH + kh;
          if (hi < 0 || hi >= g.H) continue;  // a zero-padding row contributes nothing
          const float* xrow = base + xoff + (hi - h_base) * WCI;  // staged row hi - h_base
          for (int gi = team; gi < groups; gi += g.teams) {
            const int col0 = gi * kWgWpt;
            if (col0 >= nv) break;
            const int cin0 = SW * (wo0 + col0) - g.pW;  // input column of window entry 0
            const float* xw = xrow + cin0 * CI;
            // at the image edge, input columns outside it read as zero (SAME padding)
            const bool edge = cin0 < 0 || cin0 + (NWIN - 1) / CI >= g.W;
            auto ld = [&](int q) {
              float v = xw[q];
              if (edge) {
                const int cc = cin0 + q / CI;
                if (cc < 0 || cc >= g.W) v = 0.0f;
              }
              return v;
            };
            const float* ds = dsrc0 + (rr * g.Wc + col0) * Co;
            float d[kWgWpt][CPT];
#pragma unroll
            for (int j = 0; j < kWgWpt; ++j) {
              const bool ok = col0 + j < nv;
#pragma unroll
              for (int c = 0; c < CPT; ++c) d[j][c] = ok ? ds[j * Co + c] : 0.0f;
            }
            // a rolling window of KWC + STEP floats: column j reads entries
            // j*STEP .. j*STEP + KWC - 1, entry q kept at q % NRING
            constexpr int NRING = KWC + STEP;
            float win[NRING];
#pragma unroll
            for (int q = 0; q < KWC; ++q) win[q] = ld(q);
#pragma unroll
            for (int j = 0; j < kWgWpt; ++j) {
              if (j > 0) {
#pragma unroll
                for (int t = 0; t < STEP; ++t) win[(j * STEP + KWC - STEP + t) % NRING] = ld(j * STEP + KWC - STEP + t);
              }
#pragma unroll
              for (int k = 0; k < KWC; ++k)
#pragma unroll
                for (int c = 0; c < CPT; ++c) acc[k][c] = fmaf(win[(j * STEP + k) % NRING], d[j][c], acc[k][c]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) bar_arrive(&empty[sl]);
    }
  }
  __syncthreads();  // every copy has landed (producer drain) and every slot is read

  // Fold the teams in team order, one partial per filter element (HWIO).
  float* fold = wsm;
  const bool computes = ct >= 0 && team < g.teams;
  if (computes) {
#pragma unroll
    for (int k = 0; k < KWC; ++k)
#pragma unroll
      for (int c = 0; c < CPT; ++c) fold[((size_t)(team * g.combos + r) * KWC + k) * CPT + c] = acc[k][c];
  }
  __syncthreads();
  if (computes && team == 0) {
    const int64_t F = (int64_t)g.kH * KWC * Co;
    float* out = partial + (int64_t)blockIdx.x * F;
#pragma unroll 1
    for (int k = 0; k < KWC; ++k) {
      float sum[CPT];
#pragma unroll
      for (int c = 0; c < CPT; ++c) sum[c] = fold[((size_t)r * KWC + k) * CPT + c];
      for (int t = 1; t < g.teams; ++t)
#pragma unroll
        for (int c = 0; c < CPT; ++c) sum[c] += fold[((size_t)(t * g.combos + r) * KWC + k) * CPT + c];
#pragma unroll
      for (int c = 0; c < CPT; ++c) out[((int64_t)kh * KWC + k) * Co + CPT * cgrp + c] = sum[c];
    }
  }
}

// out[f] = sum over CTAs b of part[b][f], in a fixed order: CTA (32 elements
// x kSumParts); part j adds blocks j, j + kSumParts, ... in order, then the
// parts are added in part order.
constexpr int kSumParts = 16;
__global__ void __launch_bounds__(32 * kSumParts)
    wgrad_block_sum_kernel(const float* __restrict__ part, int blocks, int F, float* __restrict__ out) {
  __shared__ float s[kSumParts][32];
  const int f = blockIdx.x * 32 + threadIdx.x;
  float a = 0.0f;
  if (f < F) {
#pragma unroll 4
    for (int b = threadIdx.y; b < blocks; b += kSumParts) a += __ldg(part + (int64_t)b * F + f);
  }
  s[threadIdx.y][threadIdx.x] = a;
  __syncthreads();
  if (threadIdx.y == 0 && f < F) {
    float t = s[0][threadIdx.x];
    for (int j = 1; j < kSumParts; ++j) t += s[j][threadIdx.x];
    out[f] = t;
  }
}

constexpr int kStemKW = 7, kStemCI = 3, kStemSW = 2;

// The geometry of a launch: units of R rows (or column chunks of one row)
// whose fused slot fits kWgSlotBudget where possible, and the largest ring (at
// most kWgMaxStages slots) that fits `max_smem`; stages = 0 if not even three
// fit.
WgGeom wg_geom(const ConvGeom& g, bool fused, int max_smem) {
  constexpr int KWC = kStemKW * kStemCI;
  WgGeom w{};
  w.N = (int)g.N; w.H = (int)g.H; w.W = (int)g.W; w.Co = (int)g.Co; w.kH = (int)g.kH; w.sH = (int)g.sH;
  w.pH = (int)g.pH; w.pW = (int)g.pW; w.Ho = (int)g.Ho; w.Wo = (int)g.Wo;
  w.cpt = (w.Co % 3 == 0 && w.kH * (w.Co / 3) <= kWgConsumers) ? 3 : 4;
  w.combos = w.kH * (w.Co / w.cpt);
  w.teams = kWgConsumers / w.combos;
  // slot bytes of one output column, sized for the fused kernel in both: the
  // unit shape fixes the order of the additions, and the fused and plain
  // kernels must add in the same order (their results agree bit for bit)
  const int per_col = w.Co * 4 * 3;
  w.R = 1;
  if ((int64_t)w.Wo * per_col <= kWgSlotBudget) {
    w.Wc = w.Wo;
    w.chunks = 1;
    for (int r = 4; r >= 2; r /= 2)
      if (w.Ho % r == 0 && (int64_t)r * w.Wo * per_col <= kWgSlotBudget) {
        w.R = r;
        break;
      }
  } else {
    const int unit = w.teams * kWgWpt;  // one column group per team
    int wc = kWgSlotBudget / per_col / unit * unit;
    if (wc < unit) wc = unit;
    w.Wc = wc;
    w.chunks = (int)ceil_div(w.Wo, wc);
  }
  w.xrows = (w.R - 1) * w.sH + w.kH;
  w.slot = (wg_slot_floats(w, fused) + 3) / 4 * 4;
  w.stages = 0;
  for (int st = kWgMaxStages; st >= 3; --st) {
    w.stages = st;
    if (wg_smem_bytes<KWC>(w) <= max_smem) break;
    w.stages = 0;
  }
  return w;
}

}  // namespace

// The shapes this kernel takes: a 7-wide filter over 3 input channels with
// column stride 2 (the README stem at any batch and image height), image
// widths that are a multiple of 4 (input rows are staged with 16-byte bulk
// copies), an even left padding (the window loads are 8-byte aligned), output
// channel counts that are multiples of 4 up to 256, filter heights up to 8,
// 16-byte aligned tensors, and a ring of at least three slots in shared
// memory.
bool conv_wgrad_rows_ok(const ConvGeom& g, const float* x, const float* dy, const float* ybn) {
  if (g.kW != kStemKW || g.Ci != kStemCI || g.sW != kStemSW) return false;
  if (g.Co < 4 || g.Co > 256 || g.Co % 4 != 0 || g.kH < 1 || g.kH > 8 || g.N < 1 || g.Ho < 1 || g.Wo < 1)
    return false;
  if (g.W % 4 != 0 || g.pW % 2 != 0 || g.kH * g.Co / 4 > kWgConsumers) return false;
  if (!aligned16(x) || !aligned16(dy) || (ybn != nullptr && !aligned16(ybn))) return false;
  if (g.W > 1 << 16 || g.H > 1 << 20 || g.N * g.Ho * g.Wo > INT_MAX || g.N * g.H * g.W * 3 > INT_MAX) return false;
  return wg_geom(g, true, 227 * 1024).stages >= 3;
}

namespace {

template <int CPT>
int launch_wgrad_rows(const WgGeom& w, int blocks, int smem, const float* x, const float* dy, const float* ybn,
                      const BnDx* fused, float* part, int device, cudaStream_t s) {
  if (fused) {
    static SmemOptIn opt_in;
    auto k = conv_wgrad_rows_kernel<kStemKW, kStemCI, kStemSW, CPT, true>;
    B2_RETURN_IF_ERROR(opt_in.ensure(reinterpret_cast<const void*>(k), device, smem));
    k<<<blocks, wg_threads(true), smem, s>>>(x, dy, ybn, *fused, w, part);
  } else {
    static SmemOptIn opt_in;
    auto k = conv_wgrad_rows_kernel<kStemKW, kStemCI, kStemSW, CPT, false>;
    B2_RETURN_IF_ERROR(opt_in.ensure(reinterpret_cast<const void*>(k), device, smem));
    k<<<blocks, wg_threads(false), smem, s>>>(x, dy, nullptr, BnDx{}, w, part);
  }
  return check_launch(s, fused ? "conv2d_bn_relu_backprop_filter" : "conv2d_backprop_filter");
}

// dW for a shape conv_wgrad_rows_ok accepts.  fused != nullptr: `dy` is the
// ReLU-output gradient dz and `ybn` the BatchNorm input, and the output
// gradient is the BatchNorm -> ReLU backward of them with these constants.
int wgrad_rows(const ConvGeom& g, const float* x, const float* dy, const float* ybn, const BnDx* fused, float* dw,
               cudaStream_t s) {
  constexpr int KWC = kStemKW * kStemCI;
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  WgGeom w = wg_geom(g, fused != nullptr, d->max_smem_optin);
  B2_REQUIRE(w.stages >= 3, "conv2d_backprop_filter: shared memory too small for this shape");
  w.units = (w.N * w.Ho / w.R) * w.chunks;
  int blocks = w.units < d->sm_count ? w.units : d->sm_count;
  w.upb = (int)ceil_div(w.units, blocks);
  blocks = (int)ceil_div(w.units, w.upb);
  w.wait = wait_params();
  const int smem = wg_smem_bytes<KWC>(w);
  const int64_t F = g.kH * KWC * g.Co;
  Scratch part;
  B2_RETURN_IF_ERROR(part.alloc(sizeof(float) * (size_t)blocks * F, s));
  if (w.cpt == 3)
    B2_RETURN_IF_ERROR(launch_wgrad_rows<3>(w, blocks, smem, x, dy, ybn, fused, part.as<float>(), d->device, s));
  else
    B2_RETURN_IF_ERROR(launch_wgrad_rows<4>(w, blocks, smem, x, dy, ybn, fused, part.as<float>(), d->device, s));
  wgrad_block_sum_kernel<<<(unsigned)ceil_div(F, 32), dim3(32, kSumParts), 0, s>>>(part.as<float>(), blocks,
                                                                                   (int)F, dw);
  return check_launch(s, "conv2d_backprop_filter_sum");
}

}  // namespace

// Expired bounded waits of the stem filter-gradient kernel (read by
// b2_device_timeouts).
unsigned int wg_timeouts() {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_wg_timeouts, sizeof(v));
  return v;
}

int conv_wgrad_rows(const ConvGeom& g, const float* x, const float* dy, float* dw, cudaStream_t s) {
  return wgrad_rows(g, x, dy, nullptr, nullptr, dw, s);
}

}  // namespace b2

using namespace b2;

// The stem's backward when its input needs no gradient: OpenclReluGrad ->
// OpenclBatchNormGrad -> OpenclConv2dBackpropFilter
// (src/ops/relu_ops.cc:101-165, src/ops/batchnorm_ops.cc:288-422,
// src/ops/conv2d_ops.cc:328-448) with the BatchNorm input gradient never
// materialised.
extern "C" int b2_conv2d_batch_norm_relu_backprop_filter(
    b2_stream_t stream, const float* input, const int64_t input_shape[4], const int32_t filter_sizes[4],
    const float* grad_z, const float* bn_input, const int64_t out_shape[4], const float* gamma, const float* beta,
    const float* saved_mean, const float* saved_var, float epsilon, const int32_t* strides, int num_strides,
    const char* padding, float* grad_filter, float* grad_gamma, float* grad_beta) {
  clear_error();
  B2_REQUIRE(filter_sizes != nullptr, "filter_sizes must have 4 elements");
  const int64_t f_shape[4] = {filter_sizes[0], filter_sizes[1], filter_sizes[2], filter_sizes[3]};
  ConvGeom g;
  B2_RETURN_IF_ERROR(check_dims_nonneg(input_shape, 4, "input"));
  B2_RETURN_IF_ERROR(check_dims_nonneg(f_shape, 4, "filter_sizes"));
  B2_RETURN_IF_ERROR(parse_conv_attrs(strides, num_strides, padding, false, &g));
  g.N = input_shape[0]; g.H = input_shape[1]; g.W = input_shape[2]; g.Ci = input_shape[3];
  g.kH = f_shape[0]; g.kW = f_shape[1]; g.Co = f_shape[3];
  finish_geom(&g);
  B2_REQUIRE(input_shape[3] == f_shape[2], "input channels != filter_sizes[2]");
  B2_RETURN_IF_ERROR(check_dims_nonneg(out_shape, 4, "grad_z"));
  B2_REQUIRE(out_shape[0] == g.N && out_shape[1] == g.Ho && out_shape[2] == g.Wo && out_shape[3] == g.Co,
             "grad_z / bn_input shape mismatch");
  B2_REQUIRE(gamma && beta && saved_mean && saved_var, "gamma, beta, saved_mean and saved_var are required");
  B2_RETURN_IF_ERROR(check_int32_sizes(g));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t rows = g.N * g.Ho * g.Wo;
  if (g.Co == 0) return B2_OK;
  if (conv_direct_ok(g) || !conv_wgrad_rows_ok(g, input, grad_z, bn_input) || rows == 0) {
    // any shape b2_conv2d_backprop_filter does not give to this kernel: the
    // two ops in sequence, the input gradient in scratch
    Scratch dx;
    B2_RETURN_IF_ERROR(dx.alloc(sizeof(float) * (size_t)(rows * g.Co > 0 ? rows * g.Co : 1), s));
    B2_RETURN_IF_ERROR(b2_batch_norm_relu_grad(stream, grad_z, out_shape, bn_input, out_shape, gamma, beta,
                                               saved_mean, saved_var, epsilon, dx.as<float>(), grad_gamma,
                                               grad_beta));
    return b2_conv2d_backprop_filter(stream, input, input_shape, filter_sizes, dx.as<float>(), out_shape, strides,
                                     num_strides, padding, grad_filter);
  }
  Scratch chan;
  B2_RETURN_IF_ERROR(chan.alloc(sizeof(float) * 2 * g.Co, s));
  float* k1 = chan.as<float>();
  float* inv = k1 + g.Co;
  B2_RETURN_IF_ERROR(bn_grad_reduce(s, grad_z, bn_input, rows, g.Co, gamma, beta, saved_mean, saved_var, epsilon,
                                    true, grad_gamma, grad_beta, k1, inv));
  const BnDx bn{saved_mean, inv, k1, grad_beta, grad_gamma, gamma, beta, (float)(int)rows};
  return wgrad_rows(g, input, grad_z, bn_input, &bn, grad_filter, s);
}
