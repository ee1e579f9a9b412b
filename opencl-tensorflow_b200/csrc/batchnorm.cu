// batchnorm.cu -- BatchNorm training forward, inference forward, gradient.
//
// Reference: kernels/batchnorm_kernels.cl and src/ops/batchnorm_ops.cc.  The
// reference reduces with ONE work-item per channel walking all N*H*W rows
// (batchnorm_kernels.cl:35-60, 84-116).  Here each reduction is two
// deterministic stages:
//
//   partial:  a grid of (row block x channel chunk) CTAs; threads own a
//             channel group (4 channels with float4 loads when C % 4 == 0)
//             and stride over the rows of their block, then the CTA folds
//             its rows in a fixed order and writes one partial per channel;
//   finalize: one warp per channel sums the partials (lane-strided, then a
//             shuffle tree) and derives the per-channel outputs and the
//             per-channel constants of the elementwise pass.
//
// The block count depends only on the shape and the SM count, so results
// are bit-reproducible run to run.  The elementwise passes evaluate the
// reference formulas with round-to-nearest intrinsics (no contraction) and
// inv_std = 1/sqrt(var+eps) in IEEE fp32, so, given the same statistics,
// y and grad_x are bit-identical to the reference's formula.
#include <atomic>
#include <mutex>

#include "b2_internal.cuh"

namespace b2 {
namespace {

constexpr int kThreads = 256;

struct ChunkGeom {
  int vec;       // 4 when C % 4 == 0 and pointers are 16-byte aligned, else 1
  int groups;    // channel groups of `vec` channels = C / vec
  int cg;        // channel groups per CTA (<= kThreads)
  int chunks;    // CTAs along the channel axis
  int rpi;       // rows a CTA advances per iteration = kThreads / cg
};

ChunkGeom chunk_geom(int64_t C, bool vec_ok) {
  ChunkGeom g;
  g.vec = vec_ok ? 4 : 1;
  g.groups = (int)(C / g.vec);
  g.cg = g.groups < kThreads ? g.groups : kThreads;
  g.chunks = (int)ceil_div(g.groups, g.cg);
  g.rpi = kThreads / g.cg;
  return g;
}

// Row blocks for the partial stage: about 4 CTAs per SM in total, at least
// 32 rows per CTA.
int row_blocks(int64_t rows, int chunks, int sm_count) {
  int64_t want = (int64_t)sm_count * 4 / chunks;
  if (want < 1) want = 1;
  int64_t cap = ceil_div(rows, 32);
  if (cap < 1) cap = 1;
  return (int)(want < cap ? want : cap);
}

template <int VEC>
struct VecT;
template <>
struct VecT<1> {
  using T = float;
  __device__ static void to(const T& v, float* o) { o[0] = v; }
  __device__ static void from(const float* o, T* p) { *p = o[0]; }
};
template <>
struct VecT<4> {
  using T = float4;
  __device__ static void to(const T& v, float* o) {
    o[0] = v.x;
    o[1] = v.y;
    o[2] = v.z;
    o[3] = v.w;
  }
  __device__ static void from(const float* o, T* p) { *p = make_float4(o[0], o[1], o[2], o[3]); }
};

// y of the forward normalisation (batchnorm_kernels.cl:77-80), operation for
// operation, so a ReLU mask recomputed from it matches the forward's.
__device__ __forceinline__ float bn_y(float x, float m, float iv, float g, float b) {
  return __fadd_rn(__fmul_rn(g, __fmul_rn(__fsub_rn(x, m), iv)), b);
}

// Stage 1.  MODE 0: (sum x, sum x^2).  MODE 1: (sum dy, sum dy * x_hat) with
// x_hat = (x - mean) * inv_std, inv_std = 1/sqrt(var + eps) per channel.
// MODE 2: as MODE 1 with dy = (y > 0 ? dz : 0), the gradient through a ReLU
// applied to the BN output y (the reference's relu_grad), y recomputed from x.
template <int VEC, int MODE>
__global__ void __launch_bounds__(kThreads)
    bn_partial_kernel(const float* __restrict__ x, const float* __restrict__ dy, const float* __restrict__ mean,
                      const float* __restrict__ var, float eps, int64_t rows, int C, ChunkGeom geo,
                      float2* __restrict__ partial, const float* __restrict__ gamma = nullptr,
                      const float* __restrict__ beta = nullptr) {
  using V = typename VecT<VEC>::T;
  __shared__ float s_a[kThreads * VEC];
  __shared__ float s_b[kThreads * VEC];
  __shared__ float s_mean[kThreads * VEC];
  __shared__ float s_inv[kThreads * VEC];
  __shared__ float s_gam[MODE == 2 ? kThreads * VEC : 1];
  __shared__ float s_bet[MODE == 2 ? kThreads * VEC : 1];

  const int chunk = blockIdx.y;
  const int t = threadIdx.x;
  const int cg_local = t % geo.cg;
  const int r_off = t / geo.cg;
  const int group = chunk * geo.cg + cg_local;
  const bool active = r_off < geo.rpi && group < geo.groups;
  const int c0 = group * VEC;

  if (MODE >= 1) {
    for (int i = t; i < geo.cg * VEC; i += kThreads) {
      const int c = chunk * geo.cg * VEC + i;
      if (c < C) {
        s_mean[i] = mean[c];
        s_inv[i] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var[c], eps)));
        if (MODE == 2) {
          s_gam[i] = gamma[c];
          s_bet[i] = beta[c];
        }
      }
    }
    __syncthreads();
  }

  const int64_t per_block = ceil_div(rows, gridDim.x);
  const int64_t r_begin = (int64_t)blockIdx.x * per_block;
  int64_t r_end = r_begin + per_block;
  if (r_end > rows) r_end = rows;

  float acc_a[VEC], acc_b[VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j) acc_a[j] = acc_b[j] = 0.0f;

  if (active) {
    const int loc = cg_local * VEC;
    float m[VEC], inv[VEC], gm[VEC], bt[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      m[j] = MODE >= 1 ? s_mean[loc + j] : 0.0f;
      inv[j] = MODE >= 1 ? s_inv[loc + j] : 0.0f;
      gm[j] = MODE == 2 ? s_gam[loc + j] : 0.0f;
      bt[j] = MODE == 2 ? s_bet[loc + j] : 0.0f;
    }
    constexpr int U = 4;  // rows per thread per iteration: U (or 2U) independent loads in flight
    const int64_t step = (int64_t)geo.rpi;
    int64_t r = r_begin + r_off;
    for (; r + (U - 1) * step < r_end; r += U * step) {
      float v[U][VEC], g[U][VEC];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        VecT<VEC>::to(*reinterpret_cast<const V*>(x + (r + u * step) * C + c0), v[u]);
        if (MODE >= 1) VecT<VEC>::to(*reinterpret_cast<const V*>(dy + (r + u * step) * C + c0), g[u]);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          if (MODE == 0) {
            acc_a[j] += v[u][j];
            acc_b[j] = fmaf(v[u][j], v[u][j], acc_b[j]);
          } else {
            const float xh = (v[u][j] - m[j]) * inv[j];
            const float gv = MODE == 2 && !(bn_y(v[u][j], m[j], inv[j], gm[j], bt[j]) > 0.0f) ? 0.0f : g[u][j];
            acc_a[j] += gv;
            acc_b[j] = fmaf(gv, xh, acc_b[j]);
          }
        }
      }
    }
    for (; r < r_end; r += step) {
      float v[VEC];
      VecT<VEC>::to(*reinterpret_cast<const V*>(x + r * C + c0), v);
      if (MODE == 0) {
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          acc_a[j] += v[j];
          acc_b[j] = fmaf(v[j], v[j], acc_b[j]);
        }
      } else {
        float g[VEC];
        VecT<VEC>::to(*reinterpret_cast<const V*>(dy + r * C + c0), g);
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const float xh = (v[j] - m[j]) * inv[j];
          const float gv = MODE == 2 && !(bn_y(v[j], m[j], inv[j], gm[j], bt[j]) > 0.0f) ? 0.0f : g[j];
          acc_a[j] += gv;
          acc_b[j] = fmaf(gv, xh, acc_b[j]);
        }
      }
    }
  }
  // Fold the rpi row lanes of each channel in a fixed order.
  if (r_off < geo.rpi) {
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      s_a[r_off * geo.cg * VEC + cg_local * VEC + j] = acc_a[j];
      s_b[r_off * geo.cg * VEC + cg_local * VEC + j] = acc_b[j];
    }
  }
  __syncthreads();
  const int width = geo.cg * VEC;
  for (int i = t; i < width; i += kThreads) {
    const int c = chunk * width + i;
    if (c >= C) continue;
    float a = 0.0f, b = 0.0f;
    for (int r = 0; r < geo.rpi; ++r) {
      a += s_a[r * width + i];
      b += s_b[r * width + i];
    }
    partial[(int64_t)c * gridDim.x + blockIdx.x] = make_float2(a, b);  // channel-major: [C][blocks]
  }
}

// Stage 2 for the statistics: saved_mean, saved_var (biased, E[x^2]-mean^2 as
// batchnorm_kernels.cl:57-59) and the constants of the normalize pass.
// Sum of the partials of channel c over all row blocks, in a fixed order: the
// partials are stored channel-major, thread t adds blocks t, t + kFinThreads,
// ... in order (coalesced across the CTA), each warp folds its 32 sums with a
// fixed xor butterfly, and thread 0 adds the warp sums in warp order.  One
// CTA of kFinThreads per channel.
constexpr int kFinThreads = 128;
__device__ __forceinline__ float2 sum_partials(const float2* __restrict__ partial, int blocks, int C, int c) {
  __shared__ float2 s_warp[kFinThreads / 32];
  const float2* pc = partial + (int64_t)c * blocks;
  float a = 0.0f, b = 0.0f;
#pragma unroll 4
  for (int i = threadIdx.x; i < blocks; i += kFinThreads) {
    const float2 p = pc[i];
    a += p.x;
    b += p.y;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  if ((threadIdx.x & 31) == 0) s_warp[threadIdx.x >> 5] = make_float2(a, b);
  __syncthreads();
  float2 r = s_warp[0];
#pragma unroll
  for (int w = 1; w < kFinThreads / 32; ++w) {
    r.x += s_warp[w].x;
    r.y += s_warp[w].y;
  }
  return r;
}

// Stage 2 of the statistics: mean = sum / NHW, var = sum_sq / NHW - mean^2
// (the reference's formula), inv_std = 1 / sqrt(var + eps).
// With moving_mean != nullptr also the layer's moving-average update (as
// bn_moving_update_kernel: momentum * moving + one_minus_momentum * batch,
// each product and the sum rounded to fp32).
__global__ void __launch_bounds__(kFinThreads) bn_stats_finalize_kernel(
    const float2* __restrict__ partial, int blocks, int C, int64_t nhw, float eps, float* __restrict__ mean,
    float* __restrict__ var, float* __restrict__ inv_std, float* __restrict__ moving_mean = nullptr,
    float* __restrict__ moving_var = nullptr, float momentum = 0.0f, float one_minus_momentum = 0.0f) {
  const int c = blockIdx.x;
  const float2 s = sum_partials(partial, blocks, C, c);
  if (threadIdx.x == 0) {
    const float n = (float)(int)nhw;  // the reference divides by (float)(int)NHW
    const float m = __fdiv_rn(s.x, n);
    const float v = __fsub_rn(__fdiv_rn(s.y, n), __fmul_rn(m, m));
    mean[c] = m;
    var[c] = v;
    inv_std[c] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(v, eps)));
    if (moving_mean) {
      moving_mean[c] = __fadd_rn(__fmul_rn(momentum, moving_mean[c]), __fmul_rn(one_minus_momentum, m));
      moving_var[c] = __fadd_rn(__fmul_rn(momentum, moving_var[c]), __fmul_rn(one_minus_momentum, v));
    }
  }
}

__global__ void bn_moving_update_kernel(float* __restrict__ mm, float* __restrict__ mv,
                                        const float* __restrict__ bm, const float* __restrict__ bv, int C,
                                        float momentum, float one_minus_momentum) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  mm[c] = __fadd_rn(__fmul_rn(momentum, mm[c]), __fmul_rn(one_minus_momentum, bm[c]));
  mv[c] = __fadd_rn(__fmul_rn(momentum, mv[c]), __fmul_rn(one_minus_momentum, bv[c]));
}

// inv_std for the inference op (batchnorm_kernels.cl:78).
__global__ void bn_inv_std_kernel(const float* __restrict__ var, int C, float eps, float* __restrict__ inv_std) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c < C) inv_std[c] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var[c], eps)));
}

// Elementwise passes are row-tiled like the reductions: thread
// (cg_local, r_off) of CTA (row block, channel chunk) owns channels
// c0 .. c0+VEC-1 and every rpi-th row of its share, so its per-channel
// constants sit in registers and each row costs one vector load per input and
// one vector store, four rows in flight per thread.  The rows are split into
// the same `ranges` as the preceding reduction pass (gridDim.x = ranges * S,
// S CTAs interleaved on a range) and walked from the end of each range
// backwards: the reduction walked its ranges forwards, so the rows it read
// last, still in L2, are read first.
struct RowTile {
  int c0;
  int64_t r, first, step;  // rows r, r - step, ... >= first
  bool active;
};

__device__ __forceinline__ RowTile row_tile(int64_t rows, const ChunkGeom& geo, int ranges) {
  RowTile rt;
  const int t = threadIdx.x;
  const int cg_local = t % geo.cg;
  const int r_off = t / geo.cg;
  const int group = blockIdx.y * geo.cg + cg_local;
  rt.active = r_off < geo.rpi && group < geo.groups;
  rt.c0 = group * geo.vec;
  const int S = gridDim.x / ranges;
  const int range = blockIdx.x / S, sub = blockIdx.x % S;
  const int64_t per_range = ceil_div(rows, ranges);
  const int64_t r_begin = (int64_t)range * per_range;
  const int64_t r_end = r_begin + per_range < rows ? r_begin + per_range : rows;
  rt.step = (int64_t)geo.rpi * S;
  rt.first = r_begin + r_off + (int64_t)sub * geo.rpi;
  rt.r = rt.first < r_end ? rt.first + (r_end - 1 - rt.first) / rt.step * rt.step : rt.first - rt.step;
  return rt;
}

// y = gamma * ((x - mean) * inv_std) + beta (batchnorm_kernels.cl:77-80);
// RELU: the reference's relu applied to y in the same pass (y > 0 ? y : 0).
template <int VEC, bool RELU>
__global__ void __launch_bounds__(kThreads)
    bn_normalize_kernel(const float* __restrict__ x, const float* __restrict__ mean,
                        const float* __restrict__ inv_std, const float* __restrict__ gamma,
                        const float* __restrict__ beta, float* __restrict__ y, int64_t rows, int C, ChunkGeom geo,
                        int ranges) {
  using V = typename VecT<VEC>::T;
  RowTile rt = row_tile(rows, geo, ranges);
  if (!rt.active) return;
  float m[VEC], iv[VEC], g[VEC], b[VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    m[j] = mean[rt.c0 + j];
    iv[j] = inv_std[rt.c0 + j];
    g[j] = gamma[rt.c0 + j];
    b[j] = beta[rt.c0 + j];
  }
  auto one = [&](const float* v, float* o) {
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float yv = bn_y(v[j], m[j], iv[j], g[j], b[j]);
      o[j] = RELU ? (yv > 0.0f ? yv : 0.0f) : yv;
    }
  };
  constexpr int U = 4;
  for (; rt.r - (U - 1) * rt.step >= rt.first; rt.r -= U * rt.step) {
    float v[U][VEC], o[U][VEC];
#pragma unroll
    for (int u = 0; u < U; ++u) VecT<VEC>::to(*reinterpret_cast<const V*>(x + (rt.r - u * rt.step) * C + rt.c0), v[u]);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      one(v[u], o[u]);
      VecT<VEC>::from(o[u], reinterpret_cast<V*>(y + (rt.r - u * rt.step) * C + rt.c0));
    }
  }
  for (; rt.r >= rt.first; rt.r -= rt.step) {
    float v[VEC], o[VEC];
    VecT<VEC>::to(*reinterpret_cast<const V*>(x + rt.r * C + rt.c0), v);
    one(v, o);
    VecT<VEC>::from(o, reinterpret_cast<V*>(y + rt.r * C + rt.c0));
  }
}

// Stage 2 of the gradient: grad_beta = sum dy, grad_gamma = sum dy * x_hat;
// also k1 = gamma * inv_std / NHW and inv_std for the dx pass.
__global__ void __launch_bounds__(kFinThreads) bn_grad_finalize_kernel(
    const float2* __restrict__ partial, int blocks, int C, int64_t nhw, float eps, const float* __restrict__ gamma,
    const float* __restrict__ var, float* __restrict__ grad_beta, float* __restrict__ grad_gamma,
    float* __restrict__ k1, float* __restrict__ inv_std) {
  const int c = blockIdx.x;
  const float2 s = sum_partials(partial, blocks, C, c);
  if (threadIdx.x == 0) {
    grad_beta[c] = s.x;
    grad_gamma[c] = s.y;
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var[c], eps)));
    const float n = (float)(int)nhw;
    inv_std[c] = inv;
    k1[c] = __fdiv_rn(__fmul_rn(gamma[c], inv), n);
  }
}

// dx = k1 * (NHW*dy - grad_beta - x_hat*grad_gamma) (batchnorm_kernels.cl:135-142);
// RELU: dy = (y > 0 ? dz : 0) through a ReLU on the BN output, y recomputed.
template <int VEC, bool RELU>
__global__ void __launch_bounds__(kThreads)
    bn_grad_dx_kernel(const float* __restrict__ dy, const float* __restrict__ x, const float* __restrict__ mean,
                      const float* __restrict__ inv_std, const float* __restrict__ k1,
                      const float* __restrict__ grad_beta, const float* __restrict__ grad_gamma,
                      float* __restrict__ dx, int64_t rows, int C, float nhw_f, ChunkGeom geo, int ranges,
                      const float* __restrict__ gamma = nullptr, const float* __restrict__ beta = nullptr) {
  using V = typename VecT<VEC>::T;
  RowTile rt = row_tile(rows, geo, ranges);
  if (!rt.active) return;
  float m[VEC], iv[VEC], kk[VEC], db[VEC], dg[VEC], gm[VEC], bt[VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    m[j] = mean[rt.c0 + j];
    iv[j] = inv_std[rt.c0 + j];
    kk[j] = k1[rt.c0 + j];
    db[j] = grad_beta[rt.c0 + j];
    dg[j] = grad_gamma[rt.c0 + j];
    gm[j] = RELU ? gamma[rt.c0 + j] : 0.0f;
    bt[j] = RELU ? beta[rt.c0 + j] : 0.0f;
  }
  auto one = [&](const float* vx, const float* vgz, float* o) {
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float xh = __fmul_rn(__fsub_rn(vx[j], m[j]), iv[j]);
      const float gv = RELU && !(__fadd_rn(__fmul_rn(gm[j], xh), bt[j]) > 0.0f) ? 0.0f : vgz[j];
      float t = __fmul_rn(nhw_f, gv);
      t = __fsub_rn(t, db[j]);
      t = __fsub_rn(t, __fmul_rn(xh, dg[j]));
      o[j] = __fmul_rn(kk[j], t);
    }
  };
  constexpr int U = 4;
  for (; rt.r - (U - 1) * rt.step >= rt.first; rt.r -= U * rt.step) {
    float vx[U][VEC], vg[U][VEC], o[VEC];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t off = (rt.r - u * rt.step) * C + rt.c0;
      VecT<VEC>::to(*reinterpret_cast<const V*>(x + off), vx[u]);
      VecT<VEC>::to(*reinterpret_cast<const V*>(dy + off), vg[u]);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      one(vx[u], vg[u], o);
      VecT<VEC>::from(o, reinterpret_cast<V*>(dx + (rt.r - u * rt.step) * C + rt.c0));
    }
  }
  for (; rt.r >= rt.first; rt.r -= rt.step) {
    float vx[VEC], vg[VEC], o[VEC];
    const int64_t off = rt.r * C + rt.c0;
    VecT<VEC>::to(*reinterpret_cast<const V*>(x + off), vx);
    VecT<VEC>::to(*reinterpret_cast<const V*>(dy + off), vg);
    one(vx, vg, o);
    VecT<VEC>::from(o, reinterpret_cast<V*>(dx + off));
  }
}

// CTAs for an elementwise row-tiled pass: about 8 per SM, at least 4 rows per
// thread.
int ew_row_blocks(int64_t rows, const ChunkGeom& geo, int sm_count) {
  int64_t want = (int64_t)sm_count * 8 / geo.chunks;
  if (want < 1) want = 1;
  int64_t cap = ceil_div(rows, (int64_t)geo.rpi * 4);
  if (cap < 1) cap = 1;
  return (int)(want < cap ? want : cap);
}

// Row CTAs of an elementwise pass that follows a reduction over `ranges` row
// blocks (0: none): `ranges` times the CTAs per range that keep about 8 CTAs
// per SM.  Sets *ranges_out to the ranges the kernel splits the rows into.
int ew_grid_x(int64_t rows, const ChunkGeom& geo, int sm_count, int ranges, int* ranges_out) {
  const int ew = ew_row_blocks(rows, geo, sm_count);
  if (ranges <= 0) {
    *ranges_out = ew;
    return ew;
  }
  const int per = ew / ranges > 1 ? ew / ranges : 1;
  *ranges_out = ranges;
  return ranges * per;
}

int validate_nhwc(const int64_t* s, const char* what) {
  B2_REQUIRE(s != nullptr, "%s shape missing", what);
  for (int i = 0; i < 4; ++i) B2_REQUIRE(s[i] >= 0, "%s must be NHWC with non-negative dims", what);
  B2_REQUIRE(s[0] * s[1] * s[2] * s[3] <= kMaxInt32 * 4, "%s is too large", what);
  return B2_OK;
}

// mode 0: statistics, 1: gradient, 2: gradient through a ReLU on the output
// (gamma, beta used to recompute the mask).
template <int VEC>
void partials_vec(dim3 grid, cudaStream_t s, int mode, const float* x, const float* dy, const float* mean,
                  const float* var, float eps, int64_t rows, int C, const ChunkGeom& geo, float2* partial,
                  const float* gamma, const float* beta) {
  if (mode == 0)
    bn_partial_kernel<VEC, 0><<<grid, kThreads, 0, s>>>(x, dy, mean, var, eps, rows, C, geo, partial);
  else if (mode == 1)
    bn_partial_kernel<VEC, 1><<<grid, kThreads, 0, s>>>(x, dy, mean, var, eps, rows, C, geo, partial);
  else
    bn_partial_kernel<VEC, 2><<<grid, kThreads, 0, s>>>(x, dy, mean, var, eps, rows, C, geo, partial, gamma, beta);
}

int launch_partials(cudaStream_t s, int mode, const float* x, const float* dy, const float* mean,
                    const float* var, float eps, int64_t rows, int C, bool vec_ok, const DeviceInfo* d,
                    float2* partial, int* blocks_out, const float* gamma = nullptr, const float* beta = nullptr) {
  const ChunkGeom geo = chunk_geom(C, vec_ok);
  const int blocks = row_blocks(rows, geo.chunks, d->sm_count);
  dim3 grid(blocks, geo.chunks);
  if (geo.vec == 4) partials_vec<4>(grid, s, mode, x, dy, mean, var, eps, rows, C, geo, partial, gamma, beta);
  else partials_vec<1>(grid, s, mode, x, dy, mean, var, eps, rows, C, geo, partial, gamma, beta);
  *blocks_out = blocks;
  return check_launch(s, mode == 0 ? "bn_reduce_stats" : "bn_backward_reduce");
}

int launch_normalize(cudaStream_t s, const float* x, const float* mean, const float* inv, const float* gamma,
                     const float* beta, float* y, int64_t total, int C, bool vec_ok, bool relu = false,
                     int ranges = 0) {
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  const ChunkGeom geo = chunk_geom(C, vec_ok);
  const int64_t rows = total / C;
  int rg = 0;
  dim3 grid(ew_grid_x(rows, geo, d->sm_count, ranges, &rg), geo.chunks);
  if (vec_ok) {
    if (relu) bn_normalize_kernel<4, true><<<grid, kThreads, 0, s>>>(x, mean, inv, gamma, beta, y, rows, C, geo, rg);
    else bn_normalize_kernel<4, false><<<grid, kThreads, 0, s>>>(x, mean, inv, gamma, beta, y, rows, C, geo, rg);
  } else {
    if (relu) bn_normalize_kernel<1, true><<<grid, kThreads, 0, s>>>(x, mean, inv, gamma, beta, y, rows, C, geo, rg);
    else bn_normalize_kernel<1, false><<<grid, kThreads, 0, s>>>(x, mean, inv, gamma, beta, y, rows, C, geo, rg);
  }
  return check_launch(s, "bn_normalize");
}

// Training forward: statistics, then y = BN(x) (relu: y = relu(BN(x))).
int bn_training(cudaStream_t s, const float* x, const int64_t* x_shape, const float* gamma, int64_t gamma_len,
                const float* beta, int64_t beta_len, float epsilon, float* y, float* saved_mean, float* saved_var,
                bool relu, float* moving_mean = nullptr, float* moving_var = nullptr, float momentum = 0.0f,
                float one_minus_momentum = 0.0f) {
  B2_RETURN_IF_ERROR(validate_nhwc(x_shape, "x"));
  const int64_t C = x_shape[3];
  B2_REQUIRE(gamma_len == C && beta_len == C, "gamma/beta size must equal channels");
  const int64_t rows = x_shape[0] * x_shape[1] * x_shape[2];
  const int64_t total = rows * C;
  if (C == 0) return B2_OK;
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  const bool vec_ok = (C % 4 == 0) && aligned16(x) && aligned16(y);
  const ChunkGeom geo = chunk_geom(C, vec_ok);
  const int blocks = row_blocks(rows, geo.chunks, d->sm_count);
  Scratch part, inv;
  B2_RETURN_IF_ERROR(part.alloc(sizeof(float2) * blocks * C, s));
  B2_RETURN_IF_ERROR(inv.alloc(sizeof(float) * C, s));
  int used_blocks = 0;
  B2_RETURN_IF_ERROR(launch_partials(s, 0, x, nullptr, nullptr, nullptr, epsilon, rows, (int)C, vec_ok, d,
                                     part.as<float2>(), &used_blocks));
  bn_stats_finalize_kernel<<<(unsigned)C, kFinThreads, 0, s>>>(part.as<float2>(), used_blocks, (int)C, rows,
                                                                epsilon, saved_mean, saved_var, inv.as<float>(),
                                                                moving_mean, moving_var, momentum, one_minus_momentum);
  B2_RETURN_IF_ERROR(check_launch(s, "bn_stats_finalize"));
  if (total == 0) return B2_OK;
  return launch_normalize(s, x, saved_mean, inv.as<float>(), gamma, beta, y, total, (int)C, vec_ok, relu,
                          used_blocks);
}

// Backward: dx, dgamma, dbeta from dy (relu: dy = (y > 0 ? dz : 0) with y
// recomputed from x, the statistics, gamma and beta).
int bn_grad(cudaStream_t s, const float* grad_y, const int64_t* grad_y_shape, const float* x,
            const int64_t* x_shape, const float* gamma, const float* beta, const float* saved_mean,
            const float* saved_var, float epsilon, float* grad_x, float* grad_gamma, float* grad_beta, bool relu) {
  B2_RETURN_IF_ERROR(validate_nhwc(x_shape, "x"));
  bool same_shape = grad_y_shape != nullptr;
  for (int i = 0; same_shape && i < 4; ++i) same_shape = grad_y_shape[i] == x_shape[i];
  B2_REQUIRE(same_shape, "grad_y and x must have matching NHWC shapes");
  const int64_t C = x_shape[3];
  const int64_t rows = x_shape[0] * x_shape[1] * x_shape[2];
  const int64_t total = rows * C;
  if (C == 0) return B2_OK;
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  const bool vec_ok = (C % 4 == 0) && aligned16(x) && aligned16(grad_y) && aligned16(grad_x);
  const ChunkGeom geo = chunk_geom(C, vec_ok);
  const int blocks = row_blocks(rows, geo.chunks, d->sm_count);
  Scratch part, chan;
  B2_RETURN_IF_ERROR(part.alloc(sizeof(float2) * blocks * C, s));
  B2_RETURN_IF_ERROR(chan.alloc(sizeof(float) * 2 * C, s));
  float* k1 = chan.as<float>();
  float* inv = k1 + C;
  int used_blocks = 0;
  B2_RETURN_IF_ERROR(launch_partials(s, relu ? 2 : 1, x, grad_y, saved_mean, saved_var, epsilon, rows, (int)C,
                                     vec_ok, d, part.as<float2>(), &used_blocks, gamma, beta));
  bn_grad_finalize_kernel<<<(unsigned)C, kFinThreads, 0, s>>>(part.as<float2>(), used_blocks, (int)C, rows,
                                                               epsilon, gamma, saved_var, grad_beta, grad_gamma, k1,
                                                               inv);
  B2_RETURN_IF_ERROR(check_launch(s, "bn_grad_finalize"));
  if (total == 0) return B2_OK;
  const float nhw_f = (float)(int)rows;
  int rg = 0;
  dim3 egrid(ew_grid_x(rows, geo, d->sm_count, used_blocks, &rg), geo.chunks);
  if (vec_ok) {
    if (relu)
      bn_grad_dx_kernel<4, true><<<egrid, kThreads, 0, s>>>(grad_y, x, saved_mean, inv, k1, grad_beta, grad_gamma,
                                                           grad_x, rows, (int)C, nhw_f, geo, rg, gamma, beta);
    else
      bn_grad_dx_kernel<4, false><<<egrid, kThreads, 0, s>>>(grad_y, x, saved_mean, inv, k1, grad_beta, grad_gamma,
                                                            grad_x, rows, (int)C, nhw_f, geo, rg);
  } else {
    if (relu)
      bn_grad_dx_kernel<1, true><<<egrid, kThreads, 0, s>>>(grad_y, x, saved_mean, inv, k1, grad_beta, grad_gamma,
                                                           grad_x, rows, (int)C, nhw_f, geo, rg, gamma, beta);
    else
      bn_grad_dx_kernel<1, false><<<egrid, kThreads, 0, s>>>(grad_y, x, saved_mean, inv, k1, grad_beta, grad_gamma,
                                                            grad_x, rows, (int)C, nhw_f, geo, rg);
  }
  return check_launch(s, "bn_backward_dx");
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" {

// src/ops/batchnorm_ops.cc:87-180
int b2_batch_norm_training(b2_stream_t stream, const float* x, const int64_t x_shape[4], const float* gamma,
                           int64_t gamma_len, const float* beta, int64_t beta_len, float epsilon, float* y,
                           float* saved_mean, float* saved_var) {
  clear_error();
  return bn_training(static_cast<cudaStream_t>(stream), x, x_shape, gamma, gamma_len, beta, beta_len, epsilon, y,
                     saved_mean, saved_var, false);
}

// OpenclBatchNormTraining followed by OpenclRelu (src/ops/batchnorm_ops.cc:87-180,
// src/ops/relu_ops.cc), one pass over x less and no intermediate tensor.
int b2_batch_norm_relu_training(b2_stream_t stream, const float* x, const int64_t x_shape[4], const float* gamma,
                                int64_t gamma_len, const float* beta, int64_t beta_len, float epsilon, float* z,
                                float* saved_mean, float* saved_var, float* moving_mean, float* moving_var,
                                float momentum, float one_minus_momentum) {
  clear_error();
  B2_REQUIRE((moving_mean == nullptr) == (moving_var == nullptr), "moving_mean and moving_var go together");
  return bn_training(static_cast<cudaStream_t>(stream), x, x_shape, gamma, gamma_len, beta, beta_len, epsilon, z,
                     saved_mean, saved_var, true, moving_mean, moving_var, momentum, one_minus_momentum);
}

// src/ops/batchnorm_ops.cc:213-275
int b2_batch_norm_inference(b2_stream_t stream, const float* x, const int64_t x_shape[4], const float* gamma,
                            int64_t gamma_len, const float* beta, int64_t beta_len, const float* mean,
                            int64_t mean_len, const float* var, int64_t var_len, float epsilon, float* y) {
  clear_error();
  B2_RETURN_IF_ERROR(validate_nhwc(x_shape, "x"));
  const int64_t C = x_shape[3];
  B2_REQUIRE(gamma_len == C && beta_len == C && mean_len == C && var_len == C,
             "gamma/beta/mean/var must have C elements");
  const int64_t total = x_shape[0] * x_shape[1] * x_shape[2] * C;
  if (total == 0) return B2_OK;
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Scratch inv;
  B2_RETURN_IF_ERROR(inv.alloc(sizeof(float) * C, s));
  bn_inv_std_kernel<<<(int)ceil_div(C, 256), 256, 0, s>>>(var, (int)C, epsilon, inv.as<float>());
  B2_RETURN_IF_ERROR(check_launch(s, "bn_inv_std"));
  const bool vec_ok = (C % 4 == 0) && aligned16(x) && aligned16(y);
  return launch_normalize(s, x, mean, inv.as<float>(), gamma, beta, y, total, (int)C, vec_ok);
}

// src/ops/batchnorm_ops.cc:313-416
int b2_batch_norm_grad(b2_stream_t stream, const float* grad_y, const int64_t grad_y_shape[4], const float* x,
                       const int64_t x_shape[4], const float* gamma, const float* saved_mean,
                       const float* saved_var, float epsilon, float* grad_x, float* grad_gamma, float* grad_beta) {
  clear_error();
  return bn_grad(static_cast<cudaStream_t>(stream), grad_y, grad_y_shape, x, x_shape, gamma, nullptr, saved_mean,
                 saved_var, epsilon, grad_x, grad_gamma, grad_beta, false);
}

// OpenclReluGrad followed by OpenclBatchNormGrad (src/ops/relu_ops.cc,
// src/ops/batchnorm_ops.cc:313-416) for z = relu(BN(x)): the ReLU mask is
// recomputed from x, so neither y nor dy is stored.
int b2_batch_norm_relu_grad(b2_stream_t stream, const float* grad_z, const int64_t grad_z_shape[4], const float* x,
                            const int64_t x_shape[4], const float* gamma, const float* beta, const float* saved_mean,
                            const float* saved_var, float epsilon, float* grad_x, float* grad_gamma,
                            float* grad_beta) {
  clear_error();
  B2_REQUIRE(beta != nullptr && gamma != nullptr, "gamma and beta are required");
  return bn_grad(static_cast<cudaStream_t>(stream), grad_z, grad_z_shape, x, x_shape, gamma, beta, saved_mean,
                 saved_var, epsilon, grad_x, grad_gamma, grad_beta, true);
}

// opencl_tf/layers.py:189-194 (the Keras layer's moving statistics):
// moving = momentum * moving + (1 - momentum) * batch for mean and variance,
// each product and the sum rounded to fp32 as the reference's three tensor ops
// are.  One launch for both buffers.
int b2_batch_norm_update_moving(b2_stream_t stream, float* moving_mean, float* moving_var, const float* batch_mean,
                                const float* batch_var, int64_t channels, float momentum,
                                float one_minus_momentum) {
  clear_error();
  B2_REQUIRE(channels >= 0 && channels <= kMaxInt32, "channels must be in [0, 2^31)");
  if (channels == 0) return B2_OK;
  B2_REQUIRE(moving_mean && moving_var && batch_mean && batch_var, "null buffer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  bn_moving_update_kernel<<<(unsigned)ceil_div(channels, 256), 256, 0, s>>>(
      moving_mean, moving_var, batch_mean, batch_var, (int)channels, momentum, one_minus_momentum);
  return check_launch(s, "bn_update_moving");
}

}  // extern "C"

// ===========================================================================
// BatchNorm training forward that allocates nothing.
//
// Some callers cannot let a library allocate device memory during a call:
// runtimes whose memory manager owns all of HBM (a framework that reserves
// its arena at start-up and accounts for every byte), or latency-critical
// serving loops where an allocation's possible device-wide synchronisation
// and unbounded cost are not acceptable once the process is warm.  For them
// this variant keeps its reduction partials in a fixed array that is part of
// the library's device image instead of taking them from the pool.
//
// Limit: 256 KiB of scratch per GPU (kNoAllocScratch float2 entries), held by
// every device that loads the library until the process exits.  Inputs need
// at most kNoAllocMaxChannels channels; the row blocks of the reduction are
// capped so that blocks * C partials plus C per-channel constants fit.
// ===========================================================================

namespace {
constexpr int kNoAllocScratch = 32768;        // float2 entries = 256 KiB
constexpr int kNoAllocMaxChannels = 16384;
constexpr int kNoAllocMaxDevices = 64;
}  // namespace

// Device scratch of the allocation-free entry point.  In host code this name
// is only a handle for cudaGetSymbolAddress, never a device address.
static __device__ __align__(256) float2 g_bn_no_alloc_scratch[kNoAllocScratch];

namespace {
std::mutex g_no_alloc_mu;
std::atomic<void*> g_no_alloc_addr[kNoAllocMaxDevices];

// The array's device address on `dev` (the current device), looked up on the
// first call there.  Only a successful lookup is kept: a lookup that failed
// (for instance one attempted while a stream was being captured) is retried
// by the next call instead of failing every later call.
cudaError_t no_alloc_scratch(int dev, void** addr) {
  *addr = g_no_alloc_addr[dev].load(std::memory_order_acquire);
  if (*addr) return cudaSuccess;
  std::lock_guard<std::mutex> lock(g_no_alloc_mu);
  *addr = g_no_alloc_addr[dev].load(std::memory_order_relaxed);
  if (*addr) return cudaSuccess;
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_bn_no_alloc_scratch);
  if (e != cudaSuccess) {
    cudaGetLastError();  // not sticky: clear it so the next call can retry
    return e;
  }
  g_no_alloc_addr[dev].store(p, std::memory_order_release);
  *addr = p;
  return cudaSuccess;
}
}  // namespace

extern "C" int b2_batch_norm_training_no_alloc(b2_stream_t stream, const float* x, const int64_t x_shape[4],
                                               const float* gamma, int64_t gamma_len, const float* beta,
                                               int64_t beta_len, float epsilon, float* y, float* saved_mean,
                                               float* saved_var) {
  using namespace b2;
  clear_error();
  B2_RETURN_IF_ERROR(validate_nhwc(x_shape, "x"));
  const int64_t C = x_shape[3];
  B2_REQUIRE(gamma_len == C && beta_len == C, "gamma/beta size must equal channels");
  B2_REQUIRE(C <= kNoAllocMaxChannels,
             "b2_batch_norm_training_no_alloc supports at most %d channels (got %lld); "
             "use b2_batch_norm_training", kNoAllocMaxChannels, (long long)C);
  const int64_t rows = x_shape[0] * x_shape[1] * x_shape[2];
  const int64_t total = rows * C;
  if (C == 0) return B2_OK;
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  const int dev = d->device;
  B2_REQUIRE(dev < kNoAllocMaxDevices, "device ordinal %d out of range", dev);
  void* scratch = nullptr;
  const cudaError_t se = no_alloc_scratch(dev, &scratch);
  if (se != cudaSuccess)
    return set_error(B2_ERR_INTERNAL, "cudaGetSymbolAddress of the static scratch failed (cuda_err=%d: %s)",
                     (int)se, cudaGetErrorString(se));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec_ok = (C % 4 == 0) && aligned16(x) && aligned16(y);
  const ChunkGeom geo = chunk_geom(C, vec_ok);
  // Partials take blocks * C entries, the per-channel inv_std ceil(C/2) more.
  const int64_t fit = (kNoAllocScratch - ceil_div(C, 2)) / C;
  int blocks = row_blocks(rows, geo.chunks, d->sm_count);
  if (blocks > fit) blocks = (int)fit;
  float2* partial = static_cast<float2*>(scratch);
  float* inv = reinterpret_cast<float*>(partial + (int64_t)blocks * C);
  // Every scratch entry read below is written earlier in this call, so no
  // clearing is needed; the previous call's contents are simply overwritten.
  dim3 grid(blocks, geo.chunks);
  if (geo.vec == 4)
    bn_partial_kernel<4, 0><<<grid, kThreads, 0, s>>>(x, nullptr, nullptr, nullptr, epsilon, rows, (int)C, geo,
                                                        partial);
  else
    bn_partial_kernel<1, 0><<<grid, kThreads, 0, s>>>(x, nullptr, nullptr, nullptr, epsilon, rows, (int)C, geo,
                                                        partial);
  B2_RETURN_IF_ERROR(check_launch(s, "bn_reduce_stats (no alloc)"));
  bn_stats_finalize_kernel<<<(unsigned)C, kFinThreads, 0, s>>>(partial, blocks, (int)C, rows, epsilon,
                                                                       saved_mean, saved_var, inv);
  B2_RETURN_IF_ERROR(check_launch(s, "bn_stats_finalize (no alloc)"));
  if (total == 0) return B2_OK;
  return launch_normalize(s, x, saved_mean, inv, gamma, beta, y, total, (int)C, vec_ok);
}
