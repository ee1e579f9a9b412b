// conv_direct.cu -- Conv2D forward, input gradient and filter gradient for
// narrow filters (at most 32 input and 32 output channels, kH*kW*Ci*Co <=
// 4608 weights): the 3x3 refinement convolutions and the 1x1 single-channel
// heatmap convolution of the uwb_loc_v3 network, and the small shapes of the
// reference's tests.
//
// Reference: kernels/conv2d_kernels.cl:30-158, src/ops/conv2d_ops.cc.  With
// so few channels an implicit GEMM has N or K of 1..16: the tensor-core
// engines spend their time gathering and splitting operands for a handful of
// MMAs each.  These kernels run on the CUDA cores instead, with the filter in
// shared memory (read as broadcasts) and every input element loaded once per
// tap through L1:
//
//   forward      one thread per (output pixel, group of COT output channels),
//                COT accumulators, taps in the reference's (kh, kw, ci) order;
//   input grad   one thread per (input pixel, group of CIT input channels),
//                taps in the reference's (kh, kw, co) order with its
//                stride / bounds tests, the filter transposed to [kh][kw][co][ci]
//                in shared memory so a thread's CIT weights are contiguous;
//   filter grad  with channel counts divisible by 4, a CTA owns a range of
//                output rows and a thread one tap's 4 x 4 (ci, co) block of dW
//                (128-bit loads of x and dy, 16 FMAs per pixel); otherwise a
//                CTA owns a range of output pixels and a thread one
//                (kh, kw, ci) and COT output channels.  Several pixel lanes
//                per CTA when the filter is small; the lanes are added in a
//                fixed order into per-CTA partials, which
//                conv_direct_finalize_kernel adds in a fixed order.
//
// Forward and input gradient multiply and add with round-to-nearest in the
// reference's order, so they are bit-identical to its sequential fp32 sums;
// the filter gradient (fused multiply-adds, four pixels' loads in flight per
// thread) is deterministic, within fp32 rounding of the reference's single
// serial sum over N*Ho*Wo.
#include <type_traits>

#include "conv_common.cuh"

namespace b2 {
namespace {

constexpr int kFwdThreads = 128;
constexpr int kWgradThreads = 256;
constexpr int kWgradUnroll = 4;
constexpr int kMaxWeights = 4608;

struct DirectArgs {
  int N, H, W, Ci, kH, kW, Co, sH, sW, pH, pW, Ho, Wo;
};

__device__ __forceinline__ float mac(float acc, float a, float b) { return __fadd_rn(acc, __fmul_rn(a, b)); }

// acc[j] += xv * w[j], j < T, with w 16-byte aligned when T % 4 == 0.
template <int T>
__device__ __forceinline__ void mac_row(float (&acc)[T], float xv, const float* w) {
  if constexpr (T % 4 == 0) {
#pragma unroll
    for (int j = 0; j < T; j += 4) {
      const float4 q = *reinterpret_cast<const float4*>(w + j);
      acc[j] = mac(acc[j], xv, q.x);
      acc[j + 1] = mac(acc[j + 1], xv, q.y);
      acc[j + 2] = mac(acc[j + 2], xv, q.z);
      acc[j + 3] = mac(acc[j + 3], xv, q.w);
    }
  } else {
#pragma unroll
    for (int j = 0; j < T; ++j) acc[j] = mac(acc[j], xv, w[j]);
  }
}

template <int T>
__device__ __forceinline__ void store_row(float* out, const float (&acc)[T], bool vec) {
  if (T % 4 == 0 && vec) {
#pragma unroll
    for (int j = 0; j < T; j += 4)
      *reinterpret_cast<float4*>(out + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < T; ++j) out[j] = acc[j];
  }
}

// y[n,ho,wo,co] = sum over (kh, kw, ci) in order of x * w (conv2d_kernels.cl:30-70).
template <int COT>
__global__ void __launch_bounds__(kFwdThreads) conv_direct_fwd_kernel(const float* __restrict__ x,
                                                                      const float* __restrict__ w,
                                                                      float* __restrict__ y, DirectArgs a,
                                                                      int pixels, bool vec, bool vec_out) {
  extern __shared__ float4 smem_f4[];
  float* ws = reinterpret_cast<float*>(smem_f4);
  const int nw = a.kH * a.kW * a.Ci * a.Co;
  for (int i = threadIdx.x; i < nw; i += blockDim.x) ws[i] = __ldg(w + i);
  __syncthreads();
  const int p = blockIdx.x * kFwdThreads + threadIdx.x;
  if (p >= pixels) return;
  const int c0 = blockIdx.y * COT;
  const int wo = p % a.Wo;
  const int t = p / a.Wo;
  const int ho = t % a.Ho;
  const int n = t / a.Ho;
  const int hi0 = ho * a.sH - a.pH, wi0 = wo * a.sW - a.pW;
  float acc[COT];
#pragma unroll
  for (int j = 0; j < COT; ++j) acc[j] = 0.0f;
  for (int kh = 0; kh < a.kH; ++kh) {
    const int hi = hi0 + kh;
    if ((unsigned)hi >= (unsigned)a.H) continue;
    for (int kw = 0; kw < a.kW; ++kw) {
      const int wi = wi0 + kw;
      if ((unsigned)wi >= (unsigned)a.W) continue;
      const float* xp = x + ((int64_t)(n * a.H + hi) * a.W + wi) * a.Ci;
      const float* wp = ws + (kh * a.kW + kw) * a.Ci * a.Co + c0;
      if (vec) {  // Ci % 4 == 0, x 16-byte aligned
        for (int ci = 0; ci < a.Ci; ci += 4) {
          const float4 xv = __ldg(reinterpret_cast<const float4*>(xp + ci));
          mac_row<COT>(acc, xv.x, wp + ci * a.Co);
          mac_row<COT>(acc, xv.y, wp + (ci + 1) * a.Co);
          mac_row<COT>(acc, xv.z, wp + (ci + 2) * a.Co);
          mac_row<COT>(acc, xv.w, wp + (ci + 3) * a.Co);
        }
      } else {
        for (int ci = 0; ci < a.Ci; ++ci) mac_row<COT>(acc, __ldg(xp + ci), wp + ci * a.Co);
      }
    }
  }
  store_row<COT>(y + (int64_t)p * a.Co + c0, acc, vec_out);
}

// dx[n,hi,wi,ci] = sum over (kh, kw, co) in order of dy * w for the output
// pixels that tap (hi, wi) (conv2d_kernels.cl:73-120).
template <int CIT>
__global__ void __launch_bounds__(kFwdThreads) conv_direct_dgrad_kernel(const float* __restrict__ dy,
                                                                        const float* __restrict__ w,
                                                                        float* __restrict__ dx, DirectArgs a,
                                                                        int pixels, bool vec, bool vec_out) {
  extern __shared__ float4 smem_f4[];
  float* wt = reinterpret_cast<float*>(smem_f4);  // [kh][kw][co][ci]
  const int nw = a.kH * a.kW * a.Ci * a.Co;
  for (int i = threadIdx.x; i < nw; i += blockDim.x) {
    const int co = i % a.Co;
    const int r = i / a.Co;  // (kh*kW + kw)*Ci + ci
    const int ci = r % a.Ci;
    const int tap = r / a.Ci;
    wt[(tap * a.Co + co) * a.Ci + ci] = __ldg(w + i);
  }
  __syncthreads();
  const int p = blockIdx.x * kFwdThreads + threadIdx.x;
  if (p >= pixels) return;
  const int c0 = blockIdx.y * CIT;
  const int wi = p % a.W;
  const int t = p / a.W;
  const int hi = t % a.H;
  const int n = t / a.H;
  float acc[CIT];
#pragma unroll
  for (int j = 0; j < CIT; ++j) acc[j] = 0.0f;
  for (int kh = 0; kh < a.kH; ++kh) {
    const int ho_num = hi + a.pH - kh;
    if (ho_num < 0 || ho_num % a.sH != 0) continue;
    const int ho = ho_num / a.sH;
    if (ho >= a.Ho) continue;
    for (int kw = 0; kw < a.kW; ++kw) {
      const int wo_num = wi + a.pW - kw;
      if (wo_num < 0 || wo_num % a.sW != 0) continue;
      const int wo = wo_num / a.sW;
      if (wo >= a.Wo) continue;
      const float* gp = dy + ((int64_t)(n * a.Ho + ho) * a.Wo + wo) * a.Co;
      const float* wp = wt + (kh * a.kW + kw) * a.Co * a.Ci + c0;
      if (vec) {  // Co % 4 == 0, dy 16-byte aligned
        for (int co = 0; co < a.Co; co += 4) {
          const float4 gv = __ldg(reinterpret_cast<const float4*>(gp + co));
          mac_row<CIT>(acc, gv.x, wp + co * a.Ci);
          mac_row<CIT>(acc, gv.y, wp + (co + 1) * a.Ci);
          mac_row<CIT>(acc, gv.z, wp + (co + 2) * a.Ci);
          mac_row<CIT>(acc, gv.w, wp + (co + 3) * a.Ci);
        }
      } else {
        for (int co = 0; co < a.Co; ++co) mac_row<CIT>(acc, __ldg(gp + co), wp + co * a.Ci);
      }
    }
  }
  store_row<CIT>(dx + (int64_t)p * a.Ci + c0, acc, vec_out);
}

// Stage 1 of dw[kh,kw,ci,co] = sum over output pixels of x * dy
// (conv2d_kernels.cl:123-158).  Entry e = (kh, kw, ci) * groups + co group;
// CTA (b, c) covers entries [c * entries, (c + 1) * entries) of the pixel
// range [b * ppb, (b + 1) * ppb).  Thread (lane, e) walks pixels p0 + lane,
// p0 + lane + lanes, ...; the lanes' sums are added in lane order into
// partial[b][f].
template <int COT>
__global__ void __launch_bounds__(kWgradThreads) conv_direct_wgrad_kernel(const float* __restrict__ x,
                                                                          const float* __restrict__ dy,
                                                                          float* __restrict__ partial,
                                                                          DirectArgs a, int pixels, int ppb,
                                                                          int entries, int lanes, bool vec) {
  extern __shared__ float4 smem_f4[];
  float* red = reinterpret_cast<float*>(smem_f4);  // [lanes][entries][COT]
  const int groups = a.Co / COT;
  const int e = threadIdx.x % entries;
  const int lane = threadIdx.x / entries;
  const int eg = blockIdx.y * entries + e;  // entry of the whole filter
  const bool live = eg < a.kH * a.kW * a.Ci * groups;
  const int m = live ? eg / groups : 0;
  const int c0 = live ? (eg - m * groups) * COT : 0;
  const int ci = m % a.Ci;
  const int kw = (m / a.Ci) % a.kW;
  const int kh = m / (a.Ci * a.kW);
  float acc[COT];
#pragma unroll
  for (int j = 0; j < COT; ++j) acc[j] = 0.0f;
  const int p0 = blockIdx.x * ppb;
  const int p1 = min(p0 + ppb, pixels);
  int p = p0 + lane;
  if (live && lane < lanes && p < p1) {
    int wo = p % a.Wo;
    int t = p / a.Wo;
    int ho = t % a.Ho;
    int n = t / a.Ho;
    // kWgradUnroll pixels per pass: all their loads are issued before the
    // multiply-adds, which then run in pixel order.
    for (; p < p1; p += kWgradUnroll * lanes) {
      float xv[kWgradUnroll];
      float gv[kWgradUnroll][COT];
      bool ok[kWgradUnroll];
#pragma unroll
      for (int u = 0; u < kWgradUnroll; ++u) {
        const int pu = p + u * lanes;
        const int hi = ho * a.sH - a.pH + kh;
        const int wi = wo * a.sW - a.pW + kw;
        ok[u] = pu < p1 && (unsigned)hi < (unsigned)a.H && (unsigned)wi < (unsigned)a.W;
        xv[u] = 0.0f;
#pragma unroll
        for (int j = 0; j < COT; ++j) gv[u][j] = 0.0f;
        if (ok[u]) {
          xv[u] = __ldg(x + ((int64_t)(n * a.H + hi) * a.W + wi) * a.Ci + ci);
          const float* gp = dy + (int64_t)pu * a.Co + c0;
          if (COT % 4 == 0 && vec) {  // Co % 4 == 0, dy 16-byte aligned
#pragma unroll
            for (int j = 0; j < COT; j += 4) {
              const float4 g4 = __ldg(reinterpret_cast<const float4*>(gp + j));
              gv[u][j] = g4.x;
              gv[u][j + 1] = g4.y;
              gv[u][j + 2] = g4.z;
              gv[u][j + 3] = g4.w;
            }
          } else {
#pragma unroll
            for (int j = 0; j < COT; ++j) gv[u][j] = __ldg(gp + j);
          }
        }
        wo += lanes;  // advance (n, ho, wo) by `lanes` pixels
        while (wo >= a.Wo) {
          wo -= a.Wo;
          if (++ho == a.Ho) {
            ho = 0;
            ++n;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kWgradUnroll; ++u) {
        if (ok[u]) {
#pragma unroll
          for (int j = 0; j < COT; ++j) acc[j] = fmaf(xv[u], gv[u][j], acc[j]);
        }
      }
    }
  }
  if (lane < lanes) {
#pragma unroll
    for (int j = 0; j < COT; ++j) red[(lane * entries + e) * COT + j] = acc[j];
  }
  __syncthreads();
  if (live && lane == 0) {
    float* out = partial + (int64_t)blockIdx.x * a.kH * a.kW * a.Ci * a.Co + m * a.Co + c0;
#pragma unroll
    for (int j = 0; j < COT; ++j) {
      float s = red[e * COT + j];
      for (int l = 1; l < lanes; ++l) s += red[(l * entries + e) * COT + j];
      out[j] = s;
    }
  }
}

// Stage 1 of the filter gradient when Ci % 4 == 0 and Co % 4 == 0 (x and dy
// 16-byte aligned): a thread owns a 4 x 4 block (input-channel quad x
// output-channel quad) of one tap's dW and walks whole output rows, so a
// pixel costs one 128-bit load of x, one of dy and 16 fused multiply-adds,
// and the tap's bounds are resolved once per row.  Entry e = (tap, ci quad,
// co quad); CTA (b, c) covers entries [c * entries, (c + 1) * entries) of the
// rows [b * rpb, (b + 1) * rpb) (row = n * Ho + ho); lane l walks rows
// r0 + l, r0 + l + lanes, ...; the lanes' sums are added in lane order.
__global__ void __launch_bounds__(kWgradThreads) conv_direct_wgrad_quad_kernel(const float* __restrict__ x,
                                                                               const float* __restrict__ dy,
                                                                               float* __restrict__ partial,
                                                                               DirectArgs a, int rows, int rpb,
                                                                               int entries, int lanes) {
  extern __shared__ float4 smem_f4[];
  float* red = reinterpret_cast<float*>(smem_f4);  // [lanes][entries][16]
  const int cq = a.Co / 4, iq = a.Ci / 4;
  const int e = threadIdx.x % entries;
  const int lane = threadIdx.x / entries;
  const int eg = blockIdx.y * entries + e;
  const bool live = eg < a.kH * a.kW * iq * cq;
  const int co4 = live ? eg % cq : 0;
  const int r = live ? eg / cq : 0;
  const int ci4 = r % iq;
  const int tap = r / iq;
  const int kw = tap % a.kW, kh = tap / a.kW;
  float acc[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) acc[j] = 0.0f;
  // output columns whose tap column wi = wo*sW - pW + kw lies inside the image
  const int lo_num = a.pW - kw;
  const int wlo = lo_num > 0 ? (lo_num + a.sW - 1) / a.sW : 0;
  const int hi_num = a.W - 1 + a.pW - kw;
  const int whi = hi_num < 0 ? 0 : min(hi_num / a.sW + 1, a.Wo);
  const int r0 = blockIdx.x * rpb;
  const int r1 = min(r0 + rpb, rows);
  if (live && lane < lanes) {
    for (int row = r0 + lane; row < r1; row += lanes) {
      const int ho = row % a.Ho;
      const int n = row / a.Ho;
      const int hi = ho * a.sH - a.pH + kh;
      if ((unsigned)hi >= (unsigned)a.H) continue;
      const int64_t xrow = (int64_t)(n * a.H + hi) * a.W * a.Ci + ci4 * 4;
      const float* grow = dy + (int64_t)row * a.Wo * a.Co + co4 * 4;
      for (int wo = wlo; wo < whi; wo += 4) {
        float4 xv[4], gv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (wo + u < whi) {
            const int wi = (wo + u) * a.sW - a.pW + kw;
            xv[u] = __ldg(reinterpret_cast<const float4*>(x + xrow + (int64_t)wi * a.Ci));
            gv[u] = __ldg(reinterpret_cast<const float4*>(grow + (int64_t)(wo + u) * a.Co));
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (wo + u < whi) {
            const float xs[4] = {xv[u].x, xv[u].y, xv[u].z, xv[u].w};
            const float gs[4] = {gv[u].x, gv[u].y, gv[u].z, gv[u].w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
              for (int j = 0; j < 4; ++j) acc[i * 4 + j] = fmaf(xs[i], gs[j], acc[i * 4 + j]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) red[(lane * entries + e) * 16 + j] = acc[j];
  __syncthreads();
  if (live && lane == 0) {
    float* out = partial + (int64_t)blockIdx.x * a.kH * a.kW * a.Ci * a.Co;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float sum = red[e * 16 + i * 4 + j];
        for (int l = 1; l < lanes; ++l) sum += red[(l * entries + e) * 16 + i * 4 + j];
        out[(tap * a.Ci + ci4 * 4 + i) * a.Co + co4 * 4 + j] = sum;
      }
    }
  }
}

// Stage 2: dw[f] = sum over CTAs of partial[b][f]; part j adds CTAs j, j+32,
// ... in order, then the 32 part sums are added in part order.
constexpr int kFinParts = 32;
__global__ void __launch_bounds__(32 * kFinParts) conv_direct_finalize_kernel(const float* __restrict__ partial,
                                                                              int blocks, int F,
                                                                              float* __restrict__ dw) {
  __shared__ float s_part[kFinParts][32];
  const int f = blockIdx.x * 32 + threadIdx.x;
  const int part = threadIdx.y;
  float acc = 0.0f;
  if (f < F) {
    for (int b = part; b < blocks; b += kFinParts) acc += __ldg(partial + (int64_t)b * F + f);
  }
  s_part[part][threadIdx.x] = acc;
  __syncthreads();
  if (part == 0 && f < F) {
    float sum = s_part[0][threadIdx.x];
    for (int j = 1; j < kFinParts; ++j) sum += s_part[j][threadIdx.x];
    dw[f] = sum;
  }
}

DirectArgs to_direct(const ConvGeom& g) {
  return DirectArgs{(int)g.N, (int)g.H, (int)g.W, (int)g.Ci, (int)g.kH, (int)g.kW, (int)g.Co,
                    (int)g.sH, (int)g.sW, (int)g.pH, (int)g.pW, (int)g.Ho, (int)g.Wo};
}

// Largest power of two <= 16 that divides c.
int channel_tile(int64_t c) {
  int t = 16;
  while (t > 1 && c % t != 0) t >>= 1;
  return t;
}

template <class F>
int dispatch_tile(int t, F&& f) {
  switch (t) {
    case 16: return f(std::integral_constant<int, 16>{});
    case 8: return f(std::integral_constant<int, 8>{});
    case 4: return f(std::integral_constant<int, 4>{});
    case 2: return f(std::integral_constant<int, 2>{});
    default: return f(std::integral_constant<int, 1>{});
  }
}

}  // namespace

bool conv_direct_ok(const ConvGeom& g) {
  return g.Ci >= 1 && g.Co >= 1 && g.Ci <= 32 && g.Co <= 32 && g.kH >= 1 && g.kW >= 1 &&
         g.kH * g.kW * g.Ci * g.Co <= kMaxWeights;
}

int conv_direct_forward(const ConvGeom& g, const float* x, const float* w, float* y, cudaStream_t s) {
  const int64_t pixels = g.N * g.Ho * g.Wo;
  if (pixels == 0) return B2_OK;
  const DirectArgs a = to_direct(g);
  const int cot = channel_tile(g.Co);
  const size_t smem = sizeof(float) * (size_t)(g.kH * g.kW * g.Ci * g.Co);
  const bool vec = g.Ci % 4 == 0 && aligned16(x);
  const bool vec_out = g.Co % 4 == 0 && aligned16(y);
  const dim3 grid((unsigned)ceil_div(pixels, kFwdThreads), (unsigned)(g.Co / cot));
  dispatch_tile(cot, [&](auto t) {
    conv_direct_fwd_kernel<decltype(t)::value><<<grid, kFwdThreads, smem, s>>>(x, w, y, a, (int)pixels, vec,
                                                                               vec_out);
    return 0;
  });
  return check_launch(s, "conv2d_forward_direct");
}

int conv_direct_backprop_input(const ConvGeom& g, const float* dy, const float* w, float* dx, cudaStream_t s) {
  const int64_t pixels = g.N * g.H * g.W;
  if (pixels == 0) return B2_OK;
  const DirectArgs a = to_direct(g);
  const int cit = channel_tile(g.Ci);
  const size_t smem = sizeof(float) * (size_t)(g.kH * g.kW * g.Ci * g.Co);
  const bool vec = g.Co % 4 == 0 && aligned16(dy);
  const bool vec_out = g.Ci % 4 == 0 && aligned16(dx);
  const dim3 grid((unsigned)ceil_div(pixels, kFwdThreads), (unsigned)(g.Ci / cit));
  dispatch_tile(cit, [&](auto t) {
    conv_direct_dgrad_kernel<decltype(t)::value><<<grid, kFwdThreads, smem, s>>>(dy, w, dx, a, (int)pixels, vec,
                                                                                 vec_out);
    return 0;
  });
  return check_launch(s, "conv2d_backprop_input_direct");
}

int conv_direct_backprop_filter(const ConvGeom& g, const float* x, const float* dy, float* dw, cudaStream_t s) {
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  const int64_t F = g.kH * g.kW * g.Ci * g.Co;
  const int64_t pixels = g.N * g.Ho * g.Wo;
  if (pixels == 0) {
    B2_CUDA_OR_RETURN(cudaMemsetAsync(dw, 0, sizeof(float) * F, s));
    return B2_OK;
  }
  const DirectArgs a = to_direct(g);
  if (g.Ci % 4 == 0 && g.Co % 4 == 0 && aligned16(x) && aligned16(dy)) {
    const int64_t all_entries = g.kH * g.kW * (g.Ci / 4) * (g.Co / 4);
    const int64_t chunks = ceil_div(all_entries, kWgradThreads);
    const int64_t entries = ceil_div(all_entries, chunks);
    const int lanes = (int)(kWgradThreads / entries);
    const int threads = (int)(entries * lanes);
    const int64_t rows = g.N * g.Ho;
    const int per_sm = 1536 / threads;
    int64_t blocks = (int64_t)d->sm_count * (per_sm < 2 ? 2 : per_sm > 8 ? 8 : per_sm);
    if (blocks > rows) blocks = rows;
    const int64_t rpb = ceil_div(rows, blocks);
    blocks = ceil_div(rows, rpb);
    Scratch part;
    B2_RETURN_IF_ERROR(part.alloc(sizeof(float) * (size_t)(blocks * F), s));
    conv_direct_wgrad_quad_kernel<<<dim3((unsigned)blocks, (unsigned)chunks), threads, sizeof(float) * 16 * threads,
                                    s>>>(x, dy, part.as<float>(), a, (int)rows, (int)rpb, (int)entries, lanes);
    B2_RETURN_IF_ERROR(check_launch(s, "conv2d_backprop_filter_direct"));
    conv_direct_finalize_kernel<<<(unsigned)ceil_div(F, 32), dim3(32, kFinParts), 0, s>>>(part.as<float>(),
                                                                                           (int)blocks, (int)F, dw);
    return check_launch(s, "conv2d_backprop_filter_direct_finalize");
  }
  const int cot = channel_tile(g.Co);
  const int64_t all_entries = g.kH * g.kW * g.Ci * (g.Co / cot);
  const int64_t chunks = ceil_div(all_entries, kWgradThreads);  // CTAs per pixel range
  const int64_t entries = ceil_div(all_entries, chunks);
  const int lanes = (int)(kWgradThreads / entries);
  const int threads = (int)(entries * lanes);
  // about 1.5k resident threads per SM: 2..8 CTAs per SM
  const int per_sm = 1536 / threads;
  int64_t blocks = (int64_t)d->sm_count * (per_sm < 2 ? 2 : per_sm > 8 ? 8 : per_sm);
  const int64_t cap = ceil_div(pixels, 64);
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const int64_t ppb = ceil_div(pixels, blocks);
  blocks = ceil_div(pixels, ppb);
  Scratch part;
  B2_RETURN_IF_ERROR(part.alloc(sizeof(float) * (size_t)(blocks * F), s));
  const size_t smem = sizeof(float) * (size_t)threads * cot;
  dispatch_tile(cot, [&](auto t) {
    conv_direct_wgrad_kernel<decltype(t)::value><<<dim3((unsigned)blocks, (unsigned)chunks), threads, smem, s>>>(
        x, dy, part.as<float>(), a, (int)pixels, (int)ppb, (int)entries, lanes, g.Co % 4 == 0 && aligned16(dy));
    return 0;
  });
  B2_RETURN_IF_ERROR(check_launch(s, "conv2d_backprop_filter_direct"));
  conv_direct_finalize_kernel<<<(unsigned)ceil_div(F, 32), dim3(32, kFinParts), 0, s>>>(part.as<float>(), (int)blocks,
                                                                                         (int)F, dw);
  return check_launch(s, "conv2d_backprop_filter_direct_finalize");
}

}  // namespace b2
