// depthwise.cu -- DepthwiseConv2D forward, input gradient, filter gradient.
//
// Reference: kernels/depthwise_conv2d_kernels.cl, src/ops/
// depthwise_conv2d_ops.cc.  Output channel co = ci*dm + d sees only input
// channel ci.  These ops are HBM-bound (about 2*kH*kW flops per output), so
// the kernels are built around coalesced NHWC traffic.  Taps are always
// summed in the reference's (kh, kw[, d]) order with round-to-nearest
// multiply and add, so forward and input gradient are bit-identical to the
// reference's sequential fp32 sums.
//
//   forward, 3x3 stride 2, dm == 1, C % 4 == 0 (the README blocks):
//     dw_fwd_s2k3_kernel -- a thread computes two horizontally adjacent
//     outputs for 4 channels, loading the five input columns they share once,
//     with the filter held in registers;
//   forward, other dm == 1 / C % 4 == 0 shapes: one thread per (pixel, 4
//     channels) with 128-bit loads (dw_fwd_vec4_kernel); any other shape: one
//     thread per element (dw_fwd_scalar_kernel);
//   input gradient, 3x3 stride 2: dw_dgrad_s2k3_kernel -- column pairs that
//     share each dy load, filter in registers; other dm == 1 shapes: one CTA
//     per input row (dw_dgrad_rows_kernel); any shape: dw_dgrad_scalar_kernel;
//   filter gradient (a sum over N*Ho*Wo per filter element), deterministic in
//     two stages: per-CTA partials, then dw_wgrad_finalize_kernel adding them
//     in a fixed tree.  For dm == 1, C % 4 == 0 the partials come from
//     dw_wgrad_staged_kernel: a producer warp streams dy rows and zero-padded
//     input rows into a ring of shared-memory slots with 1-D bulk copies
//     (full / empty mbarriers, every wait bounded), consumer warps accumulate
//     all taps from shared memory; otherwise from the register-walking
//     dw_wgrad_partial_vec4_kernel / _scalar_kernel.
#include "conv_common.cuh"

namespace b2 {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float4 fadd4(float4 a, float4 b) {
  return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}
__device__ __forceinline__ float4 fmul4(float4 a, float4 b) {
  return make_float4(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y), __fmul_rn(a.z, b.z), __fmul_rn(a.w, b.w));
}

// x / s for x >= 0 and a small runtime stride s (1 and 2, the common cases,
// need no division); x % s likewise.
__device__ __forceinline__ int div_stride(int x, int s) { return s == 1 ? x : s == 2 ? (x >> 1) : x / s; }
__device__ __forceinline__ int mod_stride(int x, int s) { return s == 1 ? 0 : s == 2 ? (x & 1) : x % s; }

struct DwArgs {
  int N, H, W, C, kH, kW, dm, sH, sW, pH, pW, Ho, Wo;
};

DwArgs to_args(const ConvGeom& g) {
  DwArgs a;
  a.N = (int)g.N; a.H = (int)g.H; a.W = (int)g.W; a.C = (int)g.Ci;
  a.kH = (int)g.kH; a.kW = (int)g.kW; a.dm = (int)g.dm;
  a.sH = (int)g.sH; a.sW = (int)g.sW; a.pH = (int)g.pH; a.pW = (int)g.pW;
  a.Ho = (int)g.Ho; a.Wo = (int)g.Wo;
  return a;
}

// --------------------------------------------------------------- forward

// depthwise_conv2d_kernels.cl:16-56, dm == 1, 4 channels per thread.
__global__ void __launch_bounds__(kThreads) dw_fwd_vec4_kernel(const float* __restrict__ x,
                                                                const float* __restrict__ w, float* __restrict__ y,
                                                                DwArgs a) {
  const int cg = a.C >> 2;
  const int64_t total = (int64_t)a.N * a.Ho * a.Wo * cg;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t g = (int64_t)blockIdx.x * kThreads + threadIdx.x; g < total; g += stride) {
    uint32_t p = (uint32_t)g / (uint32_t)cg;  // element counts < 2^31 (checked on the host)
    const int c = (int)((uint32_t)g - p * (uint32_t)cg) * 4;
    uint32_t q = p / (uint32_t)a.Wo;
    const int wo = (int)(p - q * (uint32_t)a.Wo);
    const uint32_t n32 = q / (uint32_t)a.Ho;
    const int ho = (int)(q - n32 * (uint32_t)a.Ho);
    const int n = (int)n32;
    const int hi0 = ho * a.sH - a.pH, wi0 = wo * a.sW - a.pW;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int kh = 0; kh < a.kH; ++kh) {
      const int hi = hi0 + kh;
      if ((unsigned)hi >= (unsigned)a.H) continue;
      const float* xrow = x + ((int64_t)(n * a.H + hi) * a.W) * a.C + c;
      const float* wrow = w + (int64_t)(kh * a.kW) * a.C + c;
      for (int kw = 0; kw < a.kW; ++kw) {
        const int wi = wi0 + kw;
        if ((unsigned)wi >= (unsigned)a.W) continue;
        const float4 xv = __ldg(reinterpret_cast<const float4*>(xrow + (int64_t)wi * a.C));
        const float4 wv = __ldg(reinterpret_cast<const float4*>(wrow + (int64_t)kw * a.C));
        acc = fadd4(acc, fmul4(xv, wv));
      }
    }
    reinterpret_cast<float4*>(y)[g] = acc;
  }
}

// depthwise_conv2d_kernels.cl:16-56 for the 3x3, stride-2 case (dm == 1,
// C % 4 == 0): thread (x, y) of CTA (output-row band, channel chunk) produces
// output columns 2j and 2j + 1 of each row of the band for its 4 channels from
// the five input columns they share (15 loads instead of 18, all issued
// before the adds), the filter in registers; taps are added in the
// reference's (kh, kw) order with round-to-nearest multiply and add, out-of-
// image taps skipped.
__global__ void __launch_bounds__(kThreads) dw_fwd_s2k3_kernel(const float* __restrict__ x,
                                                                const float* __restrict__ w, float* __restrict__ y,
                                                                DwArgs a, int pairs, int rows_per_block) {
  const int c4 = blockIdx.y * blockDim.x + threadIdx.x;
  if (c4 >= (a.C >> 2)) return;
  const int C = a.C, c = 4 * c4;
  float4 wr[9];
#pragma unroll
  for (int k = 0; k < 9; ++k) wr[k] = __ldg(reinterpret_cast<const float4*>(w + k * C + c));
  const int rows = a.N * a.Ho;
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = r0 + rows_per_block < rows ? r0 + rows_per_block : rows;
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int r = r0; r < r1; ++r) {
    const int n = r / a.Ho, ho = r - n * a.Ho;
    const int hi0 = 2 * ho - a.pH;
    const float* ximg = x + (int64_t)n * a.H * a.W * C + c;
    float* yrow = y + (int64_t)r * a.Wo * C + c;
    for (int j = threadIdx.y; j < pairs; j += blockDim.y) {
      const int wi0 = 4 * j - a.pW;  // first input column of output 2j
      float4 v[3][5];
      bool okr[3], okc[5];
#pragma unroll
      for (int q = 0; q < 5; ++q) okc[q] = (unsigned)(wi0 + q) < (unsigned)a.W;
#pragma unroll
      for (int kh = 0; kh < 3; ++kh) {
        const int hi = hi0 + kh;
        okr[kh] = (unsigned)hi < (unsigned)a.H;
        const float* xr = ximg + (int64_t)hi * a.W * C;
#pragma unroll
        for (int q = 0; q < 5; ++q)
          v[kh][q] = okr[kh] && okc[q] ? __ldg(reinterpret_cast<const float4*>(xr + (int64_t)(wi0 + q) * C)) : z;
      }
      float4 a0 = z, a1 = z;
#pragma unroll
      for (int kh = 0; kh < 3; ++kh) {
        if (!okr[kh]) continue;
#pragma unroll
        for (int kw = 0; kw < 3; ++kw) {
          if (okc[kw]) a0 = fadd4(a0, fmul4(v[kh][kw], wr[kh * 3 + kw]));
          if (okc[kw + 2]) a1 = fadd4(a1, fmul4(v[kh][kw + 2], wr[kh * 3 + kw]));
        }
      }
      const int wo0 = 2 * j;
      if (wo0 < a.Wo) *reinterpret_cast<float4*>(yrow + (int64_t)wo0 * C) = a0;
      if (wo0 + 1 < a.Wo) *reinterpret_cast<float4*>(yrow + (int64_t)(wo0 + 1) * C) = a1;
    }
  }
}

// depthwise_conv2d_kernels.cl:16-56, any dm / C.
__global__ void __launch_bounds__(kThreads) dw_fwd_scalar_kernel(const float* __restrict__ x,
                                                                  const float* __restrict__ w,
                                                                  float* __restrict__ y, DwArgs a) {
  const int Co = a.C * a.dm;
  const int64_t total = (int64_t)a.N * a.Ho * a.Wo * Co;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t g = (int64_t)blockIdx.x * kThreads + threadIdx.x; g < total; g += stride) {
    const int co = (int)(g % Co);
    int64_t p = g / Co;
    const int wo = (int)(p % a.Wo);
    p /= a.Wo;
    const int ho = (int)(p % a.Ho);
    const int n = (int)(p / a.Ho);
    const int ci = co / a.dm, d = co % a.dm;
    float acc = 0.0f;
    for (int kh = 0; kh < a.kH; ++kh) {
      const int hi = ho * a.sH - a.pH + kh;
      if ((unsigned)hi >= (unsigned)a.H) continue;
      for (int kw = 0; kw < a.kW; ++kw) {
        const int wi = wo * a.sW - a.pW + kw;
        if ((unsigned)wi >= (unsigned)a.W) continue;
        acc = __fadd_rn(acc, __fmul_rn(__ldg(x + ((int64_t)(n * a.H + hi) * a.W + wi) * a.C + ci),
                                       __ldg(w + ((int64_t)(kh * a.kW + kw) * a.C + ci) * a.dm + d)));
      }
    }
    y[g] = acc;
  }
}

// ----------------------------------------------------------- input grad

// depthwise_conv2d_kernels.cl:59-104, dm == 1, 4 channels per thread: CTA =
// input row (n, hi); thread (x, y) = (channel group, input column lane).
__global__ void __launch_bounds__(kThreads) dw_dgrad_rows_kernel(const float* __restrict__ dy,
                                                                  const float* __restrict__ w,
                                                                  float* __restrict__ dx, DwArgs a) {
  const int cg = a.C >> 2;
  const int row = blockIdx.x;  // n * H + hi (< 2^31, checked on the host)
  const int n = row / a.H, hi = row - n * a.H;
  const float* gimg = dy + (int64_t)n * a.Ho * a.Wo * a.C;
  // Only taps with (hi + pH - kh) % sH == 0 reach this row: start at the
  // first such kh and step by the stride (ascending, as the reference).
  const int kh0 = mod_stride(hi + a.pH, a.sH);
  for (int wi = threadIdx.y; wi < a.W; wi += blockDim.y) {
    const int kw0 = mod_stride(wi + a.pW, a.sW);
    float* xp = dx + ((int64_t)row * a.W + wi) * a.C;
    for (int c4 = threadIdx.x; c4 < cg; c4 += blockDim.x) {
      const int c = 4 * c4;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int kh = kh0; kh < a.kH; kh += a.sH) {
        const int hn = hi + a.pH - kh;
        if (hn < 0) break;
        const int ho = div_stride(hn, a.sH);
        if (ho >= a.Ho) continue;
        const float* grow = gimg + (int64_t)ho * a.Wo * a.C + c;
        for (int kw = kw0; kw < a.kW; kw += a.sW) {
          const int wn = wi + a.pW - kw;
          if (wn < 0) break;
          const int wo = div_stride(wn, a.sW);
          if (wo >= a.Wo) continue;
          const float4 gv = __ldg(reinterpret_cast<const float4*>(grow + (int64_t)wo * a.C));
          const float4 wv = __ldg(reinterpret_cast<const float4*>(w + (int64_t)(kh * a.kW + kw) * a.C + c));
          acc = fadd4(acc, fmul4(gv, wv));
        }
      }
      *reinterpret_cast<float4*>(xp + c) = acc;
    }
  }
}

// depthwise_conv2d_kernels.cl:59-104 for the 3x3, stride-2 case (dm == 1,
// C % 4 == 0): thread (x, y) of CTA (row band, channel chunk) produces, for
// each input row of the band, the two input columns with wi + pW = 2j and
// 2j + 1 for its 4 channels.  Those columns are reached by kw = 0, 2 (dy
// columns j, j - 1) and kw = 1 (dy column j), so each dy element loaded
// serves both outputs, and the filter stays in registers.  Taps are added in
// the reference's (kh, kw) order with round-to-nearest multiply and add.
__global__ void __launch_bounds__(kThreads) dw_dgrad_s2k3_kernel(const float* __restrict__ dy,
                                                                  const float* __restrict__ w,
                                                                  float* __restrict__ dx, DwArgs a, int pairs,
                                                                  int rows_per_block) {
  const int c4 = blockIdx.y * blockDim.x + threadIdx.x;
  if (c4 >= (a.C >> 2)) return;
  const int C = a.C, c = 4 * c4;
  float4 wr[9];
#pragma unroll
  for (int k = 0; k < 9; ++k) wr[k] = __ldg(reinterpret_cast<const float4*>(w + k * C + c));
  const int rows = a.N * a.H;
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = r0 + rows_per_block < rows ? r0 + rows_per_block : rows;
  // One input row: taps of rows ho_t (kh ascending), filter rows W0, W1, W2
  // of those taps; nt = 1 or 2 valid row taps.
  auto row = [&](const float* gimg, float* xrow, int nt, int ho_a, int ho_b, const float4* wa, const float4* wb) {
    for (int j = threadIdx.y; j < pairs; j += blockDim.y) {
      const bool okj = j < a.Wo, okj1 = j >= 1 && j - 1 < a.Wo;
      const float* ra = gimg + (int64_t)ho_a * a.Wo * C;
      const float* rb = gimg + (int64_t)(nt > 1 ? ho_b : ho_a) * a.Wo * C;
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 ga = nt > 0 && okj ? __ldg(reinterpret_cast<const float4*>(ra + (int64_t)j * C)) : z;
      const float4 gb = nt > 0 && okj1 ? __ldg(reinterpret_cast<const float4*>(ra + (int64_t)(j - 1) * C)) : z;
      const float4 ga2 = nt > 1 && okj ? __ldg(reinterpret_cast<const float4*>(rb + (int64_t)j * C)) : z;
      const float4 gb2 = nt > 1 && okj1 ? __ldg(reinterpret_cast<const float4*>(rb + (int64_t)(j - 1) * C)) : z;
      float4 ae = z, ao = z;
      if (nt > 0) {
        if (okj) ae = fadd4(ae, fmul4(ga, wa[0]));    // kw = 0
        if (okj1) ae = fadd4(ae, fmul4(gb, wa[2]));   // kw = 2
        if (okj) ao = fadd4(ao, fmul4(ga, wa[1]));    // kw = 1
      }
      if (nt > 1) {
        if (okj) ae = fadd4(ae, fmul4(ga2, wb[0]));
        if (okj1) ae = fadd4(ae, fmul4(gb2, wb[2]));
        if (okj) ao = fadd4(ao, fmul4(ga2, wb[1]));
      }
      const int we = 2 * j - a.pW, wo = we + 1;
      if ((unsigned)we < (unsigned)a.W) *reinterpret_cast<float4*>(xrow + (int64_t)we * C) = ae;
      if ((unsigned)wo < (unsigned)a.W) *reinterpret_cast<float4*>(xrow + (int64_t)wo * C) = ao;
    }
  };
  for (int r = r0; r < r1; ++r) {
    const int n = r / a.H, hi = r - n * a.H;
    const int hn = hi + a.pH;
    const float* gimg = dy + (int64_t)n * a.Ho * a.Wo * C + c;
    float* xrow = dx + (int64_t)r * a.W * C + c;
    if (hn & 1) {  // kh = 1 only
      const int ho = hn >> 1;
      if (ho < a.Ho) row(gimg, xrow, 1, ho, 0, wr + 3, wr + 3);
      else row(gimg, xrow, 0, 0, 0, wr, wr);
    } else {       // kh = 0 (ho = hn/2), then kh = 2 (ho = hn/2 - 1)
      const int ho0 = hn >> 1, ho2 = ho0 - 1;
      const bool v0 = ho0 < a.Ho, v2 = ho2 >= 0 && ho2 < a.Ho;
      if (v0 && v2) row(gimg, xrow, 2, ho0, ho2, wr, wr + 6);
      else if (v0) row(gimg, xrow, 1, ho0, 0, wr, wr);
      else if (v2) row(gimg, xrow, 1, ho2, 0, wr + 6, wr + 6);
      else row(gimg, xrow, 0, 0, 0, wr, wr);
    }
  }
}

// depthwise_conv2d_kernels.cl:59-104, any dm / C.
__global__ void __launch_bounds__(kThreads) dw_dgrad_scalar_kernel(const float* __restrict__ dy,
                                                                    const float* __restrict__ w,
                                                                    float* __restrict__ dx, DwArgs a) {
  const int Co = a.C * a.dm;
  const int64_t total = (int64_t)a.N * a.H * a.W * a.C;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t g = (int64_t)blockIdx.x * kThreads + threadIdx.x; g < total; g += stride) {
    const int ci = (int)(g % a.C);
    int64_t p = g / a.C;
    const int wi = (int)(p % a.W);
    p /= a.W;
    const int hi = (int)(p % a.H);
    const int n = (int)(p / a.H);
    float acc = 0.0f;
    for (int kh = 0; kh < a.kH; ++kh) {
      const int hn = hi + a.pH - kh;
      if (hn < 0 || hn % a.sH != 0) continue;
      const int ho = hn / a.sH;
      if (ho >= a.Ho) continue;
      for (int kw = 0; kw < a.kW; ++kw) {
        const int wn = wi + a.pW - kw;
        if (wn < 0 || wn % a.sW != 0) continue;
        const int wo = wn / a.sW;
        if (wo >= a.Wo) continue;
        const float* gp = dy + ((int64_t)(n * a.Ho + ho) * a.Wo + wo) * Co + (int64_t)ci * a.dm;
        const float* wp = w + ((int64_t)(kh * a.kW + kw) * a.C + ci) * a.dm;
        for (int d = 0; d < a.dm; ++d) acc = __fadd_rn(acc, __fmul_rn(__ldg(gp + d), __ldg(wp + d)));
      }
    }
    dx[g] = acc;
  }
}

// ---------------------------------------------------------- filter grad

// Stage 1, dm == 1, C % 4 == 0, kH*kW <= KMAX: thread (channel group, pixel
// lane) accumulates all taps for 4 channels over its pixels; the CTA folds
// its pixel lanes per tap in a fixed order.  partial: [blocks][kH*kW*C].
template <int KMAX>
__global__ void __launch_bounds__(kThreads) dw_wgrad_partial_vec4_kernel(const float* __restrict__ x,
                                                                          const float* __restrict__ dy,
                                                                          float* __restrict__ partial, DwArgs a,
                                                                          int cg_per_cta, int64_t pix_per_block) {
  __shared__ float4 s_fold[kThreads];
  const int cg_total = a.C >> 2;
  const int lanes = kThreads / cg_per_cta;
  const int t = threadIdx.x;
  const int cgl = t % cg_per_cta;
  const int lane = t / cg_per_cta;
  const int cgi = blockIdx.y * cg_per_cta + cgl;
  const bool active = lane < lanes && cgi < cg_total;
  const int c = cgi * 4;
  const int taps = a.kH * a.kW;
  const int64_t pixels = (int64_t)a.N * a.Ho * a.Wo;
  const int64_t p_begin = (int64_t)blockIdx.x * pix_per_block;
  int64_t p_end = p_begin + pix_per_block;
  if (p_end > pixels) p_end = pixels;

  float4 acc[KMAX];
#pragma unroll
  for (int k = 0; k < KMAX; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);

  if (active) {
    int tdh[KMAX], tdw[KMAX];  // tap offsets, divided once per thread
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      tdh[k] = k / a.kW;
      tdw[k] = k - tdh[k] * a.kW;
    }
    for (int64_t p = p_begin + lane; p < p_end; p += lanes) {
      const uint32_t q = (uint32_t)p / (uint32_t)a.Wo;  // pixel counts < 2^31 (checked on the host)
      const int wo = (int)((uint32_t)p - q * (uint32_t)a.Wo);
      const uint32_t n32 = q / (uint32_t)a.Ho;
      const int ho = (int)(q - n32 * (uint32_t)a.Ho);
      const int n = (int)n32;
      const float4 gv = __ldg(reinterpret_cast<const float4*>(dy + p * a.C + c));
      const int hi0 = ho * a.sH - a.pH, wi0 = wo * a.sW - a.pW;
#pragma unroll
      for (int k = 0; k < KMAX; ++k) {
        if (k < taps) {
          const int hi = hi0 + tdh[k], wi = wi0 + tdw[k];
          if ((unsigned)hi < (unsigned)a.H && (unsigned)wi < (unsigned)a.W) {
            const float4 xv =
                __ldg(reinterpret_cast<const float4*>(x + ((int64_t)(n * a.H + hi) * a.W + wi) * a.C + c));
            acc[k].x = fmaf(xv.x, gv.x, acc[k].x);
            acc[k].y = fmaf(xv.y, gv.y, acc[k].y);
            acc[k].z = fmaf(xv.z, gv.z, acc[k].z);
            acc[k].w = fmaf(xv.w, gv.w, acc[k].w);
          }
        }
      }
    }
  }
  const int64_t out_base = (int64_t)blockIdx.x * taps * a.C;
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    if (k >= taps) break;
    __syncthreads();
    s_fold[t] = acc[k];
    __syncthreads();
    if (lane == 0 && cgi < cg_total) {
      float4 s = s_fold[cgl];
      for (int l = 1; l < lanes; ++l) {
        const float4 v = s_fold[l * cg_per_cta + cgl];
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
      *reinterpret_cast<float4*>(partial + out_base + (int64_t)k * a.C + c) = s;
    }
  }
}

// ------------------------------------------ staged filter gradient
//
// dm == 1, C % 4 == 0, kH*kW <= 9, 16-byte aligned, staged rows fit: CTA
// (output-row band, channel chunk) walks output rows r0 .. r1 (r = n*Ho + ho)
// through a ring of S shared-memory slots.  Thread 0 fills a slot with 1-D bulk
// copies (cp.async.bulk, completion on the slot's mbarrier): the dy row and the
// kH input rows the output row reads, each input row placed after padL zero
// pixels so every tap of every output column lands inside the slot; rows
// outside the image are flagged and their taps skipped.  Threads (x, y) =
// (channel group, output-column lane) accumulate all taps of their 4 channels
// from shared memory; the CTA folds its column lanes per tap in a fixed order
// (deterministic).  Every wait is bounded.

static __device__ unsigned int g_dw_timeouts = 0;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}

__device__ __forceinline__ void bar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool bar_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase of parity `parity`, at most limit_ns; an expiry is
// counted and set in the library's host-mapped expiry word (so the op calls
// that follow return B2_ERR_TIMEOUT).
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t parity, uint64_t limit_ns, unsigned int* expired) {
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  while (!bar_try_wait(b, parity)) {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > limit_ns) {
      atomicAdd(&g_dw_timeouts, 1u);
      if (expired) {
        *reinterpret_cast<volatile unsigned int*>(expired) = 1u;
        __threadfence_system();
      }
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void bulk_g2s(float* dst, const float* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

struct DwStage {
  int slots;       // S
  int padL;        // zero pixels staged before each input row
  int Wp;          // staged input row width (pixels)
  int slot_floats; // Wo*C + kH*Wp*C
  WaitParams wait; // limit of the pipeline waits, expiry word
};

constexpr int kStagedConsumers = 256;  // consumer threads of a staged CTA (one producer warp on top)

// Warp 0 produces (lane 0 issues the bulk copies of the next row into a slot
// once its EMPTY barrier shows every consumer warp is done with it); the other
// warps consume rows as their FULL barriers complete, without block-wide
// synchronisation, and arrive on EMPTY per warp.
template <int KMAX>
__global__ void __launch_bounds__(32 + kStagedConsumers) dw_wgrad_staged_kernel(const float* __restrict__ x,
                                                                               const float* __restrict__ dy,
                                                                               float* __restrict__ partial,
                                                                               DwArgs a, DwStage st, int cgx,
                                                                               int lanes_y, int rows_per_block) {
  extern __shared__ __align__(16) uint8_t dsm[];
  float* slots = reinterpret_cast<float*>(dsm);
  uint64_t* full = reinterpret_cast<uint64_t*>(dsm + (size_t)st.slots * st.slot_floats * 4);
  uint64_t* empty = full + st.slots;
  int* valid = reinterpret_cast<int*>(empty + st.slots);  // [S][kH]
  __shared__ float4 s_fold[kStagedConsumers];

  const int C = a.C, cg = C >> 2;
  const int tid = threadIdx.x;
  const int nthr = blockDim.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int ct = tid - 32;  // consumer index
  const int cgl = ct % cgx, ly = ct / cgx;
  const bool consumer = warp > 0 && ly < lanes_y;
  const bool active = consumer && cgl < cg;
  const int c = 4 * cgl;
  const int consumer_warps = (32 * ((cgx * lanes_y + 31) / 32)) / 32;
  const int taps = a.kH * a.kW;
  const int rows = a.N * a.Ho;
  const int r0 = blockIdx.x * rows_per_block;
  const int nr = (r0 + rows_per_block < rows ? r0 + rows_per_block : rows) - r0;
  const int dy_floats = a.Wo * C;

  // Zero the slots once (the padding pixels stay zero), make the generic
  // writes visible to the bulk copies, then set up the barriers.
  for (int i = tid; i < st.slots * st.slot_floats; i += nthr) slots[i] = 0.0f;
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (tid == 0) {
    for (int i = 0; i < st.slots; ++i) {
      bar_init(&full[i], 1);
      bar_init(&empty[i], consumer_warps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  float4 acc[KMAX];
#pragma unroll
  for (int k = 0; k < KMAX; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nr; ++i, ++issued) {
        const int sl = i % st.slots;
        if (i >= st.slots && !bar_wait(&empty[sl], (uint32_t)(i / st.slots - 1) & 1u, st.wait.limit_ns, st.wait.expired))
          break;
        const int r = r0 + i;
        const int n = r / a.Ho, ho = r - n * a.Ho;
        float* base = slots + (size_t)sl * st.slot_floats;
        uint32_t bytes = (uint32_t)dy_floats * 4u;
        for (int kh = 0; kh < a.kH; ++kh) {
          const int hi = ho * a.sH - a.pH + kh;
          const bool ok = (unsigned)hi < (unsigned)a.H;
          valid[sl * a.kH + kh] = ok;
          if (ok) bytes += (uint32_t)(a.W * C) * 4u;
        }
        bar_expect_tx(&full[sl], bytes);
        bulk_g2s(base, dy + (int64_t)r * dy_floats, (uint32_t)dy_floats * 4u, &full[sl]);
        for (int kh = 0; kh < a.kH; ++kh) {
          const int hi = ho * a.sH - a.pH + kh;
          if ((unsigned)hi < (unsigned)a.H)
            bulk_g2s(base + dy_floats + (kh * st.Wp + st.padL) * C, x + ((int64_t)(n * a.H + hi) * a.W) * C,
                     (uint32_t)(a.W * C) * 4u, &full[sl]);
        }
      }
      // let every issued copy land before the CTA can exit
      const int first = issued > st.slots ? issued - st.slots : 0;
      for (int i = first; i < issued; ++i)
        bar_wait(&full[i % st.slots], (uint32_t)(i / st.slots) & 1u, kDefaultWaitLimitNs, st.wait.expired);
    }
  } else if (ct < consumer_warps * 32) {
    for (int i = 0; i < nr; ++i) {
      const int sl = i % st.slots;
      if (!bar_wait(&full[sl], (uint32_t)(i / st.slots) & 1u, st.wait.limit_ns, st.wait.expired)) break;
      const float* base = slots + (size_t)sl * st.slot_floats;
      if (active && KMAX == 9 && a.kH == 3 && a.kW == 3) {
        // 3x3: tap offsets fixed at compile time, row validity read once per row
        const bool v0 = valid[sl * 3] != 0, v1 = valid[sl * 3 + 1] != 0, v2 = valid[sl * 3 + 2] != 0;
        const int rs = st.Wp * C, ps = a.sW * C;
        const float* xrow = base + dy_floats + c;
        for (int wo = ly; wo < a.Wo; wo += lanes_y) {
          const float4 g = *reinterpret_cast<const float4*>(base + wo * C + c);
          const float* xc = xrow + wo * ps;
          auto tap = [&](int k, const float* xp) {
            const float4 xv = *reinterpret_cast<const float4*>(xp);
            acc[k].x = fmaf(xv.x, g.x, acc[k].x);
            acc[k].y = fmaf(xv.y, g.y, acc[k].y);
            acc[k].z = fmaf(xv.z, g.z, acc[k].z);
            acc[k].w = fmaf(xv.w, g.w, acc[k].w);
          };
          if (v0) {
            tap(0, xc);
            tap(1, xc + C);
            tap(2, xc + 2 * C);
          }
          if (v1) {
            tap(3, xc + rs);
            tap(4, xc + rs + C);
            tap(5, xc + rs + 2 * C);
          }
          if (v2) {
            tap(6, xc + 2 * rs);
            tap(7, xc + 2 * rs + C);
            tap(8, xc + 2 * rs + 2 * C);
          }
        }
      } else if (active) {
        for (int wo = ly; wo < a.Wo; wo += lanes_y) {
          const float4 g = *reinterpret_cast<const float4*>(base + wo * C + c);
          const float* xcol = base + dy_floats + (wo * a.sW) * C + c;
#pragma unroll
          for (int k = 0; k < KMAX; ++k) {
            if (k < taps) {
              const int kh = k / a.kW, kw = k - kh * a.kW;
              if (valid[sl * a.kH + kh] != 0) {
                const float4 xv = *reinterpret_cast<const float4*>(xcol + (kh * st.Wp + kw) * C);
                acc[k].x = fmaf(xv.x, g.x, acc[k].x);
                acc[k].y = fmaf(xv.y, g.y, acc[k].y);
                acc[k].z = fmaf(xv.z, g.z, acc[k].z);
                acc[k].w = fmaf(xv.w, g.w, acc[k].w);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&empty[sl])) : "memory");
    }
  }
  const int64_t out_base = (int64_t)blockIdx.x * taps * C;
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    if (k >= taps) break;
    __syncthreads();
    if (consumer) s_fold[ct] = acc[k];
    __syncthreads();
    if (consumer && ly == 0 && cgl < cg) {
      float4 sum = s_fold[cgl];
      for (int l = 1; l < lanes_y; ++l) sum = fadd4(sum, s_fold[l * cgx + cgl]);
      *reinterpret_cast<float4*>(partial + out_base + (int64_t)k * C + c) = sum;
    }
  }
}

// Stage 1, any shape: one CTA per (pixel chunk, filter-element chunk); each
// thread owns one filter element and walks the chunk's pixels.
__global__ void __launch_bounds__(kThreads) dw_wgrad_partial_scalar_kernel(const float* __restrict__ x,
                                                                            const float* __restrict__ dy,
                                                                            float* __restrict__ partial, DwArgs a,
                                                                            int64_t pix_per_block) {
  const int F = a.kH * a.kW * a.C * a.dm;
  const int f = blockIdx.y * kThreads + threadIdx.x;
  if (f >= F) return;
  const int d = f % a.dm;
  const int ci = (f / a.dm) % a.C;
  const int kw = (f / (a.dm * a.C)) % a.kW;
  const int kh = f / (a.dm * a.C * a.kW);
  const int Co = a.C * a.dm;
  const int co = ci * a.dm + d;
  const int64_t pixels = (int64_t)a.N * a.Ho * a.Wo;
  const int64_t p_begin = (int64_t)blockIdx.x * pix_per_block;
  int64_t p_end = p_begin + pix_per_block;
  if (p_end > pixels) p_end = pixels;
  float acc = 0.0f;
  for (int64_t p = p_begin; p < p_end; ++p) {
    const int wo = (int)(p % a.Wo);
    const int64_t q = p / a.Wo;
    const int ho = (int)(q % a.Ho);
    const int n = (int)(q / a.Ho);
    const int hi = ho * a.sH - a.pH + kh, wi = wo * a.sW - a.pW + kw;
    if ((unsigned)hi >= (unsigned)a.H || (unsigned)wi >= (unsigned)a.W) continue;
    acc = fmaf(__ldg(x + ((int64_t)(n * a.H + hi) * a.W + wi) * a.C + ci), __ldg(dy + p * Co + co), acc);
  }
  partial[(int64_t)blockIdx.x * F + f] = acc;
}

// Stage 2: dw[f] = sum over blocks of partial[b][f] in a fixed order: CTA of
// 32 x 32 threads per 32 filter elements; part j adds blocks j, j+32, ... in
// order, then the 32 part sums are added in part order.
constexpr int kFinParts = 32;
__global__ void __launch_bounds__(32 * kFinParts) dw_wgrad_finalize_kernel(const float* __restrict__ partial,
                                                                           int blocks, int F,
                                                                           float* __restrict__ dw) {
  __shared__ float s_part[kFinParts][32];
  const int f = blockIdx.x * 32 + threadIdx.x;
  const int part = threadIdx.y;
  float acc = 0.0f;
  if (f < F) {
#pragma unroll 4
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

// Threads of a row CTA: x over channel groups, y over pixels of the row.
dim3 row_block(int cg, int64_t width) {
  const int bx = cg < kThreads ? cg : kThreads;
  int by = kThreads / bx;
  if (by > width) by = (int)(width > 0 ? width : 1);
  return dim3((unsigned)bx, (unsigned)by);
}

int dw_forward_geom(const int64_t* input_shape, const int64_t* filter_shape, const int32_t* strides,
                    int num_strides, const char* padding, bool forward, ConvGeom* g) {
  B2_RETURN_IF_ERROR(check_dims_nonneg(input_shape, 4, "input"));
  B2_RETURN_IF_ERROR(check_dims_nonneg(filter_shape, 4, "filter"));
  B2_RETURN_IF_ERROR(parse_conv_attrs(strides, num_strides, padding, forward, g));
  g->N = input_shape[0]; g->H = input_shape[1]; g->W = input_shape[2]; g->Ci = input_shape[3];
  g->kH = filter_shape[0]; g->kW = filter_shape[1]; g->dm = filter_shape[3];
  g->Co = g->Ci * g->dm;
  finish_geom(g);
  return B2_OK;
}

}  // namespace

// Expired bounded waits of the staged depthwise kernels (read by
// b2_device_timeouts).
unsigned int dw_timeouts() {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_dw_timeouts, sizeof(v));
  return v;
}

}  // namespace b2

using namespace b2;

extern "C" {

int b2_depthwise_conv2d_output_shape(const int64_t input_shape[4], const int64_t filter_shape[4],
                                     const int32_t* strides, int num_strides, const char* padding,
                                     int64_t out_shape[4]) {
  clear_error();
  ConvGeom g;
  B2_RETURN_IF_ERROR(dw_forward_geom(input_shape, filter_shape, strides, num_strides, padding, true, &g));
  B2_REQUIRE(filter_shape[2] == input_shape[3], "filter[2] must equal input channels");
  out_shape[0] = g.N; out_shape[1] = g.Ho; out_shape[2] = g.Wo; out_shape[3] = g.Co;
  return B2_OK;
}

// src/ops/depthwise_conv2d_ops.cc:107-187
int b2_depthwise_conv2d(b2_stream_t stream, const float* input, const int64_t input_shape[4], const float* filter,
                        const int64_t filter_shape[4], const int32_t* strides, int num_strides, const char* padding,
                        float* output, const int64_t output_shape[4]) {
  clear_error();
  ConvGeom g;
  B2_RETURN_IF_ERROR(dw_forward_geom(input_shape, filter_shape, strides, num_strides, padding, true, &g));
  B2_REQUIRE(filter_shape[2] == g.Ci, "filter[2] must equal input channels");
  B2_RETURN_IF_ERROR(check_dims_nonneg(output_shape, 4, "output"));
  B2_REQUIRE(output_shape[0] == g.N && output_shape[1] == g.Ho && output_shape[2] == g.Wo &&
                 output_shape[3] == g.Co,
             "output shape must be [N, Hout, Wout, C*depth_multiplier] = [%lld, %lld, %lld, %lld]",
             (long long)g.N, (long long)g.Ho, (long long)g.Wo, (long long)g.Co);
  B2_RETURN_IF_ERROR(check_int32_sizes(g));
  if (g.out_elems() == 0) return B2_OK;
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const DwArgs a = to_args(g);
  if (g.dm == 1 && g.Ci % 4 == 0 && aligned16(input) && aligned16(filter) && aligned16(output)) {
    if (g.kH == 3 && g.kW == 3 && g.sH == 2 && g.sW == 2) {
      const int pairs = (int)((g.Wo + 1) / 2);
      const dim3 blk = row_block((int)(g.Ci / 4), pairs);
      const int64_t chunks = ceil_div(g.Ci / 4, (int64_t)blk.x);
      const int64_t rows = g.N * g.Ho;
      int64_t want = (int64_t)d->sm_count * 16 / chunks;
      if (want < 1) want = 1;
      int64_t rpb = ceil_div(rows, want);
      if (rpb > 8) rpb = 8;
      const dim3 grid((unsigned)ceil_div(rows, rpb), (unsigned)chunks);
      dw_fwd_s2k3_kernel<<<grid, blk, 0, s>>>(input, filter, output, a, pairs, (int)rpb);
    } else {
      dw_fwd_vec4_kernel<<<grid_for(g.out_elems() / 4, kThreads, 8), kThreads, 0, s>>>(input, filter, output, a);
    }
  } else {
    dw_fwd_scalar_kernel<<<grid_for(g.out_elems(), kThreads, 8), kThreads, 0, s>>>(input, filter, output, a);
  }
  return check_launch(s, "dwconv2d_forward");
}

// src/ops/depthwise_conv2d_ops.cc:221-305
int b2_depthwise_conv2d_backprop_input(b2_stream_t stream, const int32_t input_sizes[4], const float* filter,
                                       const int64_t filter_shape[4], const float* out_backprop,
                                       const int64_t out_backprop_shape[4], const int32_t* strides,
                                       int num_strides, const char* padding, float* output) {
  clear_error();
  B2_REQUIRE(input_sizes != nullptr, "input_sizes must have 4 elements");
  const int64_t in_shape[4] = {input_sizes[0], input_sizes[1], input_sizes[2], input_sizes[3]};
  ConvGeom g;
  B2_RETURN_IF_ERROR(dw_forward_geom(in_shape, filter_shape, strides, num_strides, padding, false, &g));
  B2_REQUIRE(filter_shape[2] == g.Ci, "filter[2] != C");
  B2_RETURN_IF_ERROR(check_dims_nonneg(out_backprop_shape, 4, "out_backprop"));
  B2_REQUIRE(out_backprop_shape[0] == g.N && out_backprop_shape[1] == g.Ho && out_backprop_shape[2] == g.Wo &&
                 out_backprop_shape[3] == g.Co,
             "out_backprop shape mismatch");
  B2_RETURN_IF_ERROR(check_int32_sizes(g));
  if (g.in_elems() == 0) return B2_OK;
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const DwArgs a = to_args(g);
  if (g.dm == 1 && g.Ci % 4 == 0 && aligned16(out_backprop) && aligned16(filter) && aligned16(output)) {
    if (g.kH == 3 && g.kW == 3 && g.sH == 2 && g.sW == 2) {
      const int pairs = (int)((g.W + g.pW + 1) / 2);
      const dim3 blk = row_block((int)(g.Ci / 4), pairs);
      const int64_t chunks = ceil_div(g.Ci / 4, (int64_t)blk.x);
      const int64_t rows = g.N * g.H;
      int64_t want = (int64_t)d->sm_count * 16 / chunks;
      if (want < 1) want = 1;
      int64_t rpb = ceil_div(rows, want);
      if (rpb > 8) rpb = 8;
      const dim3 grid((unsigned)ceil_div(rows, rpb), (unsigned)chunks);
      dw_dgrad_s2k3_kernel<<<grid, blk, 0, s>>>(out_backprop, filter, output, a, pairs, (int)rpb);
    } else {
      dw_dgrad_rows_kernel<<<(unsigned)(g.N * g.H), row_block((int)(g.Ci / 4), g.W), 0, s>>>(out_backprop, filter,
                                                                                            output, a);
    }
  } else {
    dw_dgrad_scalar_kernel<<<grid_for(g.in_elems(), kThreads, 8), kThreads, 0, s>>>(out_backprop, filter,
                                                                                    output, a);
  }
  return check_launch(s, "dwconv2d_backprop_input");
}

// src/ops/depthwise_conv2d_ops.cc:341-426
int b2_depthwise_conv2d_backprop_filter(b2_stream_t stream, const float* input, const int64_t input_shape[4],
                                        const int32_t filter_sizes[4], const float* out_backprop,
                                        const int64_t out_backprop_shape[4], const int32_t* strides,
                                        int num_strides, const char* padding, float* output) {
  clear_error();
  B2_REQUIRE(filter_sizes != nullptr, "filter_sizes must have 4 elements");
  const int64_t f_shape[4] = {filter_sizes[0], filter_sizes[1], filter_sizes[2], filter_sizes[3]};
  ConvGeom g;
  B2_RETURN_IF_ERROR(dw_forward_geom(input_shape, f_shape, strides, num_strides, padding, false, &g));
  B2_REQUIRE(input_shape[3] == f_shape[2], "input channels != filter_sizes[2]");
  B2_RETURN_IF_ERROR(check_dims_nonneg(out_backprop_shape, 4, "out_backprop"));
  B2_REQUIRE(out_backprop_shape[0] == g.N && out_backprop_shape[1] == g.Ho && out_backprop_shape[2] == g.Wo &&
                 out_backprop_shape[3] == g.Co,
             "out_backprop shape mismatch");
  B2_RETURN_IF_ERROR(check_int32_sizes(g));
  const int64_t F = g.kH * g.kW * g.Ci * g.dm;
  if (F == 0) return B2_OK;
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const DwArgs a = to_args(g);
  const int64_t pixels = g.N * g.Ho * g.Wo;
  if (pixels == 0) {
    B2_CUDA_OR_RETURN(cudaMemsetAsync(output, 0, sizeof(float) * F, s));
    return B2_OK;
  }
  const int taps = (int)(g.kH * g.kW);
  const bool vec = g.dm == 1 && g.Ci % 4 == 0 && taps <= 9 && aligned16(input) && aligned16(out_backprop);
  Scratch part;
  int blocks = 0;
  // staged path: slots of (dy row + kH padded input rows) fit ~100 KB x S
  const int64_t padL = g.pW;
  int64_t padR = (g.Wo - 1) * g.sW + g.kW - (g.W + padL);
  if (padR < 0) padR = 0;
  const int64_t Wp = g.W + padL + padR;
  const int64_t slot_floats = g.Wo * g.Ci + g.kH * Wp * g.Ci;
  const int64_t slots = slot_floats > 0 ? (int64_t)100 * 1024 / (slot_floats * 4) : 0;
  if (vec && slots >= 2 && g.Ci / 4 <= kStagedConsumers && g.N * g.Ho <= kMaxInt32) {
    const DwStage st{(int)(slots > 6 ? 6 : slots), (int)padL, (int)Wp, (int)slot_floats, wait_params()};
    const size_t smem = (size_t)st.slots * st.slot_floats * 4 + 16 * st.slots + 4 * st.slots * g.kH + 16;
    static SmemOptIn opt_in;
    B2_RETURN_IF_ERROR(
        opt_in.ensure(reinterpret_cast<const void*>(dw_wgrad_staged_kernel<9>), d->device, 110 * 1024));
    const int cgx = (int)(g.Ci / 4);
    int lanes_y = kStagedConsumers / cgx;
    if (lanes_y > g.Wo) lanes_y = (int)g.Wo;
    const int nthreads = 32 + ((cgx * lanes_y + 31) / 32) * 32;
    const int64_t rows = g.N * g.Ho;
    int per_sm = 0;
    B2_CUDA_OR_RETURN(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, dw_wgrad_staged_kernel<9>, nthreads,
                                                                    smem));
    int64_t want = (int64_t)d->sm_count * (per_sm > 0 ? per_sm : 1);
    blocks = (int)(want < rows ? want : rows);
    const int64_t rpb = ceil_div(rows, blocks);
    blocks = (int)ceil_div(rows, rpb);
    B2_RETURN_IF_ERROR(part.alloc(sizeof(float) * blocks * F, s));
    dw_wgrad_staged_kernel<9><<<blocks, nthreads, smem, s>>>(input, out_backprop, part.as<float>(), a, st, cgx,
                                                              lanes_y, (int)rpb);
  } else if (vec) {
    const int cg_total = (int)(g.Ci / 4);
    const int cg_per_cta = cg_total < kThreads ? cg_total : kThreads;
    const int chunks = (int)ceil_div(cg_total, cg_per_cta);
    int64_t want = (int64_t)d->sm_count * 8 / chunks;
    if (want < 1) want = 1;
    int64_t cap = ceil_div(pixels, 32);
    blocks = (int)(want < cap ? want : cap);
    const int64_t ppb = ceil_div(pixels, blocks);
    blocks = (int)ceil_div(pixels, ppb);
    B2_RETURN_IF_ERROR(part.alloc(sizeof(float) * blocks * F, s));
    dw_wgrad_partial_vec4_kernel<9><<<dim3(blocks, chunks), kThreads, 0, s>>>(input, out_backprop,
                                                                              part.as<float>(), a, cg_per_cta, ppb);
  } else {
    int64_t want = (int64_t)d->sm_count * 2;
    int64_t cap = ceil_div(pixels, 256);
    blocks = (int)(want < cap ? want : cap);
    if (blocks < 1) blocks = 1;
    const int64_t ppb = ceil_div(pixels, blocks);
    blocks = (int)ceil_div(pixels, ppb);
    B2_RETURN_IF_ERROR(part.alloc(sizeof(float) * blocks * F, s));
    dw_wgrad_partial_scalar_kernel<<<dim3(blocks, (unsigned)ceil_div(F, kThreads)), kThreads, 0, s>>>(
        input, out_backprop, part.as<float>(), a, ppb);
  }
  B2_RETURN_IF_ERROR(check_launch(s, "dwconv2d_backprop_filter"));
  dw_wgrad_finalize_kernel<<<(unsigned)ceil_div(F, 32), dim3(32, kFinParts), 0, s>>>(part.as<float>(), blocks,
                                                                                       (int)F, output);
  return check_launch(s, "dwconv2d_backprop_filter_finalize");
}

}  // extern "C"
