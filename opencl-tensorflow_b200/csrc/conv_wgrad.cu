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
// window in registers instead: a thread owns (kh, 4 output channels) and
// accumulates 21 x 4 sums over WPT = 4 adjacent output columns, whose windows
// overlap (stride 2: each column adds 2 pixels), so a column costs 84 FMAs
// against one 16-byte load of dy and 1.5 of x.
//
// Work unit: one output row (n, ho), or a chunk of Wc of its columns.  A CTA
// (one per SM) walks a contiguous range of units; all its threads stage
// units -- the dy chunk and the kH input row segments it reads, zero-filled
// outside the image -- with cp.async into a ring of buffers, several units
// ahead of the one they compute on.  Teams of kH * Co/4 threads split the unit's columns.  At the
// end the CTA folds its teams in team order and writes one partial per filter
// element; a second kernel adds the CTA partials in block order, so results
// are deterministic.
//
// FUSED: dy is not read but computed while staged, from the BatchNorm ->
// ReLU backward's inputs (dz and the BN input y) and its per-channel
// constants, with the same arithmetic as the BatchNorm dx pass (so the filter
// gradient equals the unfused sequence's bit for bit), and never written to
// HBM.
#include <climits>

#include "bn_common.cuh"
#include "conv_common.cuh"

namespace b2 {
namespace {

constexpr int kWgThreads = 288;  // 9 warps
constexpr int kWgWpt = 4;        // output columns per thread per unit
constexpr int kWgStages = 6;     // unit buffers: 5 units in flight while one is computed
constexpr int kWgConsts = 7;     // fused: mean, inv_std, k1, grad_beta, grad_gamma, gamma, beta

struct WgGeom {
  int N, H, W, Co, kH, sH, pH, pW, Ho, Wo;
  int teams;      // teams per CTA
  int team;       // threads per team: kH * Co / 4
  int Wc;         // output columns per unit: teams * kWgWpt
  int chunks;     // units per output row
  int seg;        // staged floats per input row (multiple of 4)
  int seg_valid;  // of which real input positions: ((Wc - 1) * sW + kW) * Ci
  int units;      // N * Ho * chunks
  int upb;        // units per CTA
};

struct BnDx {
  const float *mean, *inv_std, *k1, *grad_beta, *grad_gamma, *gamma, *beta;
  float nhw_f;
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16- / 4-byte asynchronous copies into shared memory; `valid` false writes
// zeros and reads nothing (src-size 0; src is then any valid address).
__device__ __forceinline__ void cp_async16(float* dst, const float* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
               "r"(valid ? 16u : 0u)
               : "memory");
}

__device__ __forceinline__ void cp_async4(float* dst, const float* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_addr(dst)), "l"(src),
               "r"(valid ? 4u : 0u)
               : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Shared-memory plan (floats): [fused constants 7 x Co] then kWgStages unit
// buffers (dy chunk [Wc][Co], fused: BN-input chunk [Wc][Co], input rows
// [kH][seg]), overlaid after the walk by the team fold [teams][team][KWC][4].
// One CTA per SM computes a unit in ~0.4 us; a DRAM round trip takes longer,
// so several units must be in flight at once.
struct WgSmem {
  int consts, buf, fold, total;
};

template <int KWC>
__host__ __device__ inline WgSmem wg_smem(const WgGeom& g, bool fused) {
  WgSmem s;
  s.consts = fused ? kWgConsts * g.Co : 0;
  s.buf = g.Wc * g.Co * (fused ? 2 : 1) + g.kH * g.seg;
  s.fold = g.teams * g.team * KWC * 4;
  const int body = kWgStages * s.buf > s.fold ? kWgStages * s.buf : s.fold;
  s.total = s.consts + body;
  return s;
}

template <int KW, int CI, int SW, bool FUSED>
__global__ void __launch_bounds__(kWgThreads, 1)
    conv_wgrad_rows_kernel(const float* __restrict__ x, const float* __restrict__ dy,
                           const float* __restrict__ ybn, BnDx bn, WgGeom g, float* __restrict__ partial) {
  constexpr int KWC = KW * CI;
  constexpr int STEP = SW * CI;                        // window shift per output column
  constexpr int NWIN = (kWgWpt - 1) * STEP + KWC;      // floats of x a thread's columns read per kh
  constexpr int NWIN4 = (NWIN + 3) / 4 * 4;
  static_assert((kWgWpt * STEP) % 4 == 0, "team windows must start 16-byte aligned");
  extern __shared__ __align__(16) float wsm[];
  const WgSmem plan = wg_smem<KWC>(g, FUSED);
  const int tid = threadIdx.x;
  const int Co = g.Co, cq = Co / 4;

  if (FUSED) {
    for (int c = tid; c < Co; c += blockDim.x) {
      wsm[c] = bn.mean[c];
      wsm[Co + c] = bn.inv_std[c];
      wsm[2 * Co + c] = bn.k1[c];
      wsm[3 * Co + c] = bn.grad_beta[c];
      wsm[4 * Co + c] = bn.grad_gamma[c];
      wsm[5 * Co + c] = bn.gamma[c];
      wsm[6 * Co + c] = bn.beta[c];
    }
  }
  float* body = wsm + plan.consts;

  // this thread's role: team (a group of Wc / teams output columns), filter
  // row kh, output channels 4*cg .. 4*cg+3
  const int team = tid / g.team, r = tid - team * g.team;
  const int kh = r / cq, cg = r - kh * cq;
  const bool computes = team < g.teams;

  auto stage = [&](int u, int b) {
    const int row = u / g.chunks, c = u - row * g.chunks;  // row = n * Ho + ho
    const int n = row / g.Ho, ho = row - n * g.Ho;
    const int wo0 = c * g.Wc;
    float* buf = body + b * plan.buf;
    const int64_t d0 = ((int64_t)row * g.Wo + wo0) * Co;
    const int nq = g.Wc * cq;
    for (int i = tid; i < nq; i += blockDim.x) {
      const bool ok = wo0 + i / cq < g.Wo;
      const int64_t off = d0 + 4 * (int64_t)i;
      cp_async16(buf + 4 * i, ok ? dy + off : dy, ok);
      if (FUSED) cp_async16(buf + g.Wc * Co + 4 * i, ok ? ybn + off : ybn, ok);
    }
    float* xs = buf + g.Wc * Co * (FUSED ? 2 : 1);
    const int w0 = SW * wo0 - g.pW;  // input column of staged position 0
    const int nx = g.kH * g.seg;
    for (int i = tid; i < nx; i += blockDim.x) {
      const int rk = i / g.seg, j = i - rk * g.seg;
      const int hi = ho * g.sH - g.pH + rk;
      const int wi = w0 + j / CI, ci = j - (j / CI) * CI;
      const bool ok = j < g.seg_valid && hi >= 0 && hi < g.H && wi >= 0 && wi < g.W;
      cp_async4(xs + i, ok ? x + (((int64_t)n * g.H + hi) * g.W + wi) * CI + ci : x, ok);
    }
  };

  float acc[KWC][4];
#pragma unroll
  for (int k = 0; k < KWC; ++k) acc[k][0] = acc[k][1] = acc[k][2] = acc[k][3] = 0.0f;

  const int u_begin = blockIdx.x * g.upb;
  const int u_end = u_begin + g.upb < g.units ? u_begin + g.upb : g.units;
  // ring: unit u_begin + i lives in buffer i % kWgStages; one commit group per
  // unit (empty past the end), so "at most kWgStages - 1 groups pending" means
  // the oldest unit has landed
#pragma unroll 1
  for (int j = 0; j < kWgStages - 1; ++j) {
    if (u_begin + j < u_end) stage(u_begin + j, j);
    cp_async_commit();
  }
  for (int u = u_begin; u < u_end; ++u) {
    const int i = u - u_begin;
    const int b = i % kWgStages;
    // the buffer unit u + kWgStages - 1 takes was computed on last iteration,
    // before its closing barrier
    if (u + kWgStages - 1 < u_end) stage(u + kWgStages - 1, (i + kWgStages - 1) % kWgStages);
    cp_async_commit();
    cp_async_wait<kWgStages - 1>();  // this thread's copies of unit u have landed
    __syncthreads();                 // ... and everyone's
    float* buf = body + b * plan.buf;
    if (FUSED) {
      // dy = BatchNorm -> ReLU backward of (dz, y), in place of dz
      const int row = u / g.chunks;
      const int wo0 = (u - row * g.chunks) * g.Wc;
      const float* yb = buf + g.Wc * Co;
      const float* cs = wsm;
      for (int e = tid; e < g.Wc * Co; e += blockDim.x) {
        const int wl = e / Co, ch = e - wl * Co;
        float v = 0.0f;
        if (wo0 + wl < g.Wo)
          v = bn_grad_dx_value<true>(yb[e], buf[e], cs[ch], cs[Co + ch], cs[2 * Co + ch], cs[3 * Co + ch],
                                     cs[4 * Co + ch], cs[5 * Co + ch], cs[6 * Co + ch], bn.nhw_f);
        buf[e] = v;
      }
      __syncthreads();
    }
    if (computes) {
      const float* xs = buf + g.Wc * Co * (FUSED ? 2 : 1);
      const float* xw = xs + kh * g.seg + team * kWgWpt * STEP;
      float win[NWIN4];
#pragma unroll
      for (int q = 0; q < NWIN4 / 4; ++q) {
        const float4 v = *reinterpret_cast<const float4*>(xw + 4 * q);
        win[4 * q] = v.x;
        win[4 * q + 1] = v.y;
        win[4 * q + 2] = v.z;
        win[4 * q + 3] = v.w;
      }
      float d[kWgWpt][4];
#pragma unroll
      for (int i = 0; i < kWgWpt; ++i) {
        const float4 v = *reinterpret_cast<const float4*>(buf + (team * kWgWpt + i) * Co + 4 * cg);
        d[i][0] = v.x;
        d[i][1] = v.y;
        d[i][2] = v.z;
        d[i][3] = v.w;
      }
#pragma unroll
      for (int i = 0; i < kWgWpt; ++i)
#pragma unroll
        for (int k = 0; k < KWC; ++k)
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[k][c] = fmaf(win[i * STEP + k], d[i][c], acc[k][c]);
    }
    __syncthreads();  // buffer b is restaged by the next iteration
  }
  cp_async_wait<0>();
  __syncthreads();

  // Fold the teams in team order, one partial per filter element (HWIO).
  float* fold = body;
  if (computes) {
#pragma unroll
    for (int k = 0; k < KWC; ++k)
      *reinterpret_cast<float4*>(fold + ((size_t)(team * g.team + r) * KWC + k) * 4) =
          make_float4(acc[k][0], acc[k][1], acc[k][2], acc[k][3]);
  }
  __syncthreads();
  if (computes && team == 0) {
    const int64_t F = (int64_t)g.kH * KWC * Co;
    float* out = partial + (int64_t)blockIdx.x * F;
#pragma unroll 1
    for (int k = 0; k < KWC; ++k) {
      float4 s = *reinterpret_cast<const float4*>(fold + ((size_t)r * KWC + k) * 4);
      for (int t = 1; t < g.teams; ++t) {
        const float4 v = *reinterpret_cast<const float4*>(fold + ((size_t)(t * g.team + r) * KWC + k) * 4);
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
      *reinterpret_cast<float4*>(out + ((int64_t)kh * KWC + k) * Co + 4 * cg) = s;
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

}  // namespace

// The shapes this kernel takes: a 7-wide filter over 3 input channels with
// column stride 2 (the README stem, any batch / image size / filter height up
// to 8 / output channel count that is a multiple of 4 and fits a team), and a
// 16-byte aligned output gradient.
bool conv_wgrad_rows_ok(const ConvGeom& g, const float* dy, const float* ybn) {
  if (g.kW != kStemKW || g.Ci != kStemCI || g.sW != kStemSW) return false;
  if (g.Co < 4 || g.Co % 4 != 0 || g.kH < 1 || g.kH > 8 || g.N < 1 || g.Ho < 1 || g.Wo < 1) return false;
  if (g.kH * g.Co / 4 > kWgThreads) return false;
  if (!aligned16(dy) || (ybn != nullptr && !aligned16(ybn))) return false;
  const int64_t teams = kWgThreads / (g.kH * g.Co / 4);
  const int64_t wc = teams * kWgWpt;
  // shared memory (the fused plan is the larger): 7 constants per channel, the
  // ring of unit buffers or the team fold, within the 227 KB a CTA may use
  const int64_t seg = ((wc - 1) * kStemSW + kStemKW) * kStemCI + 8;
  const int64_t ring = kWgStages * (wc * g.Co * 2 + g.kH * seg);
  const int64_t fold = kWgThreads * kStemKW * kStemCI * 4;
  if (4 * (kWgConsts * g.Co + (ring > fold ? ring : fold)) > 227 * 1024) return false;
  return g.N * g.Ho * ceil_div(g.Wo, wc) <= INT_MAX && g.H <= INT_MAX && g.W <= INT_MAX;
}

namespace {

// dW for a shape conv_wgrad_rows_ok accepts.  fused != nullptr: `dy` is the
// ReLU-output gradient dz and `ybn` the BatchNorm input, and the output
// gradient is the BatchNorm -> ReLU backward of them with these constants.
int wgrad_rows(const ConvGeom& g, const float* x, const float* dy, const float* ybn, const BnDx* fused, float* dw,
               cudaStream_t s) {
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  WgGeom w;
  w.N = (int)g.N; w.H = (int)g.H; w.W = (int)g.W; w.Co = (int)g.Co; w.kH = (int)g.kH; w.sH = (int)g.sH;
  w.pH = (int)g.pH; w.pW = (int)g.pW; w.Ho = (int)g.Ho; w.Wo = (int)g.Wo;
  w.team = w.kH * w.Co / 4;
  w.teams = kWgThreads / w.team;
  w.Wc = w.teams * kWgWpt;
  w.chunks = (int)ceil_div(w.Wo, w.Wc);
  constexpr int KWC = kStemKW * kStemCI, STEP = kStemSW * kStemCI;
  constexpr int NWIN4 = ((kWgWpt - 1) * STEP + KWC + 3) / 4 * 4;
  w.seg_valid = ((w.Wc - 1) * kStemSW + kStemKW) * kStemCI;
  const int need = (w.teams - 1) * kWgWpt * STEP + NWIN4;  // the last team's window read
  w.seg = (int)ceil_div(w.seg_valid > need ? w.seg_valid : need, 4) * 4;
  w.units = w.N * w.Ho * w.chunks;
  int blocks = w.units < d->sm_count ? w.units : d->sm_count;
  w.upb = (int)ceil_div(w.units, blocks);
  blocks = (int)ceil_div(w.units, w.upb);
  const bool is_fused = fused != nullptr;
  const WgSmem plan = wg_smem<KWC>(w, is_fused);
  const int smem = plan.total * (int)sizeof(float);
  B2_REQUIRE(smem <= d->max_smem_optin, "conv2d_backprop_filter: %d bytes of shared memory needed", smem);
  const int64_t F = g.kH * KWC * g.Co;
  Scratch part;
  B2_RETURN_IF_ERROR(part.alloc(sizeof(float) * (size_t)blocks * F, s));
  const BnDx bn = is_fused ? *fused : BnDx{};
  if (is_fused) {
    static SmemOptIn opt_in;
    auto k = conv_wgrad_rows_kernel<kStemKW, kStemCI, kStemSW, true>;
    B2_RETURN_IF_ERROR(opt_in.ensure(reinterpret_cast<const void*>(k), d->device, smem));
    k<<<blocks, kWgThreads, smem, s>>>(x, dy, ybn, bn, w, part.as<float>());
  } else {
    static SmemOptIn opt_in;
    auto k = conv_wgrad_rows_kernel<kStemKW, kStemCI, kStemSW, false>;
    B2_RETURN_IF_ERROR(opt_in.ensure(reinterpret_cast<const void*>(k), d->device, smem));
    k<<<blocks, kWgThreads, smem, s>>>(x, dy, nullptr, bn, w, part.as<float>());
  }
  B2_RETURN_IF_ERROR(check_launch(s, is_fused ? "conv2d_bn_relu_backprop_filter" : "conv2d_backprop_filter"));
  wgrad_block_sum_kernel<<<(unsigned)ceil_div(F, 32), dim3(32, kSumParts), 0, s>>>(part.as<float>(), blocks,
                                                                                   (int)F, dw);
  return check_launch(s, "conv2d_backprop_filter_sum");
}

}  // namespace

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
  if (conv_direct_ok(g) || !conv_wgrad_rows_ok(g, grad_z, bn_input) || rows == 0) {
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
