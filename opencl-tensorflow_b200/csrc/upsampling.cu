// upsampling.cu -- bilinear UpSampling2D forward and backward.
//
// Reference: kernels/upsampling_bilinear_kernels.cl, src/ops/upsampling_ops.cc.
// Half-pixel centres: src = (o + 0.5f) * (float)in / (float)out - 0.5f, floor,
// clamp both corners to [0, in-1], fraction = src - floor.
//
// Exactness: the coordinate, fraction and blend arithmetic is written with
// round-to-nearest intrinsics in the reference's evaluation order, so the
// corner indices, fractions and forward outputs are bit-identical to the
// reference evaluated in IEEE fp32.
//
// Backward: the reference zero-fills grad_in and scatters four weighted
// terms per output element with a float compare-and-swap loop
// (upsampling_bilinear_kernels.cl:22-30, 94-135), so its result depends on
// the order atomics land.  Here it is a gather: one thread per input element
// (4 channels per thread when C % 4 == 0) visits every output position whose
// clamped corners include it, in ascending (oh, ow) order and corner order
// 00, 01, 10, 11 -- the order a single-threaded run of the reference adds
// in -- so grad_in is deterministic and equal bit for bit to that run.
#include "b2_internal.cuh"

namespace b2 {
namespace {

constexpr int kThreads = 256;

struct Coord {
  int lo, hi;
  float frac;
};

// upsampling_bilinear_kernels.cl:51-64
__device__ __forceinline__ Coord up_coord(int o, int in, int out) {
  const float f =
      __fsub_rn(__fdiv_rn(__fmul_rn(__fadd_rn((float)o, 0.5f), (float)in), (float)out), 0.5f);
  const int i0 = (int)floorf(f);
  const int i1 = i0 + 1;
  Coord c;
  c.frac = __fsub_rn(f, (float)i0);
  c.lo = max(0, min(i0, in - 1));
  c.hi = max(0, min(i1, in - 1));
  return c;
}

struct UpArgs {
  int N, H, W, C, Ho, Wo;
};

template <int VEC>
struct V;
template <>
struct V<1> {
  using T = float;
};
template <>
struct V<4> {
  using T = float4;
};

__device__ __forceinline__ float blend(float dh, float dw, float v00, float v01, float v10, float v11) {
  const float a = __fsub_rn(1.0f, dh), b = __fsub_rn(1.0f, dw);
  float s = __fmul_rn(__fmul_rn(a, b), v00);
  s = __fadd_rn(s, __fmul_rn(__fmul_rn(a, dw), v01));
  s = __fadd_rn(s, __fmul_rn(__fmul_rn(dh, b), v10));
  s = __fadd_rn(s, __fmul_rn(__fmul_rn(dh, dw), v11));
  return s;
}

// upsampling_bilinear_kernels.cl:35-84; VEC channels per thread.
template <int VEC>
__global__ void __launch_bounds__(kThreads) up_fwd_kernel(const float* __restrict__ x, float* __restrict__ y,
                                                           UpArgs a) {
  using T = typename V<VEC>::T;
  const int cg = a.C / VEC;
  const int64_t total = (int64_t)a.N * a.Ho * a.Wo * cg;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t g = (int64_t)blockIdx.x * kThreads + threadIdx.x; g < total; g += stride) {
    const uint32_t p = (uint32_t)g / (uint32_t)cg;  // element counts < 2^31 (checked on the host)
    const int c = (int)((uint32_t)g - p * (uint32_t)cg) * VEC;
    const uint32_t q = p / (uint32_t)a.Wo;
    const int ow = (int)(p - q * (uint32_t)a.Wo);
    const uint32_t n32 = q / (uint32_t)a.Ho;
    const int oh = (int)(q - n32 * (uint32_t)a.Ho);
    const int n = (int)n32;
    const Coord ch = up_coord(oh, a.H, a.Ho);
    const Coord cw = up_coord(ow, a.W, a.Wo);
    const float* base = x + (int64_t)n * a.H * a.W * a.C + c;
    const T v00 = *reinterpret_cast<const T*>(base + ((int64_t)ch.lo * a.W + cw.lo) * a.C);
    const T v01 = *reinterpret_cast<const T*>(base + ((int64_t)ch.lo * a.W + cw.hi) * a.C);
    const T v10 = *reinterpret_cast<const T*>(base + ((int64_t)ch.hi * a.W + cw.lo) * a.C);
    const T v11 = *reinterpret_cast<const T*>(base + ((int64_t)ch.hi * a.W + cw.hi) * a.C);
    T out;
    if constexpr (VEC == 4) {
      out.x = blend(ch.frac, cw.frac, v00.x, v01.x, v10.x, v11.x);
      out.y = blend(ch.frac, cw.frac, v00.y, v01.y, v10.y, v11.y);
      out.z = blend(ch.frac, cw.frac, v00.z, v01.z, v10.z, v11.z);
      out.w = blend(ch.frac, cw.frac, v00.w, v01.w, v10.w, v11.w);
    } else {
      out = blend(ch.frac, cw.frac, v00, v01, v10, v11);
    }
    reinterpret_cast<T*>(y)[g] = out;
  }
}

template <int VEC>
__device__ __forceinline__ void acc_term(float* acc, float w, const float* g) {
#pragma unroll
  for (int j = 0; j < VEC; ++j) acc[j] = __fadd_rn(acc[j], __fmul_rn(w, g[j]));
}

// Gather form of upsampling_bilinear_kernels.cl:94-135 (see file comment).
template <int VEC>
__global__ void __launch_bounds__(kThreads) up_bwd_kernel(const float* __restrict__ dy, float* __restrict__ dx,
                                                           UpArgs a, int sy, int sx) {
  using T = typename V<VEC>::T;
  const int cg = a.C / VEC;
  const int64_t total = (int64_t)a.N * a.H * a.W * cg;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t g = (int64_t)blockIdx.x * kThreads + threadIdx.x; g < total; g += stride) {
    const uint32_t p = (uint32_t)g / (uint32_t)cg;  // element counts < 2^31 (checked on the host)
    const int c = (int)((uint32_t)g - p * (uint32_t)cg) * VEC;
    const uint32_t q = p / (uint32_t)a.W;
    const int iw = (int)(p - q * (uint32_t)a.W);
    const uint32_t n32 = q / (uint32_t)a.H;
    const int ih = (int)(q - n32 * (uint32_t)a.H);
    const int n = (int)n32;
    // Every output row whose corners can reach input row ih lies in
    // [(ih-1)*sy - 1, (ih+2)*sy] (the exact test below decides).
    const int oh_lo = max(0, (ih - 1) * sy - 1), oh_hi = min(a.Ho - 1, (ih + 2) * sy);
    const int ow_lo = max(0, (iw - 1) * sx - 1), ow_hi = min(a.Wo - 1, (iw + 2) * sx);
    float acc[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) acc[j] = 0.0f;
    const float* gbase = dy + (int64_t)n * a.Ho * a.Wo * a.C + c;
    // The output columns that reach input column iw, computed once per
    // thread: bit 0 = lower corner is iw, bit 1 = upper corner is iw.
    constexpr int kMaxCols = 64;
    uint8_t col_hit[kMaxCols];
    float col_frac[kMaxCols];
    const int ncols = ow_hi - ow_lo + 1;
    const bool cached = ncols <= kMaxCols;
    if (cached) {
      for (int j = 0; j < ncols; ++j) {
        const Coord cw = up_coord(ow_lo + j, a.W, a.Wo);
        col_hit[j] = (uint8_t)((cw.lo == iw ? 1 : 0) | (cw.hi == iw ? 2 : 0));
        col_frac[j] = cw.frac;
      }
    }
    for (int oh = oh_lo; oh <= oh_hi; ++oh) {
      const Coord ch = up_coord(oh, a.H, a.Ho);
      const bool h0 = ch.lo == ih, h1 = ch.hi == ih;
      if (!h0 && !h1) continue;
      const float a_h = __fsub_rn(1.0f, ch.frac);
      for (int ow = ow_lo; ow <= ow_hi; ++ow) {
        Coord cw;
        bool w0, w1;
        if (cached) {
          const int hit = col_hit[ow - ow_lo];
          w0 = hit & 1;
          w1 = hit & 2;
          cw.frac = col_frac[ow - ow_lo];
        } else {
          cw = up_coord(ow, a.W, a.Wo);
          w0 = cw.lo == iw;
          w1 = cw.hi == iw;
        }
        if (!w0 && !w1) continue;
        float gv[VEC];
        const T t = *reinterpret_cast<const T*>(gbase + ((int64_t)oh * a.Wo + ow) * a.C);
        if constexpr (VEC == 4) {
          gv[0] = t.x; gv[1] = t.y; gv[2] = t.z; gv[3] = t.w;
        } else {
          gv[0] = t;
        }
        const float b_w = __fsub_rn(1.0f, cw.frac);
        if (h0 && w0) acc_term<VEC>(acc, __fmul_rn(a_h, b_w), gv);
        if (h0 && w1) acc_term<VEC>(acc, __fmul_rn(a_h, cw.frac), gv);
        if (h1 && w0) acc_term<VEC>(acc, __fmul_rn(ch.frac, b_w), gv);
        if (h1 && w1) acc_term<VEC>(acc, __fmul_rn(ch.frac, cw.frac), gv);
      }
    }
    if constexpr (VEC == 4)
      reinterpret_cast<float4*>(dx)[g] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    else
      dx[g] = acc[0];
  }
}

// The same gather with one CTA per image: the image's dy (Ho*Wo*C floats) and
// both axes' corner coordinates are staged in shared memory first, so the
// per-element walk (same candidates, same order, same arithmetic as
// up_bwd_kernel<1>, hence the same bits) reads shared memory only.  Used when
// the image fits kStagedSmemBytes -- the small heads this op closes networks
// with, where the global-memory walk was latency-bound at a few warps per SM.
constexpr int kStagedSmemBytes = 48 * 1024;

__global__ void __launch_bounds__(kThreads) up_bwd_staged_kernel(const float* __restrict__ dy,
                                                                  float* __restrict__ dx, UpArgs a, int sy, int sx,
                                                                  int vec_copy) {
  extern __shared__ float4 smem_v[];
  float* sdy = reinterpret_cast<float*>(smem_v);
  const int64_t img = (int64_t)a.Ho * a.Wo * a.C;
  Coord* rows = reinterpret_cast<Coord*>(sdy + img);
  Coord* cols = rows + a.Ho;
  const int n = blockIdx.x;
  const float* src = dy + (int64_t)n * img;
  if (vec_copy) {
    for (int64_t i = threadIdx.x; i < img / 4; i += kThreads)
      smem_v[i] = reinterpret_cast<const float4*>(src)[i];
  } else {
    for (int64_t i = threadIdx.x; i < img; i += kThreads) sdy[i] = src[i];
  }
  for (int o = threadIdx.x; o < a.Ho; o += kThreads) rows[o] = up_coord(o, a.H, a.Ho);
  for (int o = threadIdx.x; o < a.Wo; o += kThreads) cols[o] = up_coord(o, a.W, a.Wo);
  __syncthreads();
  const int per_img = a.H * a.W * a.C;
  float* out = dx + (int64_t)n * per_img;
  for (int e = threadIdx.x; e < per_img; e += kThreads) {
    const int c = e % a.C;
    const int p = e / a.C;
    const int iw = p % a.W, ih = p / a.W;
    const int oh_lo = max(0, (ih - 1) * sy - 1), oh_hi = min(a.Ho - 1, (ih + 2) * sy);
    const int ow_lo = max(0, (iw - 1) * sx - 1), ow_hi = min(a.Wo - 1, (iw + 2) * sx);
    float acc = 0.0f;
    for (int oh = oh_lo; oh <= oh_hi; ++oh) {
      const Coord ch = rows[oh];
      const bool h0 = ch.lo == ih, h1 = ch.hi == ih;
      if (!h0 && !h1) continue;
      const float a_h = __fsub_rn(1.0f, ch.frac);
      for (int ow = ow_lo; ow <= ow_hi; ++ow) {
        const Coord cw = cols[ow];
        const bool w0 = cw.lo == iw, w1 = cw.hi == iw;
        if (!w0 && !w1) continue;
        const float g = sdy[((int64_t)oh * a.Wo + ow) * a.C + c];
        const float b_w = __fsub_rn(1.0f, cw.frac);
        if (h0 && w0) acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(a_h, b_w), g));
        if (h0 && w1) acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(a_h, cw.frac), g));
        if (h1 && w0) acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(ch.frac, b_w), g));
        if (h1 && w1) acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(ch.frac, cw.frac), g));
      }
    }
    out[e] = acc;
  }
}

__global__ void up_coords_kernel(int in, int out, int* lo, int* hi, float* frac) {
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= out) return;
  const Coord c = up_coord(o, in, out);
  lo[o] = c.lo;
  hi[o] = c.hi;
  frac[o] = c.frac;
}

int parse_size(const int32_t* size, int num_size, int* sy, int* sx) {
  B2_REQUIRE(size != nullptr && num_size == 2, "size must have exactly 2 elements");
  B2_REQUIRE(size[0] >= 1 && size[1] >= 1, "size elements must be >= 1");
  *sy = size[0];
  *sx = size[1];
  return B2_OK;
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" {

// src/ops/upsampling_ops.cc:99-156
int b2_upsampling_bilinear2d(b2_stream_t stream, const float* input, const int64_t input_shape[4],
                             const int32_t* size, int num_size, float* output) {
  clear_error();
  int sy = 1, sx = 1;
  B2_RETURN_IF_ERROR(parse_size(size, num_size, &sy, &sx));
  B2_REQUIRE(input_shape != nullptr, "input must be NHWC");
  for (int i = 0; i < 4; ++i) B2_REQUIRE(input_shape[i] >= 0, "input must be NHWC");
  UpArgs a;
  a.N = (int)input_shape[0]; a.H = (int)input_shape[1]; a.W = (int)input_shape[2]; a.C = (int)input_shape[3];
  a.Ho = a.H * sy;
  a.Wo = a.W * sx;
  const int64_t total = (int64_t)a.N * a.Ho * a.Wo * a.C;
  B2_REQUIRE(total <= kMaxInt32 && (int64_t)input_shape[0] * input_shape[1] * input_shape[2] * input_shape[3] <=
                                       kMaxInt32,
             "tensor too large for this op (more than 2^31 elements)");
  if (total == 0) return B2_OK;
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a.C % 4 == 0 && aligned16(input) && aligned16(output))
    up_fwd_kernel<4><<<grid_for(total / 4, kThreads, 8), kThreads, 0, s>>>(input, output, a);
  else
    up_fwd_kernel<1><<<grid_for(total, kThreads, 8), kThreads, 0, s>>>(input, output, a);
  return check_launch(s, "upsample_bilinear_forward");
}

// src/ops/upsampling_ops.cc:188-265
int b2_upsampling_bilinear2d_grad(b2_stream_t stream, const float* grad_out, const int64_t grad_out_shape[4],
                                  const int32_t input_sizes[4], const int32_t* size, int num_size,
                                  float* grad_in) {
  clear_error();
  int sy = 1, sx = 1;
  B2_RETURN_IF_ERROR(parse_size(size, num_size, &sy, &sx));
  B2_REQUIRE(input_sizes != nullptr, "input_sizes must have 4 elements [N,H,W,C]");
  UpArgs a;
  a.N = input_sizes[0]; a.H = input_sizes[1]; a.W = input_sizes[2]; a.C = input_sizes[3];
  B2_REQUIRE(a.N >= 0 && a.H >= 0 && a.W >= 0 && a.C >= 0, "input_sizes must be non-negative");
  a.Ho = a.H * sy;
  a.Wo = a.W * sx;
  B2_REQUIRE(grad_out_shape != nullptr && grad_out_shape[0] == a.N && grad_out_shape[1] == a.Ho &&
                 grad_out_shape[2] == a.Wo && grad_out_shape[3] == a.C,
             "grad_out shape mismatch with input_sizes + size");
  const int64_t in_total = (int64_t)a.N * a.H * a.W * a.C;
  const int64_t out_total = (int64_t)a.N * a.Ho * a.Wo * a.C;
  B2_REQUIRE(out_total <= kMaxInt32, "tensor too large for this op (more than 2^31 elements)");
  if (in_total == 0) return B2_OK;
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t staged_bytes = out_total / (a.N > 0 ? a.N : 1) * 4 + (int64_t)(a.Ho + a.Wo) * (int64_t)sizeof(Coord);
  if (staged_bytes <= kStagedSmemBytes) {
    const int64_t img = (int64_t)a.Ho * a.Wo * a.C;
    const int vec_copy = img % 4 == 0 && aligned16(grad_out);
    // the coordinate tables start after the image, on a 4-byte boundary
    up_bwd_staged_kernel<<<a.N, kThreads, (size_t)staged_bytes, s>>>(grad_out, grad_in, a, sy, sx, vec_copy);
  } else if (a.C % 4 == 0 && aligned16(grad_out) && aligned16(grad_in))
    up_bwd_kernel<4><<<grid_for(in_total / 4, kThreads, 8), kThreads, 0, s>>>(grad_out, grad_in, a, sy, sx);
  else
    up_bwd_kernel<1><<<grid_for(in_total, kThreads, 8), kThreads, 0, s>>>(grad_out, grad_in, a, sy, sx);
  return check_launch(s, "upsample_bilinear_backward");
}

int b2_upsampling_coords(b2_stream_t stream, int32_t in_size, int32_t out_size, int32_t* lo, int32_t* hi,
                         float* frac) {
  clear_error();
  B2_REQUIRE(in_size >= 1 && out_size >= 0, "in_size must be >= 1 and out_size >= 0");
  if (out_size == 0) return B2_OK;
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  up_coords_kernel<<<(out_size + 255) / 256, 256, 0, s>>>(in_size, out_size, lo, hi, frac);
  return check_launch(s, "upsample_coords");
}

}  // extern "C"
