// elementwise.cu -- ReLU, ReLU grad, Sigmoid, Sigmoid grad.
//
// Reference kernels: kernels/relu_kernels.cl:9-30, kernels/sigmoid_kernels.cl:
// 9-32 (one work-item per element, scalar loads).  Here: HBM-bound grid-stride
// kernels over 128-bit float4 loads (4 in flight per thread), a scalar tail,
// and a scalar path when a pointer is not 16-byte aligned.  Grids are sized
// to a multiple of the SM count.
//
// Exactness: every operation is written with the round-to-nearest intrinsics
// (no fused multiply-add contraction), so ReLU, ReLU grad and Sigmoid grad are
// bit-identical to the reference formula evaluated in IEEE fp32; Sigmoid's
// expf is CUDA's (within 2 ulp), the only inexact step.
#include "b2_internal.cuh"

namespace b2 {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

// y = fmax(x, 0): NaN -> 0 and -0 -> +0, as the reference's fmax gives on
// the host (relu_kernels.cl:16).
struct ReluF {
  __device__ __forceinline__ float operator()(float x) const { return x > 0.0f ? x : 0.0f; }
};
// backprops = features > 0 ? gradients : 0 (relu_kernels.cl:29)
struct ReluGradF {
  __device__ __forceinline__ float operator()(float g, float f) const { return f > 0.0f ? g : 0.0f; }
};
// 1 / (1 + exp(-x)) (sigmoid_kernels.cl:16)
struct SigmoidF {
  __device__ __forceinline__ float operator()(float x) const {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
  }
};
// dy * y * (1 - y), evaluated left to right (sigmoid_kernels.cl:30-31); the
// op's first input is y, its second dy.
struct SigmoidGradF {
  __device__ __forceinline__ float operator()(float y, float dy) const {
    return __fmul_rn(__fmul_rn(dy, y), __fsub_rn(1.0f, y));
  }
};

template <class F>
__device__ __forceinline__ float4 apply4(F f, float4 a) {
  return make_float4(f(a.x), f(a.y), f(a.z), f(a.w));
}
template <class F>
__device__ __forceinline__ float4 apply4(F f, float4 a, float4 b) {
  return make_float4(f(a.x, b.x), f(a.y, b.y), f(a.z, b.z), f(a.w, b.w));
}

template <class F>
__global__ void __launch_bounds__(kThreads) unary_vec_kernel(const float4* __restrict__ a, float4* __restrict__ out,
                                                              int64_t n4, F f) {
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  for (; i + (kUnroll - 1) * stride < n4; i += kUnroll * stride) {
    float4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) v[u] = a[i + u * stride];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) out[i + u * stride] = apply4(f, v[u]);
  }
  for (; i < n4; i += stride) out[i] = apply4(f, a[i]);
}

template <class F>
__global__ void __launch_bounds__(kThreads) binary_vec_kernel(const float4* __restrict__ a,
                                                               const float4* __restrict__ b,
                                                               float4* __restrict__ out, int64_t n4, F f) {
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  for (; i + (kUnroll - 1) * stride < n4; i += kUnroll * stride) {
    float4 va[kUnroll], vb[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      va[u] = a[i + u * stride];
      vb[u] = b[i + u * stride];
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) out[i + u * stride] = apply4(f, va[u], vb[u]);
  }
  for (; i < n4; i += stride) out[i] = apply4(f, a[i], b[i]);
}

template <class F>
__global__ void __launch_bounds__(kThreads) unary_scalar_kernel(const float* __restrict__ a, float* __restrict__ out,
                                                                int64_t begin, int64_t n, F f) {
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t i = begin + (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride) out[i] = f(a[i]);
}

template <class F>
__global__ void __launch_bounds__(kThreads) binary_scalar_kernel(const float* __restrict__ a,
                                                                 const float* __restrict__ b,
                                                                 float* __restrict__ out, int64_t begin, int64_t n,
                                                                 F f) {
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t i = begin + (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride)
    out[i] = f(a[i], b[i]);
}

template <class F>
int run_unary(b2_stream_t stream, const float* a, float* out, int64_t n, F f, const char* name) {
  clear_error();
  B2_REQUIRE(n >= 0, "%s: num_elements must be >= 0", name);
  if (n == 0) return B2_OK;  // src/ops/relu_ops.cc:67, sigmoid_ops.cc:74
  B2_REQUIRE(a != nullptr && out != nullptr, "%s: null tensor pointer", name);
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int64_t done = 0;
  if (aligned16(a) && aligned16(out) && n >= 4) {
    const int64_t n4 = n / 4;
    const int grid = grid_for(ceil_div(n4, kUnroll), kThreads, 8);
    unary_vec_kernel<<<grid, kThreads, 0, s>>>(reinterpret_cast<const float4*>(a), reinterpret_cast<float4*>(out),
                                                n4, f);
    B2_RETURN_IF_ERROR(check_launch(s, name));
    done = n4 * 4;
  }
  if (done < n) {
    unary_scalar_kernel<<<grid_for(n - done, kThreads, 8), kThreads, 0, s>>>(a, out, done, n, f);
    B2_RETURN_IF_ERROR(check_launch(s, name));
  }
  return B2_OK;
}

template <class F>
int run_binary(b2_stream_t stream, const float* a, const float* b, float* out, int64_t n, F f, const char* name) {
  clear_error();
  B2_REQUIRE(n >= 0, "%s: num_elements must be >= 0", name);
  if (n == 0) return B2_OK;
  B2_REQUIRE(a != nullptr && b != nullptr && out != nullptr, "%s: null tensor pointer", name);
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int64_t done = 0;
  if (aligned16(a) && aligned16(b) && aligned16(out) && n >= 4) {
    const int64_t n4 = n / 4;
    const int grid = grid_for(ceil_div(n4, kUnroll), kThreads, 8);
    binary_vec_kernel<<<grid, kThreads, 0, s>>>(reinterpret_cast<const float4*>(a),
                                                 reinterpret_cast<const float4*>(b), reinterpret_cast<float4*>(out),
                                                 n4, f);
    B2_RETURN_IF_ERROR(check_launch(s, name));
    done = n4 * 4;
  }
  if (done < n) {
    binary_scalar_kernel<<<grid_for(n - done, kThreads, 8), kThreads, 0, s>>>(a, b, out, done, n, f);
    B2_RETURN_IF_ERROR(check_launch(s, name));
  }
  return B2_OK;
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" {

int b2_relu(b2_stream_t stream, const float* input, float* output, int64_t num_elements) {
  return run_unary(stream, input, output, num_elements, ReluF{}, "relu_forward");
}

int b2_relu_grad(b2_stream_t stream, const float* gradients, const float* features, float* backprops,
                 int64_t num_elements) {
  return run_binary(stream, gradients, features, backprops, num_elements, ReluGradF{}, "relu_backward");
}

int b2_sigmoid(b2_stream_t stream, const float* input, float* output, int64_t num_elements) {
  return run_unary(stream, input, output, num_elements, SigmoidF{}, "sigmoid_forward");
}

int b2_sigmoid_grad(b2_stream_t stream, const float* y, const float* dy, float* grad_x, int64_t num_elements) {
  return run_binary(stream, y, dy, grad_x, num_elements, SigmoidGradF{}, "sigmoid_backward");
}

}  // extern "C"
