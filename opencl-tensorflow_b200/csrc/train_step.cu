// train_step.cu -- the training step's neighbours of the seven ops: the mean
// squared error loss (forward and gradient) and a multi-tensor Adam update.
//
// The reference trains its networks with
//   model.compile(optimizer=tf.keras.optimizers.Adam(1e-3), loss="mse")
// (README.md:188-196): both run as stock TensorFlow ops on the host (TF
// 2.10-2.15).  Here each is one kernel on the step's stream:
//
//  * mse_loss_kernel: a cluster of kLossCtas CTAs streams pred and target
//    once; each CTA reduces its share to one double in shared memory, and CTA
//    0 of the cluster adds the CTAs' values in rank order through distributed
//    shared memory -- deterministic, no scratch, no second launch.
//  * mse_grad_*_kernel: d pred = (pred - target) * (2 * dloss / n), dloss read
//    from device memory (the upstream gradient of the scalar loss).
//  * adam_kernel: Keras Adam's update (keras/optimizers/adam.py, TF 2.11+; the
//    same formula as the legacy ApplyAdam kernel of TF 2.10):
//        t      = iterations + 1
//        alpha  = lr * sqrt(1 - beta_2^t) / (1 - beta_1^t)
//        m     += (g - m) * (1 - beta_1)
//        v     += (g * g - v) * (1 - beta_2)
//        p     -= (m * alpha) / (sqrt(v) + epsilon)
//    for up to kAdamMaxTensors parameter tensors per launch, each CTA taking a
//    kAdamChunk-element chunk of one tensor.  `iterations` lives in device
//    memory so a captured CUDA graph replays correctly; every CTA reads it
//    first, and the CTA that takes the last ticket of a self-resetting
//    counter (all others have read it by then) stores t back.
//
// All arithmetic is written with round-to-nearest intrinsics in the order
// above (no contraction into fused multiply-adds); sqrt and division are the
// IEEE ones, beta^t is CUDA's powf.
#include <cooperative_groups.h>

#include "b2_internal.cuh"

namespace cg = cooperative_groups;

namespace b2 {
namespace {

constexpr int kLossCtas = 8;  // one portable cluster
constexpr int kLossThreads = 512;
constexpr int kLossWarps = kLossThreads / 32;

__device__ __forceinline__ float sq_diff(float p, float t) {
  const float d = __fsub_rn(p, t);
  return __fmul_rn(d, d);
}

template <bool kVec>
__global__ void __cluster_dims__(kLossCtas, 1, 1) __launch_bounds__(kLossThreads)
    mse_loss_kernel(const float* __restrict__ pred, const float* __restrict__ target, int64_t n,
                    float* __restrict__ loss) {
  __shared__ double warp_sum[kLossWarps];
  __shared__ double cta_sum;
  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x;
  const int64_t stride = (int64_t)kLossCtas * kLossThreads;
  const int64_t first = (int64_t)blockIdx.x * kLossThreads + tid;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  int64_t tail = 0;
  if (kVec) {
    const float4* p4 = reinterpret_cast<const float4*>(pred);
    const float4* t4 = reinterpret_cast<const float4*>(target);
    const int64_t n4 = n / 4;
    int64_t i = first;
    for (; i + stride < n4; i += 2 * stride) {  // two float4 pairs in flight
      const float4 a0 = p4[i], b0 = t4[i], a1 = p4[i + stride], b1 = t4[i + stride];
      acc[0] = __fadd_rn(acc[0], __fadd_rn(sq_diff(a0.x, b0.x), sq_diff(a1.x, b1.x)));
      acc[1] = __fadd_rn(acc[1], __fadd_rn(sq_diff(a0.y, b0.y), sq_diff(a1.y, b1.y)));
      acc[2] = __fadd_rn(acc[2], __fadd_rn(sq_diff(a0.z, b0.z), sq_diff(a1.z, b1.z)));
      acc[3] = __fadd_rn(acc[3], __fadd_rn(sq_diff(a0.w, b0.w), sq_diff(a1.w, b1.w)));
    }
    if (i < n4) {
      const float4 a = p4[i], b = t4[i];
      acc[0] = __fadd_rn(acc[0], sq_diff(a.x, b.x));
      acc[1] = __fadd_rn(acc[1], sq_diff(a.y, b.y));
      acc[2] = __fadd_rn(acc[2], sq_diff(a.z, b.z));
      acc[3] = __fadd_rn(acc[3], sq_diff(a.w, b.w));
    }
    tail = n4 * 4;
  }
  for (int64_t i = tail + first; i < n; i += stride) acc[0] = __fadd_rn(acc[0], sq_diff(pred[i], target[i]));
  double s = ((double)acc[0] + (double)acc[1]) + ((double)acc[2] + (double)acc[3]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((tid & 31) == 0) warp_sum[tid >> 5] = s;
  __syncthreads();
  if (tid == 0) {
    double c = 0.0;
    for (int w = 0; w < kLossWarps; ++w) c += warp_sum[w];
    cta_sum = c;
  }
  cluster.sync();  // every CTA's cta_sum is written
  if (cluster.block_rank() == 0 && tid == 0) {
    double total = 0.0;
    for (int r = 0; r < kLossCtas; ++r) total += *cluster.map_shared_rank(&cta_sum, r);
    *loss = (float)(total / (double)n);
  }
  cluster.sync();  // keep every CTA's shared memory alive until CTA 0 has read it
}

constexpr int kGradThreads = 256;

__global__ void __launch_bounds__(kGradThreads)
    mse_grad_vec_kernel(const float4* __restrict__ pred, const float4* __restrict__ target,
                        const float* __restrict__ dloss, float inv_n, float4* __restrict__ out, int64_t n4) {
  const float scale = __fmul_rn(__fmul_rn(2.0f, *dloss), inv_n);
  const int64_t stride = (int64_t)gridDim.x * kGradThreads;
  for (int64_t i = (int64_t)blockIdx.x * kGradThreads + threadIdx.x; i < n4; i += stride) {
    const float4 a = pred[i], b = target[i];
    out[i] = make_float4(__fmul_rn(__fsub_rn(a.x, b.x), scale), __fmul_rn(__fsub_rn(a.y, b.y), scale),
                         __fmul_rn(__fsub_rn(a.z, b.z), scale), __fmul_rn(__fsub_rn(a.w, b.w), scale));
  }
}

__global__ void __launch_bounds__(kGradThreads)
    mse_grad_scalar_kernel(const float* __restrict__ pred, const float* __restrict__ target,
                           const float* __restrict__ dloss, float inv_n, float* __restrict__ out, int64_t begin,
                           int64_t n) {
  const float scale = __fmul_rn(__fmul_rn(2.0f, *dloss), inv_n);
  const int64_t stride = (int64_t)gridDim.x * kGradThreads;
  for (int64_t i = begin + (int64_t)blockIdx.x * kGradThreads + threadIdx.x; i < n; i += stride)
    out[i] = __fmul_rn(__fsub_rn(pred[i], target[i]), scale);
}

// ------------------------------------------------------------------- Adam

constexpr int kAdamMaxTensors = 24;
constexpr int kAdamThreads = 256;
constexpr int kAdamPerThread = 8;  // two float4 of each operand
constexpr int64_t kAdamChunk = (int64_t)kAdamThreads * kAdamPerThread;

struct AdamTensors {
  float* p[kAdamMaxTensors];
  const float* g[kAdamMaxTensors];
  float* m[kAdamMaxTensors];
  float* v[kAdamMaxTensors];
  int64_t size[kAdamMaxTensors];
  int64_t chunk0[kAdamMaxTensors + 1];  // first CTA of tensor i; chunk0[n] = grid
  uint32_t vec_mask;                    // bit i: tensor i's four pointers are 16-byte aligned
  int n;
};

struct AdamHyper {
  float lr, beta_1, beta_2, epsilon, one_minus_beta_1, one_minus_beta_2;
};

struct AdamScalars {
  float alpha, epsilon, one_minus_beta_1, one_minus_beta_2;
};

__device__ __forceinline__ void adam_one(float& p, float g, float& m, float& v, const AdamScalars& s) {
  m = __fadd_rn(m, __fmul_rn(__fsub_rn(g, m), s.one_minus_beta_1));
  v = __fadd_rn(v, __fmul_rn(__fsub_rn(__fmul_rn(g, g), v), s.one_minus_beta_2));
  p = __fsub_rn(p, __fdiv_rn(__fmul_rn(m, s.alpha), __fadd_rn(__fsqrt_rn(v), s.epsilon)));
}

__global__ void __launch_bounds__(kAdamThreads)
    adam_kernel(const __grid_constant__ AdamTensors T, const AdamHyper h, int64_t* __restrict__ iterations,
                unsigned int* __restrict__ ticket, int advance) {
  __shared__ int64_t step_s;
  if (threadIdx.x == 0) step_s = *reinterpret_cast<volatile int64_t*>(iterations) + 1;
  __syncthreads();
  const int64_t step = step_s;
  int ti = 0;
  while (ti + 1 < T.n && T.chunk0[ti + 1] <= (int64_t)blockIdx.x) ++ti;
  const float t = (float)step;
  const float b1p = powf(h.beta_1, t), b2p = powf(h.beta_2, t);
  AdamScalars s;
  s.alpha = __fdiv_rn(__fmul_rn(h.lr, __fsqrt_rn(__fsub_rn(1.0f, b2p))), __fsub_rn(1.0f, b1p));
  s.epsilon = h.epsilon;
  s.one_minus_beta_1 = h.one_minus_beta_1;
  s.one_minus_beta_2 = h.one_minus_beta_2;

  const int64_t base = ((int64_t)blockIdx.x - T.chunk0[ti]) * kAdamChunk;
  const int64_t size = T.size[ti];
  float* __restrict__ P = T.p[ti];
  const float* __restrict__ G = T.g[ti];
  float* __restrict__ M = T.m[ti];
  float* __restrict__ V = T.v[ti];
  if (((T.vec_mask >> ti) & 1u) && base + kAdamChunk <= size) {
    float4 p4[2], g4[2], m4[2], v4[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int64_t e = base + 4 * ((int64_t)u * kAdamThreads + threadIdx.x);
      p4[u] = *reinterpret_cast<const float4*>(P + e);
      g4[u] = *reinterpret_cast<const float4*>(G + e);
      m4[u] = *reinterpret_cast<const float4*>(M + e);
      v4[u] = *reinterpret_cast<const float4*>(V + e);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      adam_one(p4[u].x, g4[u].x, m4[u].x, v4[u].x, s);
      adam_one(p4[u].y, g4[u].y, m4[u].y, v4[u].y, s);
      adam_one(p4[u].z, g4[u].z, m4[u].z, v4[u].z, s);
      adam_one(p4[u].w, g4[u].w, m4[u].w, v4[u].w, s);
      const int64_t e = base + 4 * ((int64_t)u * kAdamThreads + threadIdx.x);
      *reinterpret_cast<float4*>(P + e) = p4[u];
      *reinterpret_cast<float4*>(M + e) = m4[u];
      *reinterpret_cast<float4*>(V + e) = v4[u];
    }
  } else {
    const int64_t end = base + kAdamChunk < size ? base + kAdamChunk : size;
    for (int64_t e = base + threadIdx.x; e < end; e += kAdamThreads) {
      float p = P[e], m = M[e], v = V[e];
      adam_one(p, G[e], m, v, s);
      P[e] = p;
      M[e] = m;
      V[e] = v;
    }
  }
  if (!advance) return;
  // The CTA holding the last ticket knows every CTA has read `iterations`.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(ticket, 1u) == gridDim.x - 1) {
      *iterations = step;
      *ticket = 0u;
      __threadfence();
    }
  }
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" {

int b2_mse_loss(b2_stream_t stream, const float* pred, const float* target, int64_t num_elements, float* loss) {
  clear_error();
  B2_REQUIRE(num_elements > 0, "mse_loss: num_elements must be > 0 (the mean of nothing is undefined)");
  B2_REQUIRE(pred != nullptr && target != nullptr && loss != nullptr, "mse_loss: null pointer");
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (aligned16(pred) && aligned16(target))
    mse_loss_kernel<true><<<kLossCtas, kLossThreads, 0, s>>>(pred, target, num_elements, loss);
  else
    mse_loss_kernel<false><<<kLossCtas, kLossThreads, 0, s>>>(pred, target, num_elements, loss);
  return check_launch(s, "mse_loss");
}

int b2_mse_loss_grad(b2_stream_t stream, const float* pred, const float* target, int64_t num_elements,
                     const float* grad_loss, float* grad_pred) {
  clear_error();
  B2_REQUIRE(num_elements > 0, "mse_loss_grad: num_elements must be > 0");
  B2_REQUIRE(pred != nullptr && target != nullptr && grad_loss != nullptr && grad_pred != nullptr,
             "mse_loss_grad: null pointer");
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const float inv_n = (float)(1.0 / (double)num_elements);
  int64_t done = 0;
  if (aligned16(pred) && aligned16(target) && aligned16(grad_pred) && num_elements >= 4) {
    const int64_t n4 = num_elements / 4;
    mse_grad_vec_kernel<<<grid_for(n4, kGradThreads, 8), kGradThreads, 0, s>>>(
        reinterpret_cast<const float4*>(pred), reinterpret_cast<const float4*>(target), grad_loss, inv_n,
        reinterpret_cast<float4*>(grad_pred), n4);
    B2_RETURN_IF_ERROR(check_launch(s, "mse_loss_grad"));
    done = n4 * 4;
  }
  if (done < num_elements) {
    mse_grad_scalar_kernel<<<grid_for(num_elements - done, kGradThreads, 8), kGradThreads, 0, s>>>(
        pred, target, grad_loss, inv_n, grad_pred, done, num_elements);
    B2_RETURN_IF_ERROR(check_launch(s, "mse_loss_grad"));
  }
  return B2_OK;
}

int b2_adam_update(b2_stream_t stream, int num_tensors, float* const* params, const float* const* grads,
                   float* const* m, float* const* v, const int64_t* sizes, float learning_rate, float beta_1,
                   float beta_2, float one_minus_beta_1, float one_minus_beta_2, float epsilon,
                   int64_t* iterations, unsigned int* ticket) {
  clear_error();
  B2_REQUIRE(num_tensors >= 0, "adam_update: num_tensors must be >= 0");
  if (num_tensors == 0) return B2_OK;
  B2_REQUIRE(params && grads && m && v && sizes && iterations && ticket, "adam_update: null pointer");
  for (int i = 0; i < num_tensors; ++i) {
    B2_REQUIRE(sizes[i] >= 0, "adam_update: tensor %d has a negative size", i);
    B2_REQUIRE(sizes[i] == 0 || (params[i] && grads[i] && m[i] && v[i]), "adam_update: tensor %d has a null pointer",
               i);
  }
  const DeviceInfo* d = nullptr;
  B2_RETURN_IF_ERROR(device_info(&d));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  AdamHyper h;
  h.lr = learning_rate;
  h.beta_1 = beta_1;
  h.beta_2 = beta_2;
  h.epsilon = epsilon;
  h.one_minus_beta_1 = one_minus_beta_1;
  h.one_minus_beta_2 = one_minus_beta_2;
  // Launches of up to kAdamMaxTensors non-empty tensors each; all read the
  // same `iterations`, the last one advances it.  With every tensor empty
  // nothing is launched and `iterations` stays.
  int nonempty = 0;
  for (int i = 0; i < num_tensors; ++i) nonempty += sizes[i] > 0;
  int i = 0, seen = 0;
  while (seen < nonempty) {
    AdamTensors T{};
    int64_t grid = 0;
    for (; i < num_tensors && T.n < kAdamMaxTensors; ++i) {
      if (sizes[i] == 0) continue;
      const int k = T.n++;
      T.p[k] = params[i];
      T.g[k] = grads[i];
      T.m[k] = m[i];
      T.v[k] = v[i];
      T.size[k] = sizes[i];
      T.chunk0[k] = grid;
      if (aligned16(params[i]) && aligned16(grads[i]) && aligned16(m[i]) && aligned16(v[i])) T.vec_mask |= 1u << k;
      grid += ceil_div(sizes[i], kAdamChunk);
    }
    seen += T.n;
    B2_REQUIRE(grid <= kMaxInt32, "adam_update: too many elements in one launch");
    T.chunk0[T.n] = grid;
    adam_kernel<<<(unsigned)grid, kAdamThreads, 0, s>>>(T, h, iterations, ticket, seen == nonempty ? 1 : 0);
    B2_RETURN_IF_ERROR(check_launch(s, "adam_update"));
  }
  return B2_OK;
}

}  // extern "C"
