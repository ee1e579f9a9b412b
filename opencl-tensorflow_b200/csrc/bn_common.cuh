// bn_common.cuh -- BatchNorm arithmetic shared by the BatchNorm kernels and
// the kernels that fuse a BatchNorm gradient into their operand loads.
#pragma once

#include "b2_internal.cuh"

namespace b2 {

// y of the forward normalisation (batchnorm_kernels.cl:77-80), operation for
// operation, so a ReLU mask recomputed from it matches the forward's.
__device__ __forceinline__ float bn_y(float x, float m, float iv, float g, float b) {
  return __fadd_rn(__fmul_rn(g, __fmul_rn(__fsub_rn(x, m), iv)), b);
}

// One element of the BatchNorm input gradient (batchnorm_kernels.cl:135-142):
//   dx = k1 * (NHW * dy - grad_beta - x_hat * grad_gamma),
//   x_hat = (x - mean) * inv_std,  k1 = gamma * inv_std / NHW;
// RELU: dy = (y > 0 ? dz : 0), the gradient through a ReLU on the BN output y
// (recomputed from x as the forward computed it).  Every kernel that needs dx
// evaluates it here, so they agree bit for bit.
template <bool RELU>
__device__ __forceinline__ float bn_grad_dx_value(float x, float dz, float mean, float inv, float k1, float gbeta,
                                                  float ggamma, float gamma, float beta, float nhw_f) {
  const float xh = __fmul_rn(__fsub_rn(x, mean), inv);
  const float gv = RELU && !(__fadd_rn(__fmul_rn(gamma, xh), beta) > 0.0f) ? 0.0f : dz;
  float t = __fmul_rn(nhw_f, gv);
  t = __fsub_rn(t, gbeta);
  t = __fsub_rn(t, __fmul_rn(xh, ggamma));
  return __fmul_rn(k1, t);
}

// The reduction half of the BatchNorm(+ReLU) gradient (batchnorm.cu): fills
// grad_gamma, grad_beta and the per-channel constants of the dx formula, k1
// and inv_std (device arrays of C), for x / grad_y of `rows` x C.
int bn_grad_reduce(cudaStream_t s, const float* grad_y, const float* x, int64_t rows, int64_t C,
                   const float* gamma, const float* beta, const float* saved_mean, const float* saved_var,
                   float epsilon, bool relu, float* grad_gamma, float* grad_beta, float* k1, float* inv_std);

}  // namespace b2
