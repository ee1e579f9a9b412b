/* ref_driver.cc -- TEST INFRASTRUCTURE (oracle): host driver for the
 * reference's OWN kernel source.
 *
 * Built by oracle/Makefile into oracle/_ref/ from the reference checkout
 * (kernels/*.cl and src/padding_utils.h are compiled where they lie; nothing
 * of them is copied into this repository).  Each function below mirrors one
 * OpKernel::Compute of src/ops/*.cc: the same padding resolution
 * (src/padding_utils.h:22-33), the same kernel argument list, the same global
 * size RoundUp(total, 64) (src/cl_backend.h:96-98), the same multi-kernel
 * order (BN: reduce then normalize, src/ops/batchnorm_ops.cc:125-167,
 * 362-403) and the zero fill before the upsampling scatter
 * (src/ops/upsampling_ops.cc:251-256).  Work-items run as an OpenMP loop.
 */
#include "cl_shim.h"

#include <cstring>
#include <string>

#include <omp.h>

#include "padding_utils.h"  // reference: src/padding_utils.h

namespace clk {
thread_local size_t g_work_item_id = 0;
#include "batchnorm_kernels.cl"
#include "conv2d_kernels.cl"
#include "dense_kernels.cl"
#include "depthwise_conv2d_kernels.cl"
#include "relu_kernels.cl"
#include "sigmoid_kernels.cl"
#include "upsampling_bilinear_kernels.cl"
}  // namespace clk

#undef restrict
#undef __global
#undef __kernel

#define ORC_PREFIX ref_
#include "oracle_abi.h"

namespace {

constexpr size_t kLocal = 64;  // src/cl_backend.h:96 kDefaultLocalSize
int g_threads = 0;             // 0 = OpenMP default (all cores)

size_t RoundUp64(size_t n) { return ((n + kLocal - 1) / kLocal) * kLocal; }

/* One NDRange launch: work-items 0..RoundUp(total,64)-1, each calling `k`. */
template <class K>
void Launch(size_t total, K&& k) {
  const long global = static_cast<long>(RoundUp64(total));
  const int nt = g_threads > 0 ? g_threads : omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(nt)
  for (long g = 0; g < global; ++g) {
    clk::g_work_item_id = static_cast<size_t>(g);
    k();
  }
}

void Pad(int in, int k, int s, int same, int* out, int* pad) {
  opencl_tf::ResolvePadding(in, k, s, same ? std::string("SAME")
                                           : std::string("VALID"),
                            out, pad);
}

}  // namespace

extern "C" {

void ref_set_threads(int n) { g_threads = n; }
int ref_get_threads(void) {
  return g_threads > 0 ? g_threads : omp_get_max_threads();
}

int ref_resolve_padding(int in_size, int k, int stride, int same,
                        int* out_size, int* pad_before) {
  Pad(in_size, k, stride, same, out_size, pad_before);
  return 0;
}

/* src/ops/conv2d_ops.cc:107-190 */
int ref_conv2d(const float* x, const float* w, float* y, int N, int H, int W,
               int Ci, int kH, int kW, int Co, int sH, int sW, int same) {
  int Ho, Wo, pH, pW;
  Pad(H, kH, sH, same, &Ho, &pH);
  Pad(W, kW, sW, same, &Wo, &pW);
  Launch((size_t)N * Ho * Wo * Co, [&] {
    clk::conv2d_forward(x, w, y, N, H, W, Ci, kH, kW, Co, sH, sW, pH, pW, Ho,
                        Wo);
  });
  return 0;
}

/* src/ops/conv2d_ops.cc:225-314 */
int ref_conv2d_backprop_input(const float* dy, const float* w, float* dx,
                              int N, int H, int W, int Ci, int kH, int kW,
                              int Co, int sH, int sW, int same) {
  int Ho, Wo, pH, pW;
  Pad(H, kH, sH, same, &Ho, &pH);
  Pad(W, kW, sW, same, &Wo, &pW);
  Launch((size_t)N * H * W * Ci, [&] {
    clk::conv2d_backprop_input(dy, w, dx, N, H, W, Ci, kH, kW, Co, sH, sW, pH,
                               pW, Ho, Wo);
  });
  return 0;
}

/* src/ops/conv2d_ops.cc:350-440 */
int ref_conv2d_backprop_filter(const float* x, const float* dy, float* dw,
                               int N, int H, int W, int Ci, int kH, int kW,
                               int Co, int sH, int sW, int same) {
  int Ho, Wo, pH, pW;
  Pad(H, kH, sH, same, &Ho, &pH);
  Pad(W, kW, sW, same, &Wo, &pW);
  Launch((size_t)kH * kW * Ci * Co, [&] {
    clk::conv2d_backprop_filter(x, dy, dw, N, H, W, Ci, kH, kW, Co, sH, sW, pH,
                                pW, Ho, Wo);
  });
  return 0;
}

/* src/ops/depthwise_conv2d_ops.cc:107-187 */
int ref_depthwise_conv2d(const float* x, const float* w, float* y, int N,
                         int H, int W, int C, int kH, int kW, int dm, int sH,
                         int sW, int same) {
  int Ho, Wo, pH, pW;
  Pad(H, kH, sH, same, &Ho, &pH);
  Pad(W, kW, sW, same, &Wo, &pW);
  Launch((size_t)N * Ho * Wo * C * dm, [&] {
    clk::dwconv2d_forward(x, w, y, N, H, W, C, kH, kW, dm, sH, sW, pH, pW, Ho,
                          Wo);
  });
  return 0;
}

/* src/ops/depthwise_conv2d_ops.cc:221-305 */
int ref_depthwise_conv2d_backprop_input(const float* dy, const float* w,
                                        float* dx, int N, int H, int W, int C,
                                        int kH, int kW, int dm, int sH, int sW,
                                        int same) {
  int Ho, Wo, pH, pW;
  Pad(H, kH, sH, same, &Ho, &pH);
  Pad(W, kW, sW, same, &Wo, &pW);
  Launch((size_t)N * H * W * C, [&] {
    clk::dwconv2d_backprop_input(dy, w, dx, N, H, W, C, kH, kW, dm, sH, sW, pH,
                                 pW, Ho, Wo);
  });
  return 0;
}

/* src/ops/depthwise_conv2d_ops.cc:341-426 */
int ref_depthwise_conv2d_backprop_filter(const float* x, const float* dy,
                                         float* dw, int N, int H, int W,
                                         int C, int kH, int kW, int dm, int sH,
                                         int sW, int same) {
  int Ho, Wo, pH, pW;
  Pad(H, kH, sH, same, &Ho, &pH);
  Pad(W, kW, sW, same, &Wo, &pW);
  Launch((size_t)kH * kW * C * dm, [&] {
    clk::dwconv2d_backprop_filter(x, dy, dw, N, H, W, C, kH, kW, dm, sH, sW,
                                  pH, pW, Ho, Wo);
  });
  return 0;
}

/* src/ops/relu_ops.cc:56-90 */
int ref_relu(const float* x, float* y, long n) {
  if (n == 0) return 0;
  const int total = (int)n;
  Launch((size_t)n, [&] { clk::relu_forward(x, y, total); });
  return 0;
}

/* src/ops/relu_ops.cc:113-162 (gradients, features) */
int ref_relu_grad(const float* gradients, const float* features,
                  float* backprops, long n) {
  if (n == 0) return 0;
  const int total = (int)n;
  Launch((size_t)n,
         [&] { clk::relu_backward(gradients, features, backprops, total); });
  return 0;
}

/* src/ops/sigmoid_ops.cc:64-100 */
int ref_sigmoid(const float* x, float* y, long n) {
  if (n == 0) return 0;
  const int total = (int)n;
  Launch((size_t)n, [&] { clk::sigmoid_forward(x, y, total); });
  return 0;
}

/* src/ops/sigmoid_ops.cc:123-172: op inputs (y, dy); kernel args (dy, y, gx) */
int ref_sigmoid_grad(const float* y, const float* dy, float* grad_x, long n) {
  if (n == 0) return 0;
  const int total = (int)n;
  Launch((size_t)n, [&] { clk::sigmoid_backward(dy, y, grad_x, total); });
  return 0;
}

/* src/ops/batchnorm_ops.cc:87-180: bn_reduce_stats over C, then bn_normalize */
int ref_batch_norm_training(const float* x, const float* gamma,
                            const float* beta, float* y, float* saved_mean,
                            float* saved_var, int N, int H, int W, int C,
                            float epsilon) {
  Launch((size_t)C,
         [&] { clk::bn_reduce_stats(x, saved_mean, saved_var, N, H, W, C); });
  Launch((size_t)N * H * W * C, [&] {
    clk::bn_normalize(x, saved_mean, saved_var, gamma, beta, y, N, H, W, C,
                      epsilon);
  });
  return 0;
}

/* src/ops/batchnorm_ops.cc:213-275 */
int ref_batch_norm_inference(const float* x, const float* gamma,
                             const float* beta, const float* mean,
                             const float* var, float* y, int N, int H, int W,
                             int C, float epsilon) {
  Launch((size_t)N * H * W * C, [&] {
    clk::bn_normalize(x, mean, var, gamma, beta, y, N, H, W, C, epsilon);
  });
  return 0;
}

/* src/ops/batchnorm_ops.cc:313-416: bn_backward_reduce then bn_backward_dx */
int ref_batch_norm_grad(const float* grad_y, const float* x,
                        const float* gamma, const float* saved_mean,
                        const float* saved_var, float* grad_x,
                        float* grad_gamma, float* grad_beta, int N, int H,
                        int W, int C, float epsilon) {
  Launch((size_t)C, [&] {
    clk::bn_backward_reduce(grad_y, x, saved_mean, saved_var, grad_beta,
                            grad_gamma, N, H, W, C, epsilon);
  });
  Launch((size_t)N * H * W * C, [&] {
    clk::bn_backward_dx(grad_y, x, saved_mean, saved_var, gamma, grad_beta,
                        grad_gamma, grad_x, N, H, W, C, epsilon);
  });
  return 0;
}

/* src/ops/dense_ops.cc:77-143 */
int ref_dense(const float* x, const float* w, const float* b, float* y,
              int batch, int in_f, int out_f) {
  Launch((size_t)batch * out_f,
         [&] { clk::dense_forward(x, w, b, y, batch, in_f, out_f); });
  return 0;
}

/* src/ops/dense_ops.cc:170-227 */
int ref_dense_backprop_input(const float* grad_y, const float* w,
                             float* grad_x, int batch, int in_f, int out_f) {
  Launch((size_t)batch * in_f, [&] {
    clk::dense_backprop_input(grad_y, w, grad_x, batch, in_f, out_f);
  });
  return 0;
}

/* src/ops/dense_ops.cc:254-311 */
int ref_dense_backprop_weight(const float* x, const float* grad_y,
                              float* grad_w, int batch, int in_f, int out_f) {
  Launch((size_t)in_f * out_f, [&] {
    clk::dense_backprop_weight(x, grad_y, grad_w, batch, in_f, out_f);
  });
  return 0;
}

/* src/ops/dense_ops.cc:334-379 */
int ref_dense_backprop_bias(const float* grad_y, float* grad_b, int batch,
                            int out_f) {
  Launch((size_t)out_f,
         [&] { clk::dense_backprop_bias(grad_y, grad_b, batch, out_f); });
  return 0;
}

/* src/ops/upsampling_ops.cc:99-156 */
int ref_upsampling_bilinear2d(const float* x, float* y, int N, int H, int W,
                              int C, int sy, int sx) {
  const int Ho = H * sy, Wo = W * sx;
  const long total = (long)N * Ho * Wo * C;
  if (total == 0) return 0;
  Launch((size_t)total, [&] {
    clk::upsample_bilinear_forward(x, y, N, H, W, C, Ho, Wo);
  });
  return 0;
}

/* src/ops/upsampling_ops.cc:188-265: zero fill, then atomic scatter-add */
int ref_upsampling_bilinear2d_grad(const float* grad_out, float* grad_in,
                                   int N, int H, int W, int C, int sy,
                                   int sx) {
  const int Ho = H * sy, Wo = W * sx;
  const long total = (long)N * Ho * Wo * C;
  std::memset(grad_in, 0, sizeof(float) * (size_t)N * H * W * C);
  if (total == 0) return 0;
  Launch((size_t)total, [&] {
    clk::upsample_bilinear_backward(grad_out, grad_in, N, H, W, C, Ho, Wo);
  });
  return 0;
}

}  // extern "C"
