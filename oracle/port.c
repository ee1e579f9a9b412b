/* port.c -- TEST INFRASTRUCTURE (oracle): plain-C restatement of the
 * reference's arithmetic for the seven ops (amanzargari/OpenCL-Tensorflow
 * 0.3.0, kernels/*.cl + src/ops/*.cc).  Never linked into the product.
 *
 * Each function states the reference lines it follows.  The per-output
 * accumulation order is the reference's (sequential fp32, loops nested the
 * same way), so with -ffp-contract=off this library reproduces
 * oracle/_ref/libref_ocl.so bit for bit; the tests pin that.  Indices are
 * 64-bit here (the reference uses int), which changes no value.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <omp.h>

#define ORC_PREFIX port_
#include "oracle_abi.h"

static int g_threads = 0;

static int nthreads(void) {
  return g_threads > 0 ? g_threads : omp_get_max_threads();
}

void port_set_threads(int n) { g_threads = n; }
int port_get_threads(void) { return nthreads(); }

/* src/padding_utils.h:22-33 -- TF SAME/VALID output size and top/left pad. */
int port_resolve_padding(int in_size, int k, int stride, int same,
                         int* out_size, int* pad_before) {
  if (same) {
    int out = (in_size + stride - 1) / stride;
    int total = (out - 1) * stride + k - in_size;
    if (total < 0) total = 0;
    *out_size = out;
    *pad_before = total / 2;
  } else {
    *out_size = (in_size - k + stride) / stride;
    *pad_before = 0;
  }
  return 0;
}

/* ---------------------------------------------------------------- conv2d */

/* kernels/conv2d_kernels.cl:30-70: y = sum over (kh, kw, ci) in that nesting,
 * taps outside the image skipped. */
int port_conv2d(const float* x, const float* w, float* y, int N, int H, int W,
                int Ci, int kH, int kW, int Co, int sH, int sW, int same) {
  int Ho, Wo, pH, pW;
  port_resolve_padding(H, kH, sH, same, &Ho, &pH);
  port_resolve_padding(W, kW, sW, same, &Wo, &pW);
  const int64_t total = (int64_t)N * Ho * Wo * Co;
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t g = 0; g < total; ++g) {
    const int co = (int)(g % Co);
    const int wo = (int)((g / Co) % Wo);
    const int ho = (int)((g / ((int64_t)Co * Wo)) % Ho);
    const int64_t n = g / ((int64_t)Co * Wo * Ho);
    float acc = 0.0f;
    for (int kh = 0; kh < kH; ++kh) {
      const int hi = ho * sH - pH + kh;
      if (hi < 0 || hi >= H) continue;
      for (int kw = 0; kw < kW; ++kw) {
        const int wi = wo * sW - pW + kw;
        if (wi < 0 || wi >= W) continue;
        const float* xp = x + ((n * H + hi) * W + wi) * Ci;
        const float* wp = w + ((int64_t)(kh * kW + kw) * Ci) * Co + co;
        for (int ci = 0; ci < Ci; ++ci) acc += xp[ci] * wp[(int64_t)ci * Co];
      }
    }
    y[g] = acc;
  }
  return 0;
}

/* kernels/conv2d_kernels.cl:73-120: gather form; a tap contributes when
 * (hi + pH - kh) is a non-negative multiple of sH below Ho (same for w). */
int port_conv2d_backprop_input(const float* dy, const float* w, float* dx,
                               int N, int H, int W, int Ci, int kH, int kW,
                               int Co, int sH, int sW, int same) {
  int Ho, Wo, pH, pW;
  port_resolve_padding(H, kH, sH, same, &Ho, &pH);
  port_resolve_padding(W, kW, sW, same, &Wo, &pW);
  const int64_t total = (int64_t)N * H * W * Ci;
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t g = 0; g < total; ++g) {
    const int ci = (int)(g % Ci);
    const int wi = (int)((g / Ci) % W);
    const int hi = (int)((g / ((int64_t)Ci * W)) % H);
    const int64_t n = g / ((int64_t)Ci * W * H);
    float acc = 0.0f;
    for (int kh = 0; kh < kH; ++kh) {
      const int hn = hi + pH - kh;
      if (hn < 0 || hn % sH != 0) continue;
      const int ho = hn / sH;
      if (ho >= Ho) continue;
      for (int kw = 0; kw < kW; ++kw) {
        const int wn = wi + pW - kw;
        if (wn < 0 || wn % sW != 0) continue;
        const int wo = wn / sW;
        if (wo >= Wo) continue;
        const float* gp = dy + ((n * Ho + ho) * Wo + wo) * Co;
        const float* wp = w + ((int64_t)(kh * kW + kw) * Ci + ci) * Co;
        for (int co = 0; co < Co; ++co) acc += gp[co] * wp[co];
      }
    }
    dx[g] = acc;
  }
  return 0;
}

/* kernels/conv2d_kernels.cl:123-158: dw[kh,kw,ci,co] = sum over (n, ho, wo)
 * in that nesting. */
int port_conv2d_backprop_filter(const float* x, const float* dy, float* dw,
                                int N, int H, int W, int Ci, int kH, int kW,
                                int Co, int sH, int sW, int same) {
  int Ho, Wo, pH, pW;
  port_resolve_padding(H, kH, sH, same, &Ho, &pH);
  port_resolve_padding(W, kW, sW, same, &Wo, &pW);
  const int64_t total = (int64_t)kH * kW * Ci * Co;
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t g = 0; g < total; ++g) {
    const int co = (int)(g % Co);
    const int ci = (int)((g / Co) % Ci);
    const int kw = (int)((g / ((int64_t)Co * Ci)) % kW);
    const int kh = (int)(g / ((int64_t)Co * Ci * kW));
    float acc = 0.0f;
    for (int64_t n = 0; n < N; ++n) {
      for (int ho = 0; ho < Ho; ++ho) {
        const int hi = ho * sH - pH + kh;
        if (hi < 0 || hi >= H) continue;
        for (int wo = 0; wo < Wo; ++wo) {
          const int wi = wo * sW - pW + kw;
          if (wi < 0 || wi >= W) continue;
          acc += x[((n * H + hi) * W + wi) * Ci + ci] *
                 dy[((n * Ho + ho) * Wo + wo) * Co + co];
        }
      }
    }
    dw[g] = acc;
  }
  return 0;
}

/* ------------------------------------------------------- depthwise conv */

/* kernels/depthwise_conv2d_kernels.cl:16-56: output channel co = ci*dm + d,
 * sum over (kh, kw). */
int port_depthwise_conv2d(const float* x, const float* w, float* y, int N,
                          int H, int W, int C, int kH, int kW, int dm, int sH,
                          int sW, int same) {
  int Ho, Wo, pH, pW;
  port_resolve_padding(H, kH, sH, same, &Ho, &pH);
  port_resolve_padding(W, kW, sW, same, &Wo, &pW);
  const int Co = C * dm;
  const int64_t total = (int64_t)N * Ho * Wo * Co;
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t g = 0; g < total; ++g) {
    const int co = (int)(g % Co);
    const int wo = (int)((g / Co) % Wo);
    const int ho = (int)((g / ((int64_t)Co * Wo)) % Ho);
    const int64_t n = g / ((int64_t)Co * Wo * Ho);
    const int ci = co / dm, d = co % dm;
    float acc = 0.0f;
    for (int kh = 0; kh < kH; ++kh) {
      const int hi = ho * sH - pH + kh;
      if (hi < 0 || hi >= H) continue;
      for (int kw = 0; kw < kW; ++kw) {
        const int wi = wo * sW - pW + kw;
        if (wi < 0 || wi >= W) continue;
        acc += x[((n * H + hi) * W + wi) * C + ci] *
               w[((int64_t)(kh * kW + kw) * C + ci) * dm + d];
      }
    }
    y[g] = acc;
  }
  return 0;
}

/* kernels/depthwise_conv2d_kernels.cl:59-104: gather over taps, then d. */
int port_depthwise_conv2d_backprop_input(const float* dy, const float* w,
                                         float* dx, int N, int H, int W, int C,
                                         int kH, int kW, int dm, int sH, int sW,
                                         int same) {
  int Ho, Wo, pH, pW;
  port_resolve_padding(H, kH, sH, same, &Ho, &pH);
  port_resolve_padding(W, kW, sW, same, &Wo, &pW);
  const int Co = C * dm;
  const int64_t total = (int64_t)N * H * W * C;
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t g = 0; g < total; ++g) {
    const int ci = (int)(g % C);
    const int wi = (int)((g / C) % W);
    const int hi = (int)((g / ((int64_t)C * W)) % H);
    const int64_t n = g / ((int64_t)C * W * H);
    float acc = 0.0f;
    for (int kh = 0; kh < kH; ++kh) {
      const int hn = hi + pH - kh;
      if (hn < 0 || hn % sH != 0) continue;
      const int ho = hn / sH;
      if (ho >= Ho) continue;
      for (int kw = 0; kw < kW; ++kw) {
        const int wn = wi + pW - kw;
        if (wn < 0 || wn % sW != 0) continue;
        const int wo = wn / sW;
        if (wo >= Wo) continue;
        const float* gp = dy + ((n * Ho + ho) * Wo + wo) * Co + (int64_t)ci * dm;
        const float* wp = w + ((int64_t)(kh * kW + kw) * C + ci) * dm;
        for (int d = 0; d < dm; ++d) acc += gp[d] * wp[d];
      }
    }
    dx[g] = acc;
  }
  return 0;
}

/* kernels/depthwise_conv2d_kernels.cl:107-145: sum over (n, ho, wo). */
int port_depthwise_conv2d_backprop_filter(const float* x, const float* dy,
                                          float* dw, int N, int H, int W,
                                          int C, int kH, int kW, int dm,
                                          int sH, int sW, int same) {
  int Ho, Wo, pH, pW;
  port_resolve_padding(H, kH, sH, same, &Ho, &pH);
  port_resolve_padding(W, kW, sW, same, &Wo, &pW);
  const int Co = C * dm;
  const int64_t total = (int64_t)kH * kW * C * dm;
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t g = 0; g < total; ++g) {
    const int d = (int)(g % dm);
    const int ci = (int)((g / dm) % C);
    const int kw = (int)((g / ((int64_t)dm * C)) % kW);
    const int kh = (int)(g / ((int64_t)dm * C * kW));
    const int co = ci * dm + d;
    float acc = 0.0f;
    for (int64_t n = 0; n < N; ++n) {
      for (int ho = 0; ho < Ho; ++ho) {
        const int hi = ho * sH - pH + kh;
        if (hi < 0 || hi >= H) continue;
        for (int wo = 0; wo < Wo; ++wo) {
          const int wi = wo * sW - pW + kw;
          if (wi < 0 || wi >= W) continue;
          acc += x[((n * H + hi) * W + wi) * C + ci] *
                 dy[((n * Ho + ho) * Wo + wo) * Co + co];
        }
      }
    }
    dw[g] = acc;
  }
  return 0;
}

/* ------------------------------------------------------ elementwise ops */

/* kernels/relu_kernels.cl:9-17: fmax(x, 0) (a NaN input gives 0). */
int port_relu(const float* x, float* y, long n) {
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (long i = 0; i < n; ++i) y[i] = fmaxf(x[i], 0.0f);
  return 0;
}

/* kernels/relu_kernels.cl:21-30: mask from the forward input; x == 0 -> 0. */
int port_relu_grad(const float* gradients, const float* features,
                   float* backprops, long n) {
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (long i = 0; i < n; ++i)
    backprops[i] = (features[i] > 0.0f) ? gradients[i] : 0.0f;
  return 0;
}

/* kernels/sigmoid_kernels.cl:9-17 */
int port_sigmoid(const float* x, float* y, long n) {
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (long i = 0; i < n; ++i) y[i] = 1.0f / (1.0f + expf(-x[i]));
  return 0;
}

/* kernels/sigmoid_kernels.cl:22-32: dy * y * (1 - y) from the forward output. */
int port_sigmoid_grad(const float* y, const float* dy, float* grad_x, long n) {
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (long i = 0; i < n; ++i) {
    const float yi = y[i];
    grad_x[i] = dy[i] * yi * (1.0f - yi);
  }
  return 0;
}

/* ------------------------------------------------------------ batchnorm */

/* kernels/batchnorm_kernels.cl:35-60: per-channel sequential sum and sum of
 * squares over (n, h, w); biased var = E[x^2] - mean^2. */
static void bn_stats(const float* x, float* mean, float* var, int64_t NHW,
                     int C) {
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int c = 0; c < C; ++c) {
    float sum = 0.0f, sumsq = 0.0f;
    for (int64_t r = 0; r < NHW; ++r) {
      const float v = x[r * C + c];
      sum += v;
      sumsq += v * v;
    }
    const float m = sum / (float)NHW;
    mean[c] = m;
    var[c] = sumsq / (float)NHW - m * m;
  }
}

/* kernels/batchnorm_kernels.cl:63-81 */
static void bn_normalize(const float* x, const float* mean, const float* var,
                         const float* gamma, const float* beta, float* y,
                         int64_t total, int C, float eps) {
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t g = 0; g < total; ++g) {
    const int c = (int)(g % C);
    const float inv_std = 1.0f / sqrtf(var[c] + eps);
    const float x_hat = (x[g] - mean[c]) * inv_std;
    y[g] = gamma[c] * x_hat + beta[c];
  }
}

/* src/ops/batchnorm_ops.cc:87-180 */
int port_batch_norm_training(const float* x, const float* gamma,
                             const float* beta, float* y, float* saved_mean,
                             float* saved_var, int N, int H, int W, int C,
                             float epsilon) {
  const int64_t NHW = (int64_t)N * H * W;
  bn_stats(x, saved_mean, saved_var, NHW, C);
  bn_normalize(x, saved_mean, saved_var, gamma, beta, y, NHW * C, C, epsilon);
  return 0;
}

/* src/ops/batchnorm_ops.cc:213-275 */
int port_batch_norm_inference(const float* x, const float* gamma,
                              const float* beta, const float* mean,
                              const float* var, float* y, int N, int H, int W,
                              int C, float epsilon) {
  bn_normalize(x, mean, var, gamma, beta, y, (int64_t)N * H * W * C, C,
               epsilon);
  return 0;
}

/* kernels/batchnorm_kernels.cl:84-143 + src/ops/batchnorm_ops.cc:313-416:
 * dbeta = sum dy, dgamma = sum dy*x_hat (sequential), then
 * dx = (gamma*inv_std/NHW) * (NHW*dy - dbeta - x_hat*dgamma). */
int port_batch_norm_grad(const float* grad_y, const float* x,
                         const float* gamma, const float* saved_mean,
                         const float* saved_var, float* grad_x,
                         float* grad_gamma, float* grad_beta, int N, int H,
                         int W, int C, float epsilon) {
  const int64_t NHW = (int64_t)N * H * W;
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int c = 0; c < C; ++c) {
    const float inv_std = 1.0f / sqrtf(saved_var[c] + epsilon);
    const float m = saved_mean[c];
    float s_dy = 0.0f, s_dy_xh = 0.0f;
    for (int64_t r = 0; r < NHW; ++r) {
      const float dy = grad_y[r * C + c];
      const float xh = (x[r * C + c] - m) * inv_std;
      s_dy += dy;
      s_dy_xh += dy * xh;
    }
    grad_beta[c] = s_dy;
    grad_gamma[c] = s_dy_xh;
  }
  const int64_t total = NHW * C;
  /* the reference computes (float)(N*H*W) in int arithmetic */
  const float nhw_f = (float)(int)(N * H * W);
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t g = 0; g < total; ++g) {
    const int c = (int)(g % C);
    const float inv_std = 1.0f / sqrtf(saved_var[c] + epsilon);
    const float xh = (x[g] - saved_mean[c]) * inv_std;
    const float dy = grad_y[g];
    grad_x[g] = (gamma[c] * inv_std / nhw_f) *
                (nhw_f * dy - grad_beta[c] - xh * grad_gamma[c]);
  }
  return 0;
}

/* ---------------------------------------------------------------- dense */

/* kernels/dense_kernels.cl:18-38: the bias seeds the accumulator. */
int port_dense(const float* x, const float* w, const float* b, float* y,
               int batch, int in_f, int out_f) {
  const int64_t total = (int64_t)batch * out_f;
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t g = 0; g < total; ++g) {
    const int64_t n = g / out_f;
    const int o = (int)(g % out_f);
    float acc = b[o];
    for (int64_t i = 0; i < in_f; ++i) acc += x[n * in_f + i] * w[i * out_f + o];
    y[g] = acc;
  }
  return 0;
}

/* kernels/dense_kernels.cl:42-61 */
int port_dense_backprop_input(const float* grad_y, const float* w,
                              float* grad_x, int batch, int in_f, int out_f) {
  const int64_t total = (int64_t)batch * in_f;
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t g = 0; g < total; ++g) {
    const int64_t n = g / in_f;
    const int64_t i = g % in_f;
    float acc = 0.0f;
    for (int o = 0; o < out_f; ++o)
      acc += grad_y[n * out_f + o] * w[i * out_f + o];
    grad_x[g] = acc;
  }
  return 0;
}

/* kernels/dense_kernels.cl:65-84 */
int port_dense_backprop_weight(const float* x, const float* grad_y,
                               float* grad_w, int batch, int in_f, int out_f) {
  const int64_t total = (int64_t)in_f * out_f;
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t g = 0; g < total; ++g) {
    const int64_t i = g / out_f;
    const int64_t o = g % out_f;
    float acc = 0.0f;
    for (int64_t n = 0; n < batch; ++n)
      acc += x[n * in_f + i] * grad_y[n * out_f + o];
    grad_w[g] = acc;
  }
  return 0;
}

/* kernels/dense_kernels.cl:88-102 */
int port_dense_backprop_bias(const float* grad_y, float* grad_b, int batch,
                             int out_f) {
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int o = 0; o < out_f; ++o) {
    float acc = 0.0f;
    for (int64_t n = 0; n < batch; ++n) acc += grad_y[n * out_f + o];
    grad_b[o] = acc;
  }
  return 0;
}

/* ---------------------------------------------------- bilinear upsample */

/* kernels/upsampling_bilinear_kernels.cl:51-64 and 109-122: half-pixel
 * source coordinate of output row/col `o`, its floor, the clamped corner
 * pair and the fraction.  Evaluated exactly as written there:
 * ((o + 0.5f) * (float)in) / (float)out - 0.5f. */
static void up_coord(int o, int in, int out, int* i0c, int* i1c, float* frac) {
  const float f = (o + 0.5f) * (float)in / (float)out - 0.5f;
  const int i0 = (int)floorf(f);
  const int i1 = i0 + 1;
  *frac = f - (float)i0;
  *i0c = i0 < 0 ? 0 : (i0 > in - 1 ? in - 1 : i0);
  *i1c = i1 < 0 ? 0 : (i1 > in - 1 ? in - 1 : i1);
}

/* kernels/upsampling_bilinear_kernels.cl:35-84 */
int port_upsampling_bilinear2d(const float* x, float* y, int N, int H, int W,
                               int C, int sy, int sx) {
  const int Ho = H * sy, Wo = W * sx;
  const int64_t total = (int64_t)N * Ho * Wo * C;
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t g = 0; g < total; ++g) {
    const int c = (int)(g % C);
    const int ow = (int)((g / C) % Wo);
    const int oh = (int)((g / ((int64_t)C * Wo)) % Ho);
    const int64_t n = g / ((int64_t)C * Wo * Ho);
    int h0, h1, w0, w1;
    float dh, dw;
    up_coord(oh, H, Ho, &h0, &h1, &dh);
    up_coord(ow, W, Wo, &w0, &w1, &dw);
    const float* xb = x + n * H * W * C + c;
    const float v00 = xb[((int64_t)h0 * W + w0) * C];
    const float v01 = xb[((int64_t)h0 * W + w1) * C];
    const float v10 = xb[((int64_t)h1 * W + w0) * C];
    const float v11 = xb[((int64_t)h1 * W + w1) * C];
    y[g] = (1.0f - dh) * (1.0f - dw) * v00 + (1.0f - dh) * dw * v01 +
           dh * (1.0f - dw) * v10 + dh * dw * v11;
  }
  return 0;
}

/* kernels/upsampling_bilinear_kernels.cl:94-135 + src/ops/upsampling_ops.cc:
 * 251-263: zero fill, then each output adds its four weighted corner terms
 * into grad_in.  Restated without atomics: every (n, c) slice is private to
 * one thread and is visited in the reference's work-item order, which is the
 * order a single-threaded reference run adds in. */
int port_upsampling_bilinear2d_grad(const float* grad_out, float* grad_in,
                                    int N, int H, int W, int C, int sy,
                                    int sx) {
  const int Ho = H * sy, Wo = W * sx;
  memset(grad_in, 0, sizeof(float) * (size_t)N * H * W * C);
  const int64_t slices = (int64_t)N * C;
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t s = 0; s < slices; ++s) {
    const int64_t n = s / C;
    const int c = (int)(s % C);
    float* gb = grad_in + n * H * W * C + c;
    for (int oh = 0; oh < Ho; ++oh) {
      int h0, h1;
      float dh;
      up_coord(oh, H, Ho, &h0, &h1, &dh);
      for (int ow = 0; ow < Wo; ++ow) {
        int w0, w1;
        float dw;
        up_coord(ow, W, Wo, &w0, &w1, &dw);
        const float g = grad_out[((n * Ho + oh) * Wo + ow) * C + c];
        gb[((int64_t)h0 * W + w0) * C] += (1.0f - dh) * (1.0f - dw) * g;
        gb[((int64_t)h0 * W + w1) * C] += (1.0f - dh) * dw * g;
        gb[((int64_t)h1 * W + w0) * C] += dh * (1.0f - dw) * g;
        gb[((int64_t)h1 * W + w1) * C] += dh * dw * g;
      }
    }
  }
  return 0;
}
