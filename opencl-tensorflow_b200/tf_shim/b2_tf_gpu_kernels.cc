// b2_tf_gpu_kernels.cc -- TensorFlow DEVICE_GPU kernels for the 19 ops of
// OpenCL-Tensorflow, each Compute body one call into libb2ocl's C ABI
// (include/b2_opencl_tf.h) on TensorFlow's CUDA stream.
//
// The reference's src/ops/*.cc keep their REGISTER_OP blocks and DEVICE_CPU
// kernels unchanged; this file adds a GPU kernel under the same op name, so
// graphs, gradients (opencl_tf/gradients.py) and layers need no edit.  What
// changes against the reference's Compute bodies:
//   * inputs and outputs are already in HBM: no clCreateBuffer(COPY_HOST_PTR)
//     per input, no blocking clEnqueueReadBuffer per output;
//   * the work is enqueued on the op's stream and the call returns; there is
//     no global queue mutex;
//   * shape inputs (input_sizes, filter_sizes) are HostMemory, as in the
//     reference's registrations.
// Shape checks that the output allocation depends on are made here, with the
// reference's messages; every other check is the library's (it returns
// B2_ERR_INVALID_ARGUMENT with the reference's message).
//
// Build (needs TensorFlow's headers and libtensorflow_framework; neither the
// TF 2.10-2.15 wheels nor their CUDA 12.2 toolchain target sm_100a, so the
// backend stays a separate CUDA 12.9 build and this file only links its ABI):
//   TF_CFLAGS=$(python -c 'import tensorflow as tf; print(" ".join(tf.sysconfig.get_compile_flags()))')
//   TF_LFLAGS=$(python -c 'import tensorflow as tf; print(" ".join(tf.sysconfig.get_link_flags()))')
//   g++ -std=c++17 -shared -fPIC -O2 -DGOOGLE_CUDA=1 $TF_CFLAGS -I include
//       src/ops/*.cc opencl-tensorflow_b200/tf_shim/b2_tf_gpu_kernels.cc
//       -L opencl-tensorflow_b200/opencl_tf -lb2ocl $TF_LFLAGS -o opencl_tf_ops.so
//   (one command line; src/ops/*.cc are the reference's op files)
#define EIGEN_USE_GPU

#include <cstdint>
#include <string>
#include <vector>

#include "tensorflow/core/framework/op_kernel.h"
#include "tensorflow/core/framework/tensor.h"
#include "tensorflow/core/framework/tensor_shape.h"

#include "b2_opencl_tf.h"

namespace b2tf {

using tensorflow::DEVICE_GPU;
using tensorflow::OpKernel;
using tensorflow::OpKernelConstruction;
using tensorflow::OpKernelContext;
using tensorflow::Status;
using tensorflow::Tensor;
using tensorflow::TensorShape;
namespace errors = tensorflow::errors;

// b2 status -> TF status.  The reference raises errors::Internal for every
// OpenCL failure (OP_REQUIRES_CL, src/ops/conv2d_ops.cc:43-45); a bounded
// device wait that gave up (B2_ERR_TIMEOUT) becomes DeadlineExceeded.
Status ToStatus(int rc) {
  switch (rc) {
    case B2_OK: return Status();
    case B2_ERR_INVALID_ARGUMENT: return errors::InvalidArgument(b2_last_error());
    case B2_ERR_TIMEOUT: return errors::DeadlineExceeded(b2_last_error());
    case B2_ERR_OUT_OF_MEMORY: return errors::ResourceExhausted(b2_last_error());
    default: return errors::Internal(b2_last_error(), " (b2 status ", rc, ")");
  }
}

b2_stream_t StreamOf(OpKernelContext* ctx) {
  return reinterpret_cast<b2_stream_t>(ctx->eigen_gpu_device().stream());
}

void Shape4(const Tensor& t, int64_t s[4]) {
  for (int i = 0; i < 4; ++i) s[i] = t.dim_size(i);
}
void Shape2(const Tensor& t, int64_t s[2]) {
  s[0] = t.dim_size(0);
  s[1] = t.dim_size(1);
}

const float* In(const Tensor& t) { return t.flat<float>().data(); }
float* Out(Tensor* t) { return t->flat<float>().data(); }

// Reads a HostMemory int32 shape vector of 4 elements; on a wrong length it
// sets the op's status (the caller checks ctx->status()).
void Sizes4(OpKernelContext* ctx, const Tensor& t, const char* msg, int32_t s[4]) {
  OP_REQUIRES(ctx, t.NumElements() == 4, errors::InvalidArgument(msg));
  auto v = t.flat<int32_t>();
  for (int i = 0; i < 4; ++i) s[i] = v(i);
}

TensorShape Shape(const int64_t* s, int n) {
  TensorShape out;
  for (int i = 0; i < n; ++i) out.AddDim(s[i]);
  return out;
}

// ------------------------------------------------------------------ strided
// OpenclConv2d / OpenclDepthwiseConv2d and their two gradients share the
// attrs strides (list(int) >= 4) and padding ({'SAME','VALID'}).
class StridedOp : public OpKernel {
 public:
  explicit StridedOp(OpKernelConstruction* c) : OpKernel(c) {
    OP_REQUIRES_OK(c, c->GetAttr("strides", &strides_));
    OP_REQUIRES_OK(c, c->GetAttr("padding", &padding_));
  }

 protected:
  const int32_t* strides() const { return strides_.data(); }
  int num_strides() const { return static_cast<int>(strides_.size()); }
  const char* padding() const { return padding_.c_str(); }

 private:
  std::vector<int32_t> strides_;
  std::string padding_;
};

// OpenclConv2d (src/ops/conv2d_ops.cc:53-196) and OpenclDepthwiseConv2d
// (src/ops/depthwise_conv2d_ops.cc:49-192).
template <bool kDepthwise>
class ForwardOp : public StridedOp {
 public:
  using StridedOp::StridedOp;
  void Compute(OpKernelContext* ctx) override {
    const Tensor& in = ctx->input(0);
    const Tensor& fil = ctx->input(1);
    OP_REQUIRES(ctx, in.dims() == 4, errors::InvalidArgument("input must be rank 4"));
    OP_REQUIRES(ctx, fil.dims() == 4, errors::InvalidArgument("filter must be rank 4"));
    int64_t xs[4], ws[4], ys[4];
    Shape4(in, xs);
    Shape4(fil, ws);
    OP_REQUIRES_OK(ctx, ToStatus(kDepthwise
        ? b2_depthwise_conv2d_output_shape(xs, ws, strides(), num_strides(), padding(), ys)
        : b2_conv2d_output_shape(xs, ws, strides(), num_strides(), padding(), ys)));
    Tensor* out = nullptr;
    OP_REQUIRES_OK(ctx, ctx->allocate_output(0, Shape(ys, 4), &out));
    OP_REQUIRES_OK(ctx, ToStatus(kDepthwise
        ? b2_depthwise_conv2d(StreamOf(ctx), In(in), xs, In(fil), ws, strides(), num_strides(),
                              padding(), Out(out), ys)
        : b2_conv2d(StreamOf(ctx), In(in), xs, In(fil), ws, strides(), num_strides(), padding(),
                    Out(out), ys)));
  }
};

// OpenclConv2dBackpropInput (conv2d_ops.cc:203-321) and
// OpenclDepthwiseConv2dBackpropInput (depthwise_conv2d_ops.cc:198-311):
// inputs (input_sizes[HostMemory], filter, out_backprop).
template <bool kDepthwise>
class BackpropInputOp : public StridedOp {
 public:
  using StridedOp::StridedOp;
  void Compute(OpKernelContext* ctx) override {
    const Tensor& fil = ctx->input(1);
    const Tensor& go = ctx->input(2);
    int32_t sizes[4];
    Sizes4(ctx, ctx->input(0), "input_sizes must have 4 elements", sizes);
    if (!ctx->status().ok()) return;
    OP_REQUIRES(ctx, fil.dims() == 4 && go.dims() == 4,
                errors::InvalidArgument("out_backprop shape mismatch"));
    int64_t ws[4], gs[4], xs[4] = {sizes[0], sizes[1], sizes[2], sizes[3]};
    Shape4(fil, ws);
    Shape4(go, gs);
    Tensor* out = nullptr;
    OP_REQUIRES_OK(ctx, ctx->allocate_output(0, Shape(xs, 4), &out));
    OP_REQUIRES_OK(ctx, ToStatus(kDepthwise
        ? b2_depthwise_conv2d_backprop_input(StreamOf(ctx), sizes, In(fil), ws, In(go), gs,
                                             strides(), num_strides(), padding(), Out(out))
        : b2_conv2d_backprop_input(StreamOf(ctx), sizes, In(fil), ws, In(go), gs, strides(),
                                   num_strides(), padding(), Out(out))));
  }
};

// OpenclConv2dBackpropFilter (conv2d_ops.cc:328-447) and
// OpenclDepthwiseConv2dBackpropFilter (depthwise_conv2d_ops.cc:318-432):
// inputs (input, filter_sizes[HostMemory], out_backprop).
template <bool kDepthwise>
class BackpropFilterOp : public StridedOp {
 public:
  using StridedOp::StridedOp;
  void Compute(OpKernelContext* ctx) override {
    const Tensor& in = ctx->input(0);
    const Tensor& go = ctx->input(2);
    int32_t sizes[4];
    Sizes4(ctx, ctx->input(1), "filter_sizes must have 4 elements", sizes);
    if (!ctx->status().ok()) return;
    OP_REQUIRES(ctx, in.dims() == 4 && go.dims() == 4,
                errors::InvalidArgument("out_backprop shape mismatch"));
    int64_t xs[4], gs[4], fs[4] = {sizes[0], sizes[1], sizes[2], sizes[3]};
    Shape4(in, xs);
    Shape4(go, gs);
    Tensor* out = nullptr;
    OP_REQUIRES_OK(ctx, ctx->allocate_output(0, Shape(fs, 4), &out));
    OP_REQUIRES_OK(ctx, ToStatus(kDepthwise
        ? b2_depthwise_conv2d_backprop_filter(StreamOf(ctx), In(in), xs, sizes, In(go), gs,
                                              strides(), num_strides(), padding(), Out(out))
        : b2_conv2d_backprop_filter(StreamOf(ctx), In(in), xs, sizes, In(go), gs, strides(),
                                    num_strides(), padding(), Out(out))));
  }
};

// -------------------------------------------------------------- elementwise
using UnaryFn = int (*)(b2_stream_t, const float*, float*, int64_t);
using BinaryFn = int (*)(b2_stream_t, const float*, const float*, float*, int64_t);

// OpenclRelu (relu_ops.cc:40-93), OpenclSigmoid (sigmoid_ops.cc:49-103).
template <UnaryFn kFn>
class UnaryOp : public OpKernel {
 public:
  using OpKernel::OpKernel;
  void Compute(OpKernelContext* ctx) override {
    const Tensor& in = ctx->input(0);
    Tensor* out = nullptr;
    OP_REQUIRES_OK(ctx, ctx->allocate_output(0, in.shape(), &out));
    OP_REQUIRES_OK(ctx, ToStatus(kFn(StreamOf(ctx), In(in), Out(out), in.NumElements())));
  }
};

// OpenclReluGrad(gradients, features) (relu_ops.cc:101-165),
// OpenclSigmoidGrad(y, dy) (sigmoid_ops.cc:110-174).
template <BinaryFn kFn>
class BinaryOp : public OpKernel {
 public:
  explicit BinaryOp(OpKernelConstruction* c, const char* msg) : OpKernel(c), msg_(msg) {}
  void Compute(OpKernelContext* ctx) override {
    const Tensor& a = ctx->input(0);
    const Tensor& b = ctx->input(1);
    OP_REQUIRES(ctx, a.shape() == b.shape(), errors::InvalidArgument(msg_));
    Tensor* out = nullptr;
    OP_REQUIRES_OK(ctx, ctx->allocate_output(0, a.shape(), &out));
    OP_REQUIRES_OK(ctx, ToStatus(kFn(StreamOf(ctx), In(a), In(b), Out(out), a.NumElements())));
  }

 private:
  const char* msg_;
};

class ReluGradOp : public BinaryOp<b2_relu_grad> {
 public:
  explicit ReluGradOp(OpKernelConstruction* c)
      : BinaryOp(c, "gradients and features must have equal shape") {}
};
class SigmoidGradOp : public BinaryOp<b2_sigmoid_grad> {
 public:
  explicit SigmoidGradOp(OpKernelConstruction* c)
      : BinaryOp(c, "y and dy must have equal shape") {}
};

// ---------------------------------------------------------------- BatchNorm
class EpsilonOp : public OpKernel {
 public:
  explicit EpsilonOp(OpKernelConstruction* c) : OpKernel(c) {
    OP_REQUIRES_OK(c, c->GetAttr("epsilon", &epsilon_));
  }

 protected:
  float epsilon_ = 1e-3f;
};

// OpenclBatchNormTraining(x, gamma, beta) -> (y, saved_mean, saved_var)
// (batchnorm_ops.cc:64-185).
class BatchNormTrainingOp : public EpsilonOp {
 public:
  using EpsilonOp::EpsilonOp;
  void Compute(OpKernelContext* ctx) override {
    const Tensor& x = ctx->input(0);
    const Tensor& gamma = ctx->input(1);
    const Tensor& beta = ctx->input(2);
    OP_REQUIRES(ctx, x.dims() == 4, errors::InvalidArgument("x must be NHWC"));
    int64_t xs[4];
    Shape4(x, xs);
    Tensor *y = nullptr, *mean = nullptr, *var = nullptr;
    OP_REQUIRES_OK(ctx, ctx->allocate_output(0, x.shape(), &y));
    OP_REQUIRES_OK(ctx, ctx->allocate_output(1, Shape(xs + 3, 1), &mean));
    OP_REQUIRES_OK(ctx, ctx->allocate_output(2, Shape(xs + 3, 1), &var));
    OP_REQUIRES_OK(ctx, ToStatus(b2_batch_norm_training(
        StreamOf(ctx), In(x), xs, In(gamma), gamma.NumElements(), In(beta), beta.NumElements(),
        epsilon_, Out(y), Out(mean), Out(var))));
  }
};

// OpenclBatchNormInference(x, gamma, beta, mean, var) -> y
// (batchnorm_ops.cc:192-281).
class BatchNormInferenceOp : public EpsilonOp {
 public:
  using EpsilonOp::EpsilonOp;
  void Compute(OpKernelContext* ctx) override {
    const Tensor& x = ctx->input(0);
    const Tensor& gamma = ctx->input(1);
    const Tensor& beta = ctx->input(2);
    const Tensor& mean = ctx->input(3);
    const Tensor& var = ctx->input(4);
    OP_REQUIRES(ctx, x.dims() == 4, errors::InvalidArgument("x must be NHWC"));
    int64_t xs[4];
    Shape4(x, xs);
    Tensor* y = nullptr;
    OP_REQUIRES_OK(ctx, ctx->allocate_output(0, x.shape(), &y));
    OP_REQUIRES_OK(ctx, ToStatus(b2_batch_norm_inference(
        StreamOf(ctx), In(x), xs, In(gamma), gamma.NumElements(), In(beta), beta.NumElements(),
        In(mean), mean.NumElements(), In(var), var.NumElements(), epsilon_, Out(y))));
  }
};

// OpenclBatchNormGrad(grad_y, x, gamma, saved_mean, saved_var)
//   -> (grad_x, grad_gamma, grad_beta)  (batchnorm_ops.cc:288-421).
class BatchNormGradOp : public EpsilonOp {
 public:
  using EpsilonOp::EpsilonOp;
  void Compute(OpKernelContext* ctx) override {
    const Tensor& gy = ctx->input(0);
    const Tensor& x = ctx->input(1);
    OP_REQUIRES(ctx, x.dims() == 4 && gy.shape() == x.shape(),
                errors::InvalidArgument("grad_y and x must have matching NHWC shapes"));
    int64_t xs[4];
    Shape4(x, xs);
    Tensor *gx = nullptr, *gg = nullptr, *gb = nullptr;
    OP_REQUIRES_OK(ctx, ctx->allocate_output(0, x.shape(), &gx));
    OP_REQUIRES_OK(ctx, ctx->allocate_output(1, Shape(xs + 3, 1), &gg));
    OP_REQUIRES_OK(ctx, ctx->allocate_output(2, Shape(xs + 3, 1), &gb));
    OP_REQUIRES_OK(ctx, ToStatus(b2_batch_norm_grad(
        StreamOf(ctx), In(gy), xs, In(x), xs, In(ctx->input(2)), In(ctx->input(3)),
        In(ctx->input(4)), epsilon_, Out(gx), Out(gg), Out(gb))));
  }
};

// -------------------------------------------------------------------- Dense
// OpenclDense(x, w, b) -> y (dense_ops.cc:57-146).
class DenseOp : public OpKernel {
 public:
  using OpKernel::OpKernel;
  void Compute(OpKernelContext* ctx) override {
    const Tensor& x = ctx->input(0);
    const Tensor& w = ctx->input(1);
    const Tensor& b = ctx->input(2);
    OP_REQUIRES(ctx, x.dims() == 2, errors::InvalidArgument("x must be rank 2"));
    OP_REQUIRES(ctx, w.dims() == 2, errors::InvalidArgument("W must be rank 2"));
    OP_REQUIRES(ctx, b.dims() == 1, errors::InvalidArgument("b must be rank 1"));
    int64_t xs[2], ws[2];
    Shape2(x, xs);
    Shape2(w, ws);
    const int64_t ys[2] = {xs[0], ws[1]};
    Tensor* y = nullptr;
    OP_REQUIRES_OK(ctx, ctx->allocate_output(0, Shape(ys, 2), &y));
    OP_REQUIRES_OK(ctx, ToStatus(b2_dense(StreamOf(ctx), In(x), xs, In(w), ws, In(b),
                                          b.NumElements(), Out(y))));
  }
};

// OpenclDenseBackpropInput(grad_y, w) -> grad_x (dense_ops.cc:152-229).
class DenseBackpropInputOp : public OpKernel {
 public:
  using OpKernel::OpKernel;
  void Compute(OpKernelContext* ctx) override {
    const Tensor& gy = ctx->input(0);
    const Tensor& w = ctx->input(1);
    OP_REQUIRES(ctx, gy.dims() == 2, errors::InvalidArgument("grad_y must be rank 2"));
    OP_REQUIRES(ctx, w.dims() == 2, errors::InvalidArgument("W must be rank 2"));
    int64_t gs[2], ws[2];
    Shape2(gy, gs);
    Shape2(w, ws);
    const int64_t xs[2] = {gs[0], ws[0]};
    Tensor* gx = nullptr;
    OP_REQUIRES_OK(ctx, ctx->allocate_output(0, Shape(xs, 2), &gx));
    OP_REQUIRES_OK(ctx, ToStatus(b2_dense_backprop_input(StreamOf(ctx), In(gy), gs, In(w), ws,
                                                         Out(gx))));
  }
};

// OpenclDenseBackpropWeight(x, grad_y) -> grad_w (dense_ops.cc:236-313).
class DenseBackpropWeightOp : public OpKernel {
 public:
  using OpKernel::OpKernel;
  void Compute(OpKernelContext* ctx) override {
    const Tensor& x = ctx->input(0);
    const Tensor& gy = ctx->input(1);
    OP_REQUIRES(ctx, x.dims() == 2, errors::InvalidArgument("x must be rank 2"));
    OP_REQUIRES(ctx, gy.dims() == 2, errors::InvalidArgument("grad_y must be rank 2"));
    int64_t xs[2], gs[2];
    Shape2(x, xs);
    Shape2(gy, gs);
    const int64_t ws[2] = {xs[1], gs[1]};
    Tensor* gw = nullptr;
    OP_REQUIRES_OK(ctx, ctx->allocate_output(0, Shape(ws, 2), &gw));
    OP_REQUIRES_OK(ctx, ToStatus(b2_dense_backprop_weight(StreamOf(ctx), In(x), xs, In(gy), gs,
                                                          Out(gw))));
  }
};

// OpenclDenseBackpropBias(grad_y) -> grad_b (dense_ops.cc:320-381).
class DenseBackpropBiasOp : public OpKernel {
 public:
  using OpKernel::OpKernel;
  void Compute(OpKernelContext* ctx) override {
    const Tensor& gy = ctx->input(0);
    OP_REQUIRES(ctx, gy.dims() == 2, errors::InvalidArgument("grad_y must be rank 2"));
    int64_t gs[2];
    Shape2(gy, gs);
    Tensor* gb = nullptr;
    OP_REQUIRES_OK(ctx, ctx->allocate_output(0, Shape(gs + 1, 1), &gb));
    OP_REQUIRES_OK(ctx, ToStatus(b2_dense_backprop_bias(StreamOf(ctx), In(gy), gs, Out(gb))));
  }
};

// ------------------------------------------------------------- UpSampling2D
class SizeOp : public OpKernel {
 public:
  explicit SizeOp(OpKernelConstruction* c) : OpKernel(c) {
    OP_REQUIRES_OK(c, c->GetAttr("size", &size_));
    OP_REQUIRES(c, size_.size() == 2,
                errors::InvalidArgument("size must have exactly 2 elements"));
    OP_REQUIRES(c, size_[0] >= 1 && size_[1] >= 1,
                errors::InvalidArgument("size elements must be >= 1"));
  }

 protected:
  std::vector<int32_t> size_;
};

// OpenclUpsamplingBilinear2d(input; size) (upsampling_ops.cc:59-159).
class UpsamplingOp : public SizeOp {
 public:
  using SizeOp::SizeOp;
  void Compute(OpKernelContext* ctx) override {
    const Tensor& in = ctx->input(0);
    OP_REQUIRES(ctx, in.dims() == 4, errors::InvalidArgument("input must be NHWC"));
    int64_t xs[4];
    Shape4(in, xs);
    const int64_t ys[4] = {xs[0], xs[1] * size_[0], xs[2] * size_[1], xs[3]};
    Tensor* out = nullptr;
    OP_REQUIRES_OK(ctx, ctx->allocate_output(0, Shape(ys, 4), &out));
    OP_REQUIRES_OK(ctx, ToStatus(b2_upsampling_bilinear2d(StreamOf(ctx), In(in), xs, size_.data(),
                                                          2, Out(out))));
  }
};

// OpenclUpsamplingBilinear2dGrad(grad_out, input_sizes[HostMemory]; size)
// (upsampling_ops.cc:166-272).
class UpsamplingGradOp : public SizeOp {
 public:
  using SizeOp::SizeOp;
  void Compute(OpKernelContext* ctx) override {
    const Tensor& go = ctx->input(0);
    int32_t sizes[4];
    Sizes4(ctx, ctx->input(1), "input_sizes must have 4 elements [N,H,W,C]", sizes);
    if (!ctx->status().ok()) return;
    OP_REQUIRES(ctx, go.dims() == 4,
                errors::InvalidArgument("grad_out shape mismatch with input_sizes + size"));
    int64_t gs[4], xs[4] = {sizes[0], sizes[1], sizes[2], sizes[3]};
    Shape4(go, gs);
    Tensor* gi = nullptr;
    OP_REQUIRES_OK(ctx, ctx->allocate_output(0, Shape(xs, 4), &gi));
    OP_REQUIRES_OK(ctx, ToStatus(b2_upsampling_bilinear2d_grad(StreamOf(ctx), In(go), gs, sizes,
                                                               size_.data(), 2, Out(gi))));
  }
};

REGISTER_KERNEL_BUILDER(Name("OpenclConv2d").Device(DEVICE_GPU), ForwardOp<false>);
REGISTER_KERNEL_BUILDER(Name("OpenclConv2dBackpropInput").Device(DEVICE_GPU).HostMemory("input_sizes"),
                        BackpropInputOp<false>);
REGISTER_KERNEL_BUILDER(Name("OpenclConv2dBackpropFilter").Device(DEVICE_GPU).HostMemory("filter_sizes"),
                        BackpropFilterOp<false>);
REGISTER_KERNEL_BUILDER(Name("OpenclDepthwiseConv2d").Device(DEVICE_GPU), ForwardOp<true>);
REGISTER_KERNEL_BUILDER(
    Name("OpenclDepthwiseConv2dBackpropInput").Device(DEVICE_GPU).HostMemory("input_sizes"),
    BackpropInputOp<true>);
REGISTER_KERNEL_BUILDER(
    Name("OpenclDepthwiseConv2dBackpropFilter").Device(DEVICE_GPU).HostMemory("filter_sizes"),
    BackpropFilterOp<true>);
REGISTER_KERNEL_BUILDER(Name("OpenclRelu").Device(DEVICE_GPU), UnaryOp<b2_relu>);
REGISTER_KERNEL_BUILDER(Name("OpenclReluGrad").Device(DEVICE_GPU), ReluGradOp);
REGISTER_KERNEL_BUILDER(Name("OpenclSigmoid").Device(DEVICE_GPU), UnaryOp<b2_sigmoid>);
REGISTER_KERNEL_BUILDER(Name("OpenclSigmoidGrad").Device(DEVICE_GPU), SigmoidGradOp);
REGISTER_KERNEL_BUILDER(Name("OpenclBatchNormTraining").Device(DEVICE_GPU), BatchNormTrainingOp);
REGISTER_KERNEL_BUILDER(Name("OpenclBatchNormInference").Device(DEVICE_GPU), BatchNormInferenceOp);
REGISTER_KERNEL_BUILDER(Name("OpenclBatchNormGrad").Device(DEVICE_GPU), BatchNormGradOp);
REGISTER_KERNEL_BUILDER(Name("OpenclDense").Device(DEVICE_GPU), DenseOp);
REGISTER_KERNEL_BUILDER(Name("OpenclDenseBackpropInput").Device(DEVICE_GPU), DenseBackpropInputOp);
REGISTER_KERNEL_BUILDER(Name("OpenclDenseBackpropWeight").Device(DEVICE_GPU), DenseBackpropWeightOp);
REGISTER_KERNEL_BUILDER(Name("OpenclDenseBackpropBias").Device(DEVICE_GPU), DenseBackpropBiasOp);
REGISTER_KERNEL_BUILDER(Name("OpenclUpsamplingBilinear2d").Device(DEVICE_GPU), UpsamplingOp);
REGISTER_KERNEL_BUILDER(
    Name("OpenclUpsamplingBilinear2dGrad").Device(DEVICE_GPU).HostMemory("input_sizes"),
    UpsamplingGradOp);

}  // namespace b2tf
