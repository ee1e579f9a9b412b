"""Gradient functions of the seven forward ops.

The wiring is the reference's (opencl_tf/gradients.py:18-119) because it is
part of the drop-in contract: which backward op each forward op uses, and
which tensors those ops receive --

* Conv2D / DepthwiseConv2D: input grad from the HOST shape of x, filter grad
  from the host shape of w, both with the forward strides and padding;
* ReLU: masked by the forward INPUT;
* BatchNorm (training): grad of y only (grad_mean / grad_var are ignored),
  using the forward op's saved mean / variance outputs;
* Sigmoid: from the forward OUTPUT y;
* Dense: three backward ops (input, weight, bias);
* bilinear UpSampling2D: the backward op with the input's host shape;
* BatchNorm (inference): no gradient (a LookupError if one is requested);
* the extensions: BatchNorm->ReLU (fused_ops) and the step's MSE loss
  (step_ops), each with its own one-launch backward.

An input whose gradient nobody needs gets no backward launch -- what TF's
graph pruning does for ``model.fit`` -- so the network's first convolution
never computes a gradient for the image batch.
"""
from __future__ import annotations

from ._library import RegisterGradient, fused_ops, raw_ops, step_ops


def _host_shape(t):
    return list(t.shape)


@RegisterGradient("OpenclConv2d")
def _conv2d_grad(op, grad):
    x, w = op.inputs
    strides, padding = op.get_attr("strides"), op.get_attr("padding")
    need_x, need_w = op.needs_input_grad
    dx = raw_ops.opencl_conv2d_backprop_input(_host_shape(x), w, grad, strides=strides,
                                              padding=padding) if need_x else None
    dw = raw_ops.opencl_conv2d_backprop_filter(x, _host_shape(w), grad, strides=strides,
                                               padding=padding) if need_w else None
    return [dx, dw]


@RegisterGradient("OpenclDepthwiseConv2d")
def _depthwise_conv2d_grad(op, grad):
    x, w = op.inputs
    strides, padding = op.get_attr("strides"), op.get_attr("padding")
    need_x, need_w = op.needs_input_grad
    dx = raw_ops.opencl_depthwise_conv2d_backprop_input(_host_shape(x), w, grad, strides=strides,
                                                        padding=padding) if need_x else None
    dw = raw_ops.opencl_depthwise_conv2d_backprop_filter(x, _host_shape(w), grad, strides=strides,
                                                         padding=padding) if need_w else None
    return [dx, dw]


@RegisterGradient("OpenclRelu")
def _relu_grad(op, grad):
    return [raw_ops.opencl_relu_grad(grad, op.inputs[0])]


@RegisterGradient("OpenclBatchNormTraining")
def _batch_norm_training_grad(op, grad_y, grad_mean=None, grad_var=None):
    x, gamma, _beta = op.inputs
    _y, saved_mean, saved_var = op.outputs
    gx, ggamma, gbeta = raw_ops.opencl_batch_norm_grad(grad_y, x, gamma, saved_mean, saved_var,
                                                       epsilon=op.get_attr("epsilon"))
    return [gx, ggamma, gbeta]


@RegisterGradient("OpenclBatchNormReluTraining")
def _batch_norm_relu_training_grad(op, grad_z, grad_mean=None, grad_var=None):
    x, gamma, beta = op.inputs
    _z, saved_mean, saved_var = op.outputs
    gx, ggamma, gbeta = fused_ops.opencl_batch_norm_relu_grad(grad_z, x, gamma, beta, saved_mean, saved_var,
                                                            epsilon=op.get_attr("epsilon"))
    return [gx, ggamma, gbeta]


@RegisterGradient("OpenclSigmoid")
def _sigmoid_grad(op, grad):
    return [raw_ops.opencl_sigmoid_grad(op.outputs[0], grad)]


@RegisterGradient("OpenclDense")
def _dense_grad(op, grad):
    x, w, _b = op.inputs
    need_x, need_w, need_b = op.needs_input_grad
    dx = raw_ops.opencl_dense_backprop_input(grad, w) if need_x else None
    dw = raw_ops.opencl_dense_backprop_weight(x, grad) if need_w else None
    db = raw_ops.opencl_dense_backprop_bias(grad) if need_b else None
    return [dx, dw, db]


@RegisterGradient("OpenclDenseRelu")
def _dense_relu_grad(op, grad):
    """ReluGrad then the three dense gradients.  The mask is taken from the
    op's output z = relu(x W + b): z > 0 exactly where x W + b > 0 (NaN gives
    z = 0 and fails both tests), so the bits equal those of the unfused pair."""
    x, w, _b = op.inputs
    g = raw_ops.opencl_relu_grad(grad, op.outputs[0])
    need_x, need_w, need_b = op.needs_input_grad
    dx = raw_ops.opencl_dense_backprop_input(g, w) if need_x else None
    dw = raw_ops.opencl_dense_backprop_weight(x, g) if need_w else None
    db = raw_ops.opencl_dense_backprop_bias(g) if need_b else None
    return [dx, dw, db]


@RegisterGradient("OpenclUpsamplingBilinear2d")
def _upsampling_bilinear_grad(op, grad):
    return [raw_ops.opencl_upsampling_bilinear2d_grad(grad, _host_shape(op.inputs[0]), size=op.get_attr("size"))]


@RegisterGradient("OpenclMseLoss")
def _mse_loss_grad(op, grad):
    y_pred, y_true = op.inputs
    need_pred, need_true = op.needs_input_grad
    g = step_ops.opencl_mse_loss_grad(y_pred, y_true, grad)
    return [g if need_pred else None, g.neg() if need_true else None]
