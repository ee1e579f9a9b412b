"""Python op API, one function per reference op (opencl_tf/ops/__init__.py)."""
from .conv2d import conv2d, conv2d_backprop_input, conv2d_backprop_filter
from .depthwise_conv2d import (depthwise_conv2d, depthwise_conv2d_backprop_input,
                               depthwise_conv2d_backprop_filter)
from .relu import relu, relu_grad
from .batchnorm import batch_norm_training, batch_norm_inference, batch_norm_grad
from .sigmoid import sigmoid, sigmoid_grad
from .dense import dense, dense_backprop_input, dense_backprop_weight, dense_backprop_bias
from .upsampling import upsampling_bilinear_2d, upsampling_bilinear_2d_grad

__all__ = [
    "conv2d", "conv2d_backprop_input", "conv2d_backprop_filter",
    "depthwise_conv2d", "depthwise_conv2d_backprop_input", "depthwise_conv2d_backprop_filter",
    "relu", "relu_grad",
    "batch_norm_training", "batch_norm_inference", "batch_norm_grad",
    "sigmoid", "sigmoid_grad",
    "dense", "dense_backprop_input", "dense_backprop_weight", "dense_backprop_bias",
    "upsampling_bilinear_2d", "upsampling_bilinear_2d_grad",
]
