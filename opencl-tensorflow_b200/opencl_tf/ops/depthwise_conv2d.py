"""DepthwiseConv2D ops (reference: opencl_tf/ops/depthwise_conv2d.py,
src/ops/depthwise_conv2d_ops.cc)."""
from __future__ import annotations

from typing import Sequence

from .._library import raw_ops


def depthwise_conv2d(x, w, strides: Sequence[int] = (1, 1, 1, 1), padding: str = "SAME"):
    """x [N,H,W,C], w [kH,kW,C,depth_multiplier] -> [N,Hout,Wout,C*dm];
    output channel ci*dm + d sees only input channel ci."""
    return raw_ops.opencl_depthwise_conv2d(x, w, strides=list(strides), padding=padding)


def depthwise_conv2d_backprop_input(input_sizes, w, grad_out, strides: Sequence[int], padding: str):
    return raw_ops.opencl_depthwise_conv2d_backprop_input(input_sizes, w, grad_out, strides=list(strides),
                                                          padding=padding)


def depthwise_conv2d_backprop_filter(x, filter_sizes, grad_out, strides: Sequence[int], padding: str):
    return raw_ops.opencl_depthwise_conv2d_backprop_filter(x, filter_sizes, grad_out, strides=list(strides),
                                                           padding=padding)
