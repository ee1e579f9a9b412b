"""Conv2D ops (reference: opencl_tf/ops/conv2d.py, src/ops/conv2d_ops.cc)."""
from __future__ import annotations

from typing import Sequence

from .._library import raw_ops


def conv2d(x, w, strides: Sequence[int] = (1, 1, 1, 1), padding: str = "SAME"):
    """Forward convolution: x [N,H,W,Cin] (NHWC), w [kH,kW,Cin,Cout] (HWIO);
    ``strides`` NHWC with strides[0] == strides[3] == 1; ``padding`` "SAME" or
    "VALID".  Returns [N,Hout,Wout,Cout]."""
    return raw_ops.opencl_conv2d(x, w, strides=list(strides), padding=padding)


def conv2d_backprop_input(input_sizes, w, grad_out, strides: Sequence[int], padding: str):
    """dL/dx.  ``input_sizes`` is the host shape [N,H,W,Cin] of x."""
    return raw_ops.opencl_conv2d_backprop_input(input_sizes, w, grad_out, strides=list(strides),
                                                padding=padding)


def conv2d_backprop_filter(x, filter_sizes, grad_out, strides: Sequence[int], padding: str):
    """dL/dw.  ``filter_sizes`` is the host shape [kH,kW,Cin,Cout] of w."""
    return raw_ops.opencl_conv2d_backprop_filter(x, filter_sizes, grad_out, strides=list(strides),
                                                 padding=padding)
