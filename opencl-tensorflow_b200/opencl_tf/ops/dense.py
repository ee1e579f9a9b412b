"""Dense ops (reference: opencl_tf/ops/dense.py, src/ops/dense_ops.cc)."""
from __future__ import annotations

from .._library import raw_ops


def dense(x, w, b):
    """y = x @ W + b; x [batch,in_f], W [in_f,out_f], b [out_f]."""
    return raw_ops.opencl_dense(x, w, b)


def dense_backprop_input(grad_y, w):
    """grad_x = grad_y @ W^T."""
    return raw_ops.opencl_dense_backprop_input(grad_y, w)


def dense_backprop_weight(x, grad_y):
    """grad_W = x^T @ grad_y."""
    return raw_ops.opencl_dense_backprop_weight(x, grad_y)


def dense_backprop_bias(grad_y):
    """grad_b = sum over the batch of grad_y."""
    return raw_ops.opencl_dense_backprop_bias(grad_y)
