"""Sigmoid ops (reference: opencl_tf/ops/sigmoid.py, src/ops/sigmoid_ops.cc)."""
from __future__ import annotations

from .._library import raw_ops


def sigmoid(x):
    """Elementwise 1 / (1 + exp(-x))."""
    return raw_ops.opencl_sigmoid(x)


def sigmoid_grad(y, dy):
    """dy * y * (1 - y) where ``y`` is the forward OUTPUT sigmoid(x)."""
    return raw_ops.opencl_sigmoid_grad(y, dy)
