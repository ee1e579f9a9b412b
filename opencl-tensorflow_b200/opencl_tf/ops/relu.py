"""ReLU ops (reference: opencl_tf/ops/relu.py, src/ops/relu_ops.cc)."""
from __future__ import annotations

from .._library import raw_ops


def relu(x):
    """Elementwise max(x, 0); a NaN input gives 0."""
    return raw_ops.opencl_relu(x)


def relu_grad(gradients, features):
    """``gradients`` where the forward INPUT ``features`` > 0, else 0."""
    return raw_ops.opencl_relu_grad(gradients, features)
