"""Bilinear UpSampling2D ops (reference: opencl_tf/ops/upsampling.py,
src/ops/upsampling_ops.cc)."""
from __future__ import annotations

from typing import List

from .._library import raw_ops


def upsampling_bilinear_2d(x, size: List[int]):
    """x [N,H,W,C] -> [N,H*sy,W*sx,C], half-pixel centres, clamped edges."""
    return raw_ops.opencl_upsampling_bilinear2d(x, size=list(size))


def upsampling_bilinear_2d_grad(grad_out, input_sizes, size: List[int]):
    """Backward of upsampling_bilinear_2d; ``input_sizes`` is the host shape
    [N,H,W,C] of the forward input."""
    return raw_ops.opencl_upsampling_bilinear2d_grad(grad_out, [int(v) for v in input_sizes], size=list(size))
