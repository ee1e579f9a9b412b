"""DepthwiseConv2D parity on the GPU (reference tests:
tests/test_depthwise_conv2d.py).  Forward and input gradient sum the taps in
the reference's order and are bit-exact; the filter gradient (a reduction
over N*Ho*Wo) is within the fp32 tolerance."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_bitexact, assert_close, to_np

pytestmark = pytest.mark.gpu

CASES = [((1, 1, 1, 1), "SAME"), ((1, 2, 2, 1), "SAME"), ((1, 1, 1, 1), "VALID"), ((1, 2, 2, 1), "VALID")]


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def _inputs(seed, shape_x, shape_w):
    rng = np.random.default_rng(seed)
    return rng.standard_normal(shape_x).astype(np.float32), rng.standard_normal(shape_w).astype(np.float32)


@pytest.mark.parametrize("dm", [1, 2])
@pytest.mark.parametrize("strides,padding", CASES)
def test_dwconv2d_forward(otf, port, strides, padding, dm):
    x, w = _inputs(0, (2, 9, 9, 4), (3, 3, 4, dm))
    got = to_np(otf.depthwise_conv2d(_cuda(x), _cuda(w), strides=strides, padding=padding))
    assert_bitexact(got, port.depthwise_conv2d(x, w, strides, padding), "dw fwd")


@pytest.mark.parametrize("dm", [1, 2])
@pytest.mark.parametrize("strides,padding", CASES)
def test_dwconv2d_gradients(otf, port, strides, padding, dm):
    x, w = _inputs(1, (2, 9, 9, 4), (3, 3, 4, dm))
    xt, wt = _cuda(x).requires_grad_(True), _cuda(w).requires_grad_(True)
    y = otf.depthwise_conv2d(xt, wt, strides=strides, padding=padding)
    (0.5 * (y * y).sum()).backward()
    ry = port.depthwise_conv2d(x, w, strides, padding)
    assert_bitexact(to_np(xt.grad), port.depthwise_conv2d_backprop_input(x.shape, w, ry, strides, padding), "dx")
    assert_close(to_np(wt.grad), port.depthwise_conv2d_backprop_filter(x, w.shape, ry, strides, padding),
                 what="dw")


@pytest.mark.parametrize("shape_x,k,s,padding", [((64, 32, 16, 48), 3, 2, "SAME"), ((8, 64, 32, 48), 3, 2, "SAME"),
                                                ((4, 17, 13, 12), 5, 3, "SAME"), ((3, 11, 10, 6), 3, 1, "VALID"),
                                                ((2, 8, 8, 96), 3, 2, "VALID"), ((5, 7, 9, 7), 2, 2, "SAME")])
def test_dwconv2d_shapes(otf, port, shape_x, k, s, padding):
    x, w = _inputs(7, shape_x, (k, k, shape_x[3], 1))
    st = (1, s, s, 1)
    y = otf.depthwise_conv2d(_cuda(x), _cuda(w), strides=st, padding=padding)
    ry = port.depthwise_conv2d(x, w, st, padding)
    assert_bitexact(to_np(y), ry, "fwd")
    dy = np.random.default_rng(8).standard_normal(ry.shape).astype(np.float32)
    dx = otf.depthwise_conv2d_backprop_input(list(x.shape), _cuda(w), _cuda(dy), strides=st, padding=padding)
    assert_bitexact(to_np(dx), port.depthwise_conv2d_backprop_input(x.shape, w, dy, st, padding), "dgrad")
    dw = otf.depthwise_conv2d_backprop_filter(_cuda(x), list(w.shape), _cuda(dy), strides=st, padding=padding)
    assert_close(to_np(dw), port.depthwise_conv2d_backprop_filter(x, w.shape, dy, st, padding), what="wgrad")


def test_dwconv2d_bad_args(otf):
    x = torch.zeros(1, 5, 5, 4, device="cuda")
    with pytest.raises(otf.errors.InvalidArgumentError, match="filter\\[2\\] must equal input channels"):
        otf.depthwise_conv2d(x, torch.zeros(3, 3, 3, 1, device="cuda"))
    with pytest.raises(otf.errors.InvalidArgumentError, match="strides on N and C must be 1"):
        otf.depthwise_conv2d(x, torch.zeros(3, 3, 4, 1, device="cuda"), strides=(2, 1, 1, 1))
    with pytest.raises(otf.errors.InvalidArgumentError, match="out_backprop shape mismatch"):
        otf.depthwise_conv2d_backprop_input([1, 5, 5, 4], torch.zeros(3, 3, 4, 1, device="cuda"),
                                            torch.zeros(1, 4, 5, 4, device="cuda"), strides=(1, 1, 1, 1),
                                            padding="SAME")


@pytest.mark.parametrize("shape_x,ws,st,padding", [((2, 20, 6, 8), (9, 1, 8, 1), (1, 1, 1, 1), "SAME"),
                                                   ((3, 12, 10, 16), (1, 9, 16, 1), (1, 2, 1, 1), "SAME"),
                                                   ((2, 30, 33, 4), (3, 3, 4, 1), (1, 2, 2, 1), "VALID")])
def test_dwconv2d_filter_grad_tall_and_wide_taps(otf, port, shape_x, ws, st, padding):
    """Filter gradients with 9 taps in one direction and odd widths (staged-row
    path: up to nine kernel rows per output row, right padding columns)."""
    x, w = _inputs(9, shape_x, ws)
    ry = port.depthwise_conv2d(x, w, st, padding)
    dy = np.random.default_rng(10).standard_normal(ry.shape).astype(np.float32)
    dw = otf.depthwise_conv2d_backprop_filter(_cuda(x), list(ws), _cuda(dy), strides=st, padding=padding)
    assert_close(to_np(dw), port.depthwise_conv2d_backprop_filter(x, ws, dy, st, padding), what="dw")


@pytest.mark.parametrize("shape_x,padding", [((2, 30, 33, 4), "VALID"), ((3, 11, 10, 8), "VALID"),
                                             ((2, 11, 13, 12), "SAME"), ((4, 16, 8, 96), "SAME")])
def test_dwconv2d_3x3_stride2_column_pairs(otf, port, shape_x, padding):
    """3x3 stride-2 forward and input gradient (the column-pair kernels),
    including odd widths, padding taps and input rows and columns that no tap
    reaches: bit-exact with the reference."""
    x, w = _inputs(12, shape_x, (3, 3, shape_x[3], 1))
    st = (1, 2, 2, 1)
    ry = port.depthwise_conv2d(x, w, st, padding)
    y = otf.depthwise_conv2d(_cuda(x), _cuda(w), strides=st, padding=padding)
    assert_bitexact(to_np(y), ry, "fwd")
    dy = np.random.default_rng(13).standard_normal(ry.shape).astype(np.float32)
    dx = otf.depthwise_conv2d_backprop_input(list(shape_x), _cuda(w), _cuda(dy), strides=st, padding=padding)
    assert_bitexact(to_np(dx), port.depthwise_conv2d_backprop_input(shape_x, w, dy, st, padding), "dx")
