"""Conv2D parity on the GPU (reference tests: tests/test_conv2d.py).  All three
ops run on the tcgen05 3xTF32 implicit-GEMM engine; results are compared with
the oracle within max-rel 1e-4 / L2-rel 1e-5, at the reference tests'
fixtures and at the shapes of the README network."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_close, to_np

pytestmark = pytest.mark.gpu

CASES = [((1, 1, 1, 1), "SAME"), ((1, 2, 2, 1), "SAME"), ((1, 1, 1, 1), "VALID"), ((1, 2, 2, 1), "VALID")]


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def _inputs(seed, shape_x, shape_w):
    rng = np.random.default_rng(seed)
    return rng.standard_normal(shape_x).astype(np.float32), rng.standard_normal(shape_w).astype(np.float32)


@pytest.mark.parametrize("strides,padding", CASES)
def test_conv2d_forward(otf, port, strides, padding):
    x, w = _inputs(0, (2, 9, 9, 3), (3, 3, 3, 5))
    got = to_np(otf.conv2d(_cuda(x), _cuda(w), strides=strides, padding=padding))
    assert_close(got, port.conv2d(x, w, strides, padding), what="conv fwd")


@pytest.mark.parametrize("strides,padding", CASES)
def test_conv2d_gradients(otf, port, strides, padding):
    x, w = _inputs(1, (2, 9, 9, 3), (3, 3, 3, 5))
    xt, wt = _cuda(x).requires_grad_(True), _cuda(w).requires_grad_(True)
    y = otf.conv2d(xt, wt, strides=strides, padding=padding)
    (0.5 * (y * y).sum()).backward()
    ry = port.conv2d(x, w, strides, padding)
    assert_close(to_np(xt.grad), port.conv2d_backprop_input(x.shape, w, ry, strides, padding), what="dx")
    assert_close(to_np(wt.grad), port.conv2d_backprop_filter(x, w.shape, ry, strides, padding), what="dw")


SHAPES = [
    # x, w, strides, padding
    ((2, 16, 16, 3), (3, 7, 3, 48), (1, 1, 2, 1), "SAME"),      # the network's stem
    ((4, 8, 8, 48), (1, 1, 48, 96), (1, 1, 1, 1), "SAME"),      # pointwise 48 -> 96
    ((4, 8, 4, 96), (1, 1, 96, 144), (1, 1, 1, 1), "SAME"),     # pointwise 96 -> 144
    ((3, 11, 13, 8), (3, 3, 8, 20), (1, 2, 2, 1), "SAME"),
    ((2, 10, 9, 5), (5, 3, 5, 7), (1, 3, 2, 1), "VALID"),
    ((1, 1, 1, 1), (1, 1, 1, 1), (1, 1, 1, 1), "SAME"),
    ((3, 6, 6, 12), (2, 2, 12, 300), (1, 2, 2, 1), "SAME"),     # N > 256: several N tiles
    ((2, 7, 7, 16), (3, 3, 16, 16), (1, 1, 1, 1), "VALID"),
    # staged-row im2col path of the TMA engine (whole input rows <= 256 floats)
    ((2, 16, 16, 4), (3, 3, 4, 40), (1, 1, 1, 1), "SAME"),
    ((2, 32, 16, 4), (5, 5, 4, 24), (1, 2, 2, 1), "SAME"),
    ((2, 33, 17, 4), (3, 3, 4, 20), (1, 2, 2, 1), "VALID"),
    ((4, 32, 32, 3), (3, 3, 3, 36), (1, 1, 1, 1), "SAME"),
]


@pytest.mark.parametrize("xs,ws,strides,padding", SHAPES)
def test_conv2d_shapes(otf, port, xs, ws, strides, padding):
    x, w = _inputs(3, xs, ws)
    y = otf.conv2d(_cuda(x), _cuda(w), strides=strides, padding=padding)
    ry = port.conv2d(x, w, strides, padding)
    assert_close(to_np(y), ry, what="fwd")
    dy = np.random.default_rng(4).standard_normal(ry.shape).astype(np.float32)
    dx = otf.conv2d_backprop_input(list(xs), _cuda(w), _cuda(dy), strides=strides, padding=padding)
    assert_close(to_np(dx), port.conv2d_backprop_input(xs, w, dy, strides, padding), what="dgrad")
    dw = otf.conv2d_backprop_filter(_cuda(x), list(ws), _cuda(dy), strides=strides, padding=padding)
    assert_close(to_np(dw), port.conv2d_backprop_filter(x, ws, dy, strides, padding), what="wgrad")


def test_conv2d_deterministic(otf):
    x = torch.randn(16, 64, 32, 3, device="cuda")
    w = torch.randn(3, 7, 3, 48, device="cuda")
    dy = torch.randn(16, 64, 16, 48, device="cuda")
    st = (1, 1, 2, 1)
    a = otf.conv2d_backprop_filter(x, [3, 7, 3, 48], dy, strides=st, padding="SAME")
    b = otf.conv2d_backprop_filter(x, [3, 7, 3, 48], dy, strides=st, padding="SAME")
    assert torch.equal(a, b)
    assert torch.equal(otf.conv2d(x, w, strides=st, padding="SAME"), otf.conv2d(x, w, strides=st, padding="SAME"))


def test_conv2d_bad_args(otf):
    x = torch.zeros(1, 5, 5, 3, device="cuda")
    w = torch.zeros(3, 3, 3, 4, device="cuda")
    with pytest.raises(otf.errors.InvalidArgumentError, match="strides must be length 4"):
        otf.conv2d(x, w, strides=(1, 1, 1, 1, 1))
    with pytest.raises(otf.errors.InvalidArgumentError, match="strides on N and C must be 1"):
        otf.conv2d(x, w, strides=(1, 1, 1, 2))
    with pytest.raises(otf.errors.InvalidArgumentError, match="padding"):
        otf.conv2d(x, w, padding="FULL")
    with pytest.raises(otf.errors.InvalidArgumentError, match="filter\\[2\\] must equal input channels"):
        otf.conv2d(x, torch.zeros(3, 3, 2, 4, device="cuda"))
    with pytest.raises(otf.errors.InvalidArgumentError, match="rank 4"):
        otf.conv2d(x[0], w)
    with pytest.raises(otf.errors.InvalidArgumentError, match="out_backprop shape mismatch"):
        otf.conv2d_backprop_input([1, 5, 5, 3], w, torch.zeros(1, 4, 5, 4, device="cuda"), strides=(1, 1, 1, 1),
                                  padding="SAME")
    with pytest.raises(otf.errors.InvalidArgumentError, match="input_sizes must have 4 elements"):
        otf.conv2d_backprop_input([1, 5, 5], w, torch.zeros(1, 5, 5, 4, device="cuda"), strides=(1, 1, 1, 1),
                                  padding="SAME")
