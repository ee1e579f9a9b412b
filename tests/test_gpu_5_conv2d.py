"""Conv2D parity on the GPU (reference tests: tests/test_conv2d.py).  Filters
with more than 32 input or output channels run on the tcgen05 3xTF32
implicit-GEMM engines, compared with the oracle within max-rel 1e-4 / L2-rel
1e-5; narrow filters (Ci, Co <= 32, kH*kW*Ci*Co <= 4608, which includes the
reference tests' fixtures) run on the direct CUDA-core kernels, whose forward
and input gradient equal the oracle bit for bit."""
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


@pytest.mark.parametrize("strides,padding", CASES)
def test_conv2d_forward(otf, port, strides, padding):
    x, w = _inputs(0, (2, 9, 9, 3), (3, 3, 3, 5))
    got = to_np(otf.conv2d(_cuda(x), _cuda(w), strides=strides, padding=padding))
    assert_bitexact(got, port.conv2d(x, w, strides, padding), "conv fwd")


@pytest.mark.parametrize("strides,padding", CASES)
def test_conv2d_gradients(otf, port, strides, padding):
    x, w = _inputs(1, (2, 9, 9, 3), (3, 3, 3, 5))
    xt, wt = _cuda(x).requires_grad_(True), _cuda(w).requires_grad_(True)
    y = otf.conv2d(xt, wt, strides=strides, padding=padding)
    (0.5 * (y * y).sum()).backward()
    ry = port.conv2d(x, w, strides, padding)
    assert_bitexact(to_np(xt.grad), port.conv2d_backprop_input(x.shape, w, ry, strides, padding), "dx")
    assert_close(to_np(wt.grad), port.conv2d_backprop_filter(x, w.shape, ry, strides, padding), what="dw")


SHAPES = [
    # x, w, strides, padding
    ((2, 16, 16, 3), (3, 7, 3, 48), (1, 1, 2, 1), "SAME"),      # the network's stem
    ((4, 8, 8, 48), (1, 1, 48, 96), (1, 1, 1, 1), "SAME"),      # pointwise 48 -> 96
    ((4, 8, 4, 96), (1, 1, 96, 144), (1, 1, 1, 1), "SAME"),     # pointwise 96 -> 144
    ((3, 11, 13, 8), (3, 3, 8, 36), (1, 2, 2, 1), "SAME"),     # register-fed im2col engine
    ((2, 10, 9, 5), (5, 3, 5, 40), (1, 3, 2, 1), "VALID"),
    ((3, 6, 6, 12), (2, 2, 12, 300), (1, 2, 2, 1), "SAME"),     # N > 256: several N tiles
    ((2, 7, 7, 36), (3, 3, 36, 16), (1, 1, 1, 1), "VALID"),
    # staged-row im2col path of the TMA engine (whole input rows <= 256 floats)
    ((2, 16, 16, 4), (3, 3, 4, 40), (1, 1, 1, 1), "SAME"),
    ((2, 32, 16, 4), (5, 5, 4, 40), (1, 2, 2, 1), "SAME"),
    ((2, 33, 17, 4), (3, 3, 4, 44), (1, 2, 2, 1), "VALID"),
    ((4, 32, 32, 3), (3, 3, 3, 36), (1, 1, 1, 1), "SAME"),
]

DIRECT = [
    # x, w, strides, padding -- narrow filters: direct CUDA-core kernels
    ((2, 36, 24, 16), (3, 3, 16, 16), (1, 1, 1, 1), "SAME"),    # uwb_loc_v3 hm_refine2
    ((3, 18, 12, 8), (3, 3, 8, 16), (1, 1, 1, 1), "SAME"),      # uwb_loc_v3 hm_refine1
    ((2, 36, 24, 16), (1, 1, 16, 1), (1, 1, 1, 1), "SAME"),     # uwb_loc_v3 heatmap_conv
    ((3, 11, 13, 8), (3, 3, 8, 20), (1, 2, 2, 1), "SAME"),      # 5 output-channel groups of 4
    ((2, 10, 9, 5), (5, 3, 5, 7), (1, 3, 2, 1), "VALID"),       # odd channels: scalar loads, 1-wide groups
    ((2, 7, 7, 32), (3, 3, 32, 16), (1, 1, 1, 1), "VALID"),     # 4608 weights: filter gradient over 2 CTAs
    ((2, 9, 9, 1), (3, 3, 1, 32), (1, 2, 1, 1), "SAME"),        # two 16-wide output groups
    ((2, 8, 8, 6), (5, 5, 6, 30), (1, 1, 1, 1), "SAME"),        # 4500 weights, 2-wide groups
    ((1, 1, 1, 1), (1, 1, 1, 1), (1, 1, 1, 1), "SAME"),
    ((1, 2, 2, 3), (3, 3, 3, 4), (1, 1, 1, 1), "VALID"),        # empty output: zero input/filter gradients
]


@pytest.mark.parametrize("xs,ws,strides,padding", DIRECT)
def test_conv2d_direct_bitexact(otf, port, xs, ws, strides, padding):
    x, w = _inputs(5, xs, ws)
    ry = port.conv2d(x, w, strides, padding)
    assert_bitexact(to_np(otf.conv2d(_cuda(x), _cuda(w), strides=strides, padding=padding)), ry, "fwd")
    dy = np.random.default_rng(6).standard_normal(ry.shape).astype(np.float32)
    dx = otf.conv2d_backprop_input(list(xs), _cuda(w), _cuda(dy), strides=strides, padding=padding)
    assert_bitexact(to_np(dx), port.conv2d_backprop_input(xs, w, dy, strides, padding), "dgrad")
    dw = otf.conv2d_backprop_filter(_cuda(x), list(ws), _cuda(dy), strides=strides, padding=padding)
    assert_close(to_np(dw), port.conv2d_backprop_filter(x, ws, dy, strides, padding), what="wgrad")


def test_conv2d_direct_unaligned_views(otf, port):
    """Tensors one float into their buffers: the scalar-load / scalar-store paths."""
    x, w = _inputs(7, (2, 6, 6, 4), (3, 3, 4, 8))
    st = (1, 1, 1, 1)
    ry = port.conv2d(x, w, st, "SAME")
    dy = np.random.default_rng(8).standard_normal(ry.shape).astype(np.float32)

    def view(a):
        base = torch.zeros(a.size + 1, device="cuda")
        base[1:] = _cuda(a).reshape(-1)
        return base[1:].view(a.shape)

    assert_bitexact(to_np(otf.conv2d(view(x), view(w), strides=st, padding="SAME")), ry, "fwd")
    dx = otf.conv2d_backprop_input(list(x.shape), view(w), view(dy), strides=st, padding="SAME")
    assert_bitexact(to_np(dx), port.conv2d_backprop_input(x.shape, w, dy, st, "SAME"), "dgrad")
    dw = otf.conv2d_backprop_filter(view(x), list(w.shape), view(dy), strides=st, padding="SAME")
    assert_close(to_np(dw), port.conv2d_backprop_filter(x, w.shape, dy, st, "SAME"), what="wgrad")


def test_conv2d_direct_large_batch(otf, port):
    """The uwb_loc_v3 refinement at batch 64: forward and input gradient bit
    for bit; the filter gradient (a sum over 55k pixels) within tolerance."""
    x, w = _inputs(9, (64, 36, 24, 16), (3, 3, 16, 16))
    st = (1, 1, 1, 1)
    ry = port.conv2d(x, w, st, "SAME")
    assert_bitexact(to_np(otf.conv2d(_cuda(x), _cuda(w), strides=st, padding="SAME")), ry, "fwd")
    dy = np.random.default_rng(10).standard_normal(ry.shape).astype(np.float32)
    dx = otf.conv2d_backprop_input(list(x.shape), _cuda(w), _cuda(dy), strides=st, padding="SAME")
    assert_bitexact(to_np(dx), port.conv2d_backprop_input(x.shape, w, dy, st, "SAME"), "dgrad")
    dw = otf.conv2d_backprop_filter(_cuda(x), list(w.shape), _cuda(dy), strides=st, padding="SAME")
    assert_close(to_np(dw), port.conv2d_backprop_filter(x, w.shape, dy, st, "SAME"), what="wgrad")


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
