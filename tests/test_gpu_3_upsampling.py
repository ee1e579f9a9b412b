"""Bilinear UpSampling2D parity on the GPU (reference tests:
tests/test_upsampling.py).  The source-coordinate arithmetic (clamped corner
indices and fractions) and the forward blend are bit-exact against the
reference formula; the backward gather adds in the order of a
single-threaded reference run and is bit-exact against it."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_bitexact, assert_close, to_np

pytestmark = pytest.mark.gpu


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


@pytest.mark.parametrize("in_size,scale", [(4, 2), (4, 3), (5, 2), (7, 2), (1, 3), (6, 1), (3, 4), (8, 2),
                                           (13, 5), (256, 2), (1000, 3)])
def test_coordinate_math_bitexact(otf, in_size, scale):
    from oracle.oracle import f64
    from opencl_tf._library import upsampling_coords
    out = in_size * scale
    lo, hi, frac = (to_np(t) for t in upsampling_coords(in_size, out))
    rlo, rhi, rfrac = f64.upsample_coords(in_size, out)
    assert np.array_equal(lo, rlo) and np.array_equal(hi, rhi)
    assert_bitexact(frac, rfrac, "fractions")


def test_upsampling_forward_2x2(otf, port):
    x = np.random.default_rng(0).standard_normal((2, 4, 4, 3)).astype(np.float32)
    assert_bitexact(to_np(otf.upsampling_bilinear_2d(_cuda(x), size=[2, 2])),
                    port.upsampling_bilinear_2d(x, [2, 2]), "up 2x2")


@pytest.mark.parametrize("sy,sx", [(2, 2), (3, 3), (2, 3), (4, 2)])
def test_upsampling_forward_factors(otf, port, sy, sx):
    x = np.random.default_rng(42).standard_normal((2, 4, 6, 8)).astype(np.float32)
    assert_bitexact(to_np(otf.upsampling_bilinear_2d(_cuda(x), size=[sy, sx])),
                    port.upsampling_bilinear_2d(x, [sy, sx]), "up")


def test_upsampling_agrees_with_torch_interpolate(otf):
    x = np.random.default_rng(1).standard_normal((2, 5, 7, 4)).astype(np.float32)
    got = to_np(otf.upsampling_bilinear_2d(_cuda(x), size=[2, 2]))
    want = torch.nn.functional.interpolate(torch.from_numpy(x).permute(0, 3, 1, 2), size=(10, 14), mode="bilinear",
                                           align_corners=False).permute(0, 2, 3, 1).numpy()
    np.testing.assert_allclose(got, want, atol=1e-5)


def test_upsampling_single_pixel(otf, port):
    x = np.array([[[[3.0, -1.0, 2.5]]]], np.float32)
    got = to_np(otf.upsampling_bilinear_2d(_cuda(x), size=[3, 4]))
    np.testing.assert_allclose(got, np.broadcast_to(x, got.shape), atol=1e-4)
    assert_bitexact(got, port.upsampling_bilinear_2d(x, [3, 4]), "single pixel")


def test_upsampling_1x_is_identity(otf):
    x = np.random.default_rng(5).standard_normal((2, 6, 8, 4)).astype(np.float32)
    assert_bitexact(to_np(otf.upsampling_bilinear_2d(_cuda(x), size=[1, 1])), x, "identity")


@pytest.mark.parametrize("shape,size", [((2, 4, 4, 3), (2, 2)), ((2, 3, 5, 4), (2, 2)), ((2, 3, 5, 4), (3, 2)),
                                        ((1, 1, 1, 5), (3, 4)), ((2, 4, 6, 8), (4, 2)), ((256, 4, 4, 8), (2, 2)),
                                        ((3, 7, 5, 6), (3, 3)),
                                        # images over 48 KB of dy take the global-memory gather
                                        ((2, 18, 12, 16), (2, 2)), ((1, 25, 25, 9), (2, 2)),
                                        ((2, 40, 40, 8), (2, 2)), ((1, 33, 30, 5), (3, 2))])
def test_upsampling_grad_matches_single_thread_reference(otf, port1, shape, size):
    rng = np.random.default_rng(3)
    x = rng.standard_normal(shape).astype(np.float32)
    dy = rng.standard_normal((shape[0], shape[1] * size[0], shape[2] * size[1], shape[3])).astype(np.float32)
    got = to_np(otf.upsampling_bilinear_2d_grad(_cuda(dy), list(shape), size=list(size)))
    assert_bitexact(got, port1.upsampling_bilinear_2d_grad(dy, shape, size), "up grad")


def test_upsampling_gradient_via_autograd(otf, port1):
    x = np.random.default_rng(2).standard_normal((2, 4, 4, 3)).astype(np.float32)
    xt = _cuda(x).requires_grad_(True)
    y = otf.upsampling_bilinear_2d(xt, size=[2, 2])
    (0.5 * (y * y).sum()).backward()
    want = port1.upsampling_bilinear_2d_grad(to_np(y), x.shape, [2, 2])
    assert_bitexact(to_np(xt.grad), want, "autograd")
    # and the adjoint of torch's bilinear resize
    xr = torch.from_numpy(x).permute(0, 3, 1, 2).requires_grad_(True)
    yr = torch.nn.functional.interpolate(xr, size=(8, 8), mode="bilinear", align_corners=False)
    (0.5 * (yr * yr).sum()).backward()
    assert_close(to_np(xt.grad), xr.grad.permute(0, 2, 3, 1).numpy(), what="vs torch")


def test_upsampling_grad_deterministic(otf):
    dy = torch.randn(64, 16, 16, 8, device="cuda")
    a = otf.upsampling_bilinear_2d_grad(dy, [64, 8, 8, 8], size=[2, 2])
    b = otf.upsampling_bilinear_2d_grad(dy, [64, 8, 8, 8], size=[2, 2])
    assert torch.equal(a, b)


def test_upsampling_bad_args(otf):
    x = torch.zeros(1, 2, 2, 3, device="cuda")
    with pytest.raises(otf.errors.InvalidArgumentError, match="exactly 2 elements"):
        otf.upsampling_bilinear_2d(x, size=[2])
    with pytest.raises(otf.errors.InvalidArgumentError, match=">= 1"):
        otf.upsampling_bilinear_2d(x, size=[0, 2])
    with pytest.raises(otf.errors.InvalidArgumentError, match="shape mismatch"):
        otf.upsampling_bilinear_2d_grad(torch.zeros(1, 4, 4, 3, device="cuda"), [1, 2, 3, 3], size=[2, 2])
