"""BatchNorm parity on the GPU (reference tests: tests/test_batchnorm.py).
The per-channel reductions run in a different order than the reference's
serial loop, so statistics and reductions are within the fp32 tolerance;
given identical statistics the elementwise passes are bit-exact."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_bitexact, assert_close, to_np

pytestmark = pytest.mark.gpu


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def _inputs(seed, shape):
    rng = np.random.default_rng(seed)
    C = shape[-1]
    x = rng.standard_normal(shape).astype(np.float32)
    g = (rng.standard_normal(C) + 1.0).astype(np.float32)
    b = (rng.standard_normal(C) * 0.1).astype(np.float32)
    return x, g, b


@pytest.mark.parametrize("shape", [(4, 7, 7, 8), (2, 5, 5, 6), (3, 5, 5, 4), (1, 1, 1, 3), (2, 3, 3, 1),
                                   (8, 16, 16, 48), (4, 9, 7, 144), (2, 4, 4, 1100)])
def test_bn_training_forward(otf, port, shape):
    x, g, b = _inputs(0, shape)
    y, m, v = (to_np(t) for t in otf.batch_norm_training(_cuda(x), _cuda(g), _cuda(b)))
    ry, rm, rv = port.batch_norm_training(x, g, b)
    assert_close(m, rm, what="mean")
    assert_close(v, rv, what="var")
    assert_close(y, ry, what="y")
    # given the GPU's statistics the normalisation is the reference formula bit for bit
    assert_bitexact(y, port.batch_norm_inference(x, g, b, m, v), "normalize")


def test_bn_inference_forward_bitexact(otf, port):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 5, 5, 6)).astype(np.float32)
    g = (rng.standard_normal(6) + 1.0).astype(np.float32)
    b = (rng.standard_normal(6) * 0.1).astype(np.float32)
    m = (rng.standard_normal(6) * 0.5).astype(np.float32)
    v = (np.abs(rng.standard_normal(6)) + 0.1).astype(np.float32)
    got = to_np(otf.batch_norm_inference(_cuda(x), _cuda(g), _cuda(b), _cuda(m), _cuda(v)))
    assert_bitexact(got, port.batch_norm_inference(x, g, b, m, v), "bn inference")


@pytest.mark.parametrize("shape", [(3, 5, 5, 4), (4, 7, 7, 8), (8, 16, 16, 48), (2, 3, 3, 5)])
def test_bn_grad(otf, port, shape):
    x, g, _ = _inputs(2, shape)
    dy = np.random.default_rng(5).standard_normal(shape).astype(np.float32)
    _, m, v = port.batch_norm_training(x, g, np.zeros_like(g))
    gx, gg, gb = (to_np(t) for t in otf.batch_norm_grad(_cuda(dy), _cuda(x), _cuda(g), _cuda(m), _cuda(v)))
    rx, rg, rb = port.batch_norm_grad(dy, x, g, m, v)
    assert_close(gb, rb, what="grad_beta")
    assert_close(gg, rg, what="grad_gamma")
    assert_close(gx, rx, what="grad_x")


def test_bn_training_gradients_via_autograd(otf, port):
    """loss = 0.5*sum(y^2) as in the reference test (tests/test_batchnorm.py:71-101).
    Its true input gradient is ~0 (|y| is invariant to x), so dx is rounding
    noise on both sides; like the reference test, dx is compared with an
    absolute tolerance.  gamma / beta gradients are well conditioned."""
    x, g, b = _inputs(2, (3, 5, 5, 4))
    xt, gt, bt = (_cuda(a).requires_grad_(True) for a in (x, g, b))
    y, _, _ = otf.batch_norm_training(xt, gt, bt)
    (0.5 * (y * y).sum()).backward()
    ry, rm, rv = port.batch_norm_training(x, g, b)
    rx, rg, rb = port.batch_norm_grad(ry, x, g, rm, rv)
    np.testing.assert_allclose(to_np(xt.grad), rx, atol=1e-4, rtol=1e-4)
    assert_close(to_np(gt.grad), rg, what="dgamma")
    assert_close(to_np(bt.grad), rb, what="dbeta")


def test_bn_inference_has_no_gradient(otf):
    x = torch.randn(1, 2, 2, 3, device="cuda", requires_grad=True)
    c = torch.ones(3, device="cuda")
    y = otf.batch_norm_inference(x, c, c * 0, c * 0, c)
    with pytest.raises(LookupError):
        y.sum().backward()


def test_bn_deterministic(otf):
    x = torch.randn(64, 32, 16, 48, device="cuda")
    g, b = torch.ones(48, device="cuda"), torch.zeros(48, device="cuda")
    a = otf.batch_norm_training(x, g, b)
    c = otf.batch_norm_training(x, g, b)
    for u, w in zip(a, c):
        assert torch.equal(u, w)


def test_bn_bad_shapes(otf):
    x = torch.zeros(1, 2, 2, 3, device="cuda")
    with pytest.raises(otf.errors.InvalidArgumentError, match="gamma/beta size must equal channels"):
        otf.batch_norm_training(x, torch.ones(4, device="cuda"), torch.zeros(3, device="cuda"))
    with pytest.raises(otf.errors.InvalidArgumentError, match="NHWC"):
        otf.batch_norm_training(torch.zeros(2, 3, device="cuda"), torch.ones(3, device="cuda"),
                                torch.zeros(3, device="cuda"))
    with pytest.raises(otf.errors.InvalidArgumentError, match="matching NHWC shapes"):
        otf.batch_norm_grad(torch.zeros(1, 2, 2, 4, device="cuda"), x, torch.ones(3, device="cuda"),
                            torch.zeros(3, device="cuda"), torch.ones(3, device="cuda"))


def test_moving_statistics_update_rounding(otf):
    """The layer's moving-average update (reference opencl_tf/layers.py:189-194,
    three fp32 tensor ops) runs as one launch with the same rounding."""
    from opencl_tf import _library as L
    rng = np.random.default_rng(5)
    C = 37
    mm, mv, bm, bv = (rng.standard_normal(C).astype(np.float32) for _ in range(4))
    t = [torch.from_numpy(a.copy()).cuda() for a in (mm, mv, bm, bv)]
    L.batch_norm_update_moving(*t, 0.99)
    m32, om32 = np.float32(0.99), np.float32(1.0 - 0.99)
    want_m = (m32 * mm).astype(np.float32) + (om32 * bm).astype(np.float32)
    want_v = (m32 * mv).astype(np.float32) + (om32 * bv).astype(np.float32)
    assert np.array_equal(t[0].cpu().numpy(), want_m)
    assert np.array_equal(t[1].cpu().numpy(), want_v)
    assert np.array_equal(t[2].cpu().numpy(), bm) and np.array_equal(t[3].cpu().numpy(), bv)


@pytest.mark.parametrize("shape", [(4, 6, 5, 8), (3, 7, 5, 3), (2, 64, 32, 48)])
def test_fused_bn_relu_equals_the_two_ops(otf, shape):
    """BatchNormTraining -> Relu fused (forward) and ReluGrad -> BatchNormGrad
    fused (backward, mask recomputed from x) equal the reference ops in
    sequence bit for bit."""
    from opencl_tf import _library as L
    rng = np.random.default_rng(11)
    C = shape[-1]
    x = torch.from_numpy(rng.standard_normal(shape).astype(np.float32) * 2 + 0.3).cuda()
    g = torch.from_numpy(rng.standard_normal(C).astype(np.float32)).cuda()
    b = torch.from_numpy(rng.standard_normal(C).astype(np.float32)).cuda()
    dz = torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).cuda()
    y, m, v = L._k_batch_norm_training(x, g, b, 1e-3)
    z_ref = L._k_relu(y)
    z, m2, v2 = L._k_batch_norm_relu_training(x, g, b, 1e-3)
    assert torch.equal(z, z_ref) and torch.equal(m, m2) and torch.equal(v, v2)
    dy = L._k_relu_grad(dz, y)
    dx_ref, dg_ref, db_ref = L._k_batch_norm_grad(dy, x, g, m, v, 1e-3)
    dx, dg, db = L._k_batch_norm_relu_grad(dz, x, g, b, m, v, 1e-3)
    assert torch.equal(dx, dx_ref) and torch.equal(dg, dg_ref) and torch.equal(db, db_ref)
