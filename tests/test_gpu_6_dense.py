"""Dense parity on the GPU (reference tests: tests/test_dense.py).  Forward,
input and weight gradients run on the tcgen05 3xTF32 engine (fp32
tolerance); the bias gradient sums in the reference's order (bit-exact)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_bitexact, assert_close, rel_errs, to_np

pytestmark = pytest.mark.gpu


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def test_dense_forward_basic(otf, port):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((4, 8)).astype(np.float32)
    W = rng.standard_normal((8, 16)).astype(np.float32)
    b = rng.standard_normal((16,)).astype(np.float32)
    assert_close(to_np(otf.dense(_cuda(x), _cuda(W), _cuda(b))), port.dense(x, W, b), what="dense")


@pytest.mark.parametrize("batch,in_f,out_f", [(1, 1, 1), (8, 32, 64), (16, 64, 32), (3, 128, 10), (256, 1152, 128),
                                              (130, 300, 270), (5, 0, 3), (2, 4097, 17),
                                              # ragged sizes with 16-byte-aligned rows (TMA-fed engine)
                                              (130, 300, 276), (3, 4100, 20), (300, 20, 36), (257, 2052, 132)])
def test_dense_all_ops(otf, port, batch, in_f, out_f):
    rng = np.random.default_rng(42)
    x = rng.standard_normal((batch, in_f)).astype(np.float32)
    W = rng.standard_normal((in_f, out_f)).astype(np.float32)
    b = rng.standard_normal((out_f,)).astype(np.float32)
    dy = rng.standard_normal((batch, out_f)).astype(np.float32)
    assert_close(to_np(otf.dense(_cuda(x), _cuda(W), _cuda(b))), port.dense(x, W, b), what="fwd")
    if in_f:
        assert_close(to_np(otf.dense_backprop_input(_cuda(dy), _cuda(W))), port.dense_backprop_input(dy, W),
                     what="dgrad")
        assert_close(to_np(otf.dense_backprop_weight(_cuda(x), _cuda(dy))), port.dense_backprop_weight(x, dy),
                     what="wgrad")
    assert_bitexact(to_np(otf.dense_backprop_bias(_cuda(dy))), port.dense_backprop_bias(dy), "bias grad")


def test_dense_gradient_via_autograd(otf, port):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((6, 20)).astype(np.float32)
    W = rng.standard_normal((20, 9)).astype(np.float32)
    b = rng.standard_normal((9,)).astype(np.float32)
    xt, Wt, bt = (_cuda(a).requires_grad_(True) for a in (x, W, b))
    y = otf.dense(xt, Wt, bt)
    (0.5 * (y * y).sum()).backward()
    ry = port.dense(x, W, b)
    assert_close(to_np(xt.grad), port.dense_backprop_input(ry, W), what="dx")
    assert_close(to_np(Wt.grad), port.dense_backprop_weight(x, ry), what="dW")
    assert_close(to_np(bt.grad), port.dense_backprop_bias(ry), what="db")


def _bits(t):
    return t.detach().contiguous().view(torch.int32)


@pytest.mark.parametrize("batch,in_f,out_f", [(256, 1152, 128),  # the README head: TMA engine, one split
                                              (257, 2052, 132),  # TMA engine, split-K reduce
                                              (130, 300, 270),   # fallback engine, one split (in-place ReLU)
                                              (2, 4097, 17),     # fallback engine, split-K reduce
                                              (5, 0, 3), (1, 1, 1)])
def test_dense_relu_matches_pair(otf, batch, in_f, out_f):
    """The fused Dense -> ReLU against OpenclDense then OpenclRelu: the same
    bits forward (NaN rows included) and backward."""
    from opencl_tf._library import fused_ops, raw_ops
    rng = np.random.default_rng(batch + in_f + out_f)
    x = rng.standard_normal((batch, in_f)).astype(np.float32)
    if in_f:
        x[0, 0] = np.nan  # row 0 of the sum is NaN; ReLU maps it to 0 on both paths
    W = rng.standard_normal((in_f, out_f)).astype(np.float32)
    b = rng.standard_normal((out_f,)).astype(np.float32)
    dz = _cuda(rng.standard_normal((batch, out_f)))
    fused = [_cuda(a).requires_grad_(True) for a in (x, W, b)]
    pair = [_cuda(a).requires_grad_(True) for a in (x, W, b)]
    zf = fused_ops.opencl_dense_relu(*fused)
    zp = raw_ops.opencl_relu(raw_ops.opencl_dense(*pair))
    assert torch.equal(_bits(zf), _bits(zp))
    assert not torch.isnan(zf).any()
    zf.backward(dz)
    zp.backward(dz)
    for a, c, what in zip(fused, pair, ("dx", "dW", "db")):
        assert torch.equal(_bits(a.grad), _bits(c.grad)), what


def test_dense_relu_bad_args(otf):
    from opencl_tf._library import fused_ops
    x = torch.zeros(2, 3, device="cuda")
    with pytest.raises(otf.errors.InvalidArgumentError, match="in_features"):
        fused_ops.opencl_dense_relu(x, torch.zeros(4, 5, device="cuda"), torch.zeros(5, device="cuda"))
    with pytest.raises(otf.errors.InvalidArgumentError, match="out_features"):
        fused_ops.opencl_dense_relu(x, torch.zeros(3, 5, device="cuda"), torch.zeros(4, device="cuda"))


def test_stress_gemm_reduced(otf):
    """The stress GEMM's shape family (M=8192, K=N=4096 at full size) at a
    quarter of each dimension, against float64."""
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(2048, 1024, device="cuda", generator=g)
    W = torch.randn(1024, 1024, device="cuda", generator=g)
    b = torch.zeros(1024, device="cuda")
    y = otf.dense(x, W, b)
    want = (x.double() @ W.double()).cpu().numpy()
    mx, l2 = rel_errs(to_np(y), want)
    assert mx <= 1e-4 and l2 <= 1e-5, (mx, l2)


def test_dense_bad_args(otf):
    x = torch.zeros(2, 3, device="cuda")
    with pytest.raises(otf.errors.InvalidArgumentError, match="in_features"):
        otf.dense(x, torch.zeros(4, 5, device="cuda"), torch.zeros(5, device="cuda"))
    with pytest.raises(otf.errors.InvalidArgumentError, match="out_features"):
        otf.dense(x, torch.zeros(3, 5, device="cuda"), torch.zeros(4, device="cuda"))
    with pytest.raises(otf.errors.InvalidArgumentError, match="rank 2"):
        otf.dense(x[0], torch.zeros(3, 5, device="cuda"), torch.zeros(5, device="cuda"))
    with pytest.raises(otf.errors.InvalidArgumentError, match="same batch size"):
        otf.dense_backprop_weight(x, torch.zeros(3, 5, device="cuda"))
