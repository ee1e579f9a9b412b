"""ReLU / Sigmoid parity on the GPU (reference tests: tests/test_relu.py,
tests/test_sigmoid.py).  ReLU forward/backward and SigmoidGrad are bit-exact
against the oracle; Sigmoid within the fp32 tolerance (expf differs by ulps)."""
from __future__ import annotations

import threading

import numpy as np
import pytest
import torch

from helpers import assert_bitexact, assert_close, to_np

pytestmark = pytest.mark.gpu


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


EDGE = np.array([-100.0, 100.0, 0.0, -0.0, -30.0, 30.0, np.nan, np.inf, -np.inf, 1e-38, -1e-38,
                 3.4e38, -3.4e38, 1.0, -1.0], np.float32)


def test_relu_forward(otf, port):
    x = np.random.default_rng(0).standard_normal((2, 5, 5, 3)).astype(np.float32)
    assert_bitexact(to_np(otf.relu(_cuda(x))), port.relu(x), "relu")


def test_relu_edge_values_bitexact(otf, port):
    assert_bitexact(to_np(otf.relu(_cuda(EDGE))), port.relu(EDGE), "relu edges")


@pytest.mark.parametrize("n", [1, 3, 4, 5, 1023, 4096 + 3, 1 << 20])
def test_relu_sizes_and_grad_bitexact(otf, port, n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    x[::7] = 0.0
    g = rng.standard_normal(n).astype(np.float32)
    assert_bitexact(to_np(otf.relu(_cuda(x))), port.relu(x), "relu")
    assert_bitexact(to_np(otf.relu_grad(_cuda(g), _cuda(x))), port.relu_grad(g, x), "relu_grad")


def test_relu_misaligned_views(otf, port):
    x = np.random.default_rng(3).standard_normal(1001).astype(np.float32)
    xd = _cuda(x)[1:]  # 4-byte offset: the scalar path
    assert_bitexact(to_np(otf.relu(xd)), port.relu(x[1:]), "relu misaligned")


def test_relu_gradient_via_autograd(otf, port):
    x = np.random.default_rng(1).standard_normal((2, 5, 5, 3)).astype(np.float32)
    xt = _cuda(x).requires_grad_(True)
    y = otf.relu(xt)
    (0.5 * (y * y).sum()).backward()
    want = port.relu_grad(port.relu(x), x)
    assert_bitexact(to_np(xt.grad), want, "relu grad")


def test_relu_at_zero_grad_is_zero(otf):
    x = torch.zeros(4, device="cuda", requires_grad=True)
    otf.relu(x).sum().backward()
    assert torch.equal(x.grad, torch.zeros_like(x))


def test_sigmoid_forward(otf, port):
    x = np.random.default_rng(0).standard_normal((2, 5, 5, 3)).astype(np.float32)
    assert_close(to_np(otf.sigmoid(_cuda(x))), port.sigmoid(x), what="sigmoid")


@pytest.mark.parametrize("shape", [(1, 1, 1, 1), (4, 8, 8, 16), (8, 4, 4, 32), (3, 1, 1, 64)])
def test_sigmoid_forward_shapes(otf, port, shape):
    x = np.random.default_rng(42).standard_normal(shape).astype(np.float32)
    assert_close(to_np(otf.sigmoid(_cuda(x))), port.sigmoid(x), what="sigmoid")


def test_sigmoid_extreme_values(otf, port):
    x = np.array([[-100.0, 100.0, 0.0, -30.0, 30.0]], np.float32)
    got = to_np(otf.sigmoid(_cuda(x)))
    np.testing.assert_allclose(got, port.sigmoid(x), rtol=1e-6, atol=1e-30)
    assert got[0, 0] == 0.0 and got[0, 1] == 1.0


def test_sigmoid_grad_bitexact(otf, port):
    rng = np.random.default_rng(2)
    y = np.clip(rng.uniform(0.01, 0.99, (2, 4, 4, 3)).astype(np.float32), 0.01, 0.99)
    dy = rng.standard_normal((2, 4, 4, 3)).astype(np.float32)
    assert_bitexact(to_np(otf.sigmoid_grad(_cuda(y), _cuda(dy))), port.sigmoid_grad(y, dy), "sigmoid_grad")


def test_sigmoid_gradient_via_autograd_uses_output(otf, port):
    x = np.random.default_rng(1).standard_normal((3, 6, 6, 4)).astype(np.float32)
    xt = _cuda(x).requires_grad_(True)
    y = otf.sigmoid(xt)
    (0.5 * (y * y).sum()).backward()
    yd = to_np(y)
    assert_bitexact(to_np(xt.grad), port.sigmoid_grad(yd, yd), "sigmoid grad from output")


def test_sigmoid_concurrent_threads(otf):
    """16 host threads x 10 calls each on their own streams (the reference's
    race test, tests/test_sigmoid.py:119-162)."""
    rng = np.random.default_rng(99)
    inputs = [rng.standard_normal((4, 8, 8, 8)).astype(np.float32) for _ in range(16)]
    refs = [1.0 / (1.0 + np.exp(-x.astype(np.float64))) for x in inputs]
    errors = []

    def worker(i):
        try:
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                x = _cuda(inputs[i])
                for _ in range(10):
                    y = to_np(otf.sigmoid(x))
                    if np.abs(y - refs[i]).max() > 1e-6:
                        errors.append(i)
        except Exception as e:  # noqa: BLE001
            errors.append(repr(e))

    ts = [threading.Thread(target=worker, args=(i,)) for i in range(16)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errors, errors


def test_sigmoid_stress_sequential(otf):
    x = torch.from_numpy(np.random.default_rng(77).standard_normal((8, 16, 16, 4)).astype(np.float32)).cuda()
    first = otf.sigmoid(x)
    for _ in range(200):
        assert torch.equal(otf.sigmoid(x), first)


def test_shape_mismatch_is_invalid_argument(otf):
    with pytest.raises(otf.errors.InvalidArgumentError, match="equal shape"):
        otf.relu_grad(torch.zeros(3, device="cuda"), torch.zeros(4, device="cuda"))
    with pytest.raises(otf.errors.InvalidArgumentError, match="equal shape"):
        otf.sigmoid_grad(torch.zeros(3, device="cuda"), torch.zeros(4, device="cuda"))


def test_empty_tensors(otf):
    e = torch.empty(0, 3, device="cuda")
    assert otf.relu(e).shape == e.shape
    assert otf.sigmoid(e).shape == e.shape
