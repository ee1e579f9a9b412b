"""The training step's loss and optimizer kernels against Keras's formulas
(oracle/keras_step.py): the MSE loss and its gradient within the fp32
tolerance of float64, Adam's moment slots bit for bit and its parameters
within the ulps that ``beta ** t`` leaves; the device step counter under
CUDA-graph replay; several launches for more than 24 tensors; unaligned and
ragged sizes."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_bitexact, to_np
from oracle.keras_step import adam_update_f32, mse_loss_f64, mse_loss_grad_f64

pytestmark = pytest.mark.gpu


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


@pytest.mark.parametrize("n", [1, 3, 4, 5, 4097, 131072, 1 << 20, 3 * (1 << 19) + 7])
def test_mse_loss_and_grad(otf, n):
    from opencl_tf._library import step_ops
    rng = np.random.default_rng(n)
    p = rng.uniform(0, 1, n).astype(np.float32)
    t = rng.uniform(0, 1, n).astype(np.float32)
    pd = _cuda(p).requires_grad_(True)
    loss = step_ops.opencl_mse_loss(pd, _cuda(t))
    loss.backward()
    want = mse_loss_f64(p, t)
    assert abs(float(loss) - want) <= 1e-6 * want, (float(loss), want)
    g = to_np(pd.grad)
    gw = mse_loss_grad_f64(p, t)
    assert np.abs(g - gw).max() <= 2e-7 * np.abs(gw).max() + 1e-30


def test_mse_unaligned_views_and_errors(otf):
    from opencl_tf import errors
    from opencl_tf._library import step_ops
    rng = np.random.default_rng(1)
    base_p = _cuda(rng.standard_normal(10001))
    base_t = _cuda(rng.standard_normal(10001))
    p, t = base_p[1:], base_t[1:]  # 4-byte offset: the scalar path
    loss = step_ops.opencl_mse_loss(p, t)
    want = mse_loss_f64(to_np(p), to_np(t))
    assert abs(float(loss) - want) <= 1e-6 * want
    g = step_ops.opencl_mse_loss_grad(p, t, torch.ones((), device="cuda"))
    assert np.abs(to_np(g) - mse_loss_grad_f64(to_np(p), to_np(t))).max() <= 1e-6 * float(np.abs(to_np(g)).max())
    with pytest.raises(errors.InvalidArgumentError):
        step_ops.opencl_mse_loss(p, t[:-1])
    with pytest.raises(errors.InvalidArgumentError):
        step_ops.opencl_mse_loss(torch.empty(0, device="cuda"), torch.empty(0, device="cuda"))


def test_mse_loss_deterministic(otf):
    from opencl_tf._library import step_ops
    rng = np.random.default_rng(2)
    p, t = _cuda(rng.standard_normal(1 << 20)), _cuda(rng.standard_normal(1 << 20))
    a = step_ops.opencl_mse_loss(p, t)
    b = step_ops.opencl_mse_loss(p, t)
    assert torch.equal(a, b)


def _adam_case(sizes, seed=0, unaligned=()):
    rng = np.random.default_rng(seed)
    ps, gs = [], []
    for i, n in enumerate(sizes):
        p = rng.standard_normal(n).astype(np.float32)
        g = (rng.standard_normal(n) * 10.0 ** rng.integers(-6, 2)).astype(np.float32)
        if i in unaligned:  # a view one float into a larger buffer
            bp, bg = torch.zeros(n + 1, device="cuda"), torch.zeros(n + 1, device="cuda")
            bp[1:] = _cuda(p)
            bg[1:] = _cuda(g)
            ps.append(bp[1:])
            gs.append(bg[1:])
        else:
            ps.append(_cuda(p))
            gs.append(_cuda(g))
    return ps, gs


@pytest.mark.parametrize("sizes,unaligned", [
    ([1], ()),
    ([7, 2048, 2049, 4096 * 3 + 5], ()),
    ([1000, 0, 33, 65536], (0, 2)),
    ([5 + 3 * i for i in range(30)], (4, 17)),  # 30 tensors: two launches
])
def test_adam_matches_keras(otf, sizes, unaligned):
    from opencl_tf._library import adam_update
    ps, gs = _adam_case(sizes, seed=len(sizes), unaligned=unaligned)
    ms = [torch.zeros_like(p) for p in ps]
    vs = [torch.zeros_like(p) for p in ps]
    it = torch.zeros((), dtype=torch.int64, device="cuda")
    ticket = torch.zeros((), dtype=torch.int32, device="cuda")
    ref = [(to_np(p), np.zeros(p.numel(), np.float32), np.zeros(p.numel(), np.float32)) for p in ps]
    rng = np.random.default_rng(99)
    for step in range(4):
        if step:  # fresh gradients each step
            for g in gs:
                g.copy_(_cuda(rng.standard_normal(g.numel())))
        adam_update(ps, gs, ms, vs, 1e-3, 0.9, 0.999, 1e-7, it, ticket)
        ref = [adam_update_f32(rp, to_np(g), rm, rv, step) for (rp, rm, rv), g in zip(ref, gs)]
        torch.cuda.synchronize()
        assert int(it) == step + 1 and int(ticket) == 0
        for k, ((rp, rm, rv), p, m, v) in enumerate(zip(ref, ps, ms, vs)):
            assert_bitexact(to_np(m), rm, f"m[{k}] step {step}")
            assert_bitexact(to_np(v), rv, f"v[{k}] step {step}")
            d = np.abs(to_np(p).astype(np.float64) - rp)
            assert d.max(initial=0.0) <= 4e-7 * max(1.0, float(np.abs(rp).max(initial=0.0))), (k, step, d.max())


def test_adam_under_graph_replay(otf):
    """A captured update advances the device counter on every replay and
    equals the eager updates."""
    from opencl_tf.optimizers import Adam
    torch.manual_seed(0)
    a = [torch.randn(300, device="cuda", requires_grad=True), torch.randn(64, 3, device="cuda", requires_grad=True)]
    b = [t.detach().clone().requires_grad_(True) for t in a]
    grads = [torch.randn_like(t) for t in a]
    for t, g in zip(a, grads):
        t.grad = g.clone()
    for t, g in zip(b, grads):
        t.grad = g.clone()
    oa, ob = Adam(a), Adam(b)
    oa.step()  # warm
    ob.step()
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph):
            oa.step()
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(5):
        graph.replay()
        ob.step()
    torch.cuda.synchronize()
    assert int(oa.iterations) == 6 and int(ob.iterations) == 6
    for x, y in zip(a, b):
        assert torch.equal(x, y)
