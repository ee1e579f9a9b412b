"""The network-level oracle (oracle/netstep.py) pinned: the README network's
training step composed from the restated kernels equals the same step
composed from the reference's own kernels, bit for bit, and agrees with a
float64 torch autograd of the same network."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_bitexact, assert_close


@pytest.fixture(scope="module")
def setup():
    from opencl_tf.model import build_model
    from oracle.netstep import params_of
    torch.manual_seed(0)
    m = build_model()
    rng = np.random.default_rng(3)
    x = rng.uniform(0, 1, (1, 64, 64, 3)).astype(np.float32)
    t = rng.uniform(0, 1, (1, 8, 8, 8)).astype(np.float32)
    return params_of(m), x, t


def test_netstep_port_equals_reference_kernels(setup, port, ref):
    from oracle.netstep import train_grads
    p, x, t = setup
    lp, op, gp = train_grads(port, p, x, t)
    lr, orf, gr = train_grads(ref, p, x, t)
    assert lp == lr
    assert_bitexact(op, orf, "output")
    for k in ("stem_w", "stem_g", "stem_b", "dense_w", "dense_b"):
        assert_bitexact(gp[k], gr[k], k)
    for a, b in zip(gp["blocks"], gr["blocks"]):
        for k in a:
            assert_bitexact(a[k], b[k], k)


def test_netstep_against_float64_autograd(setup, port):
    """Same network in torch float64 (NCHW convs, align_corners=False
    bilinear, biased-variance BN) -- an independent check of the wiring."""
    from oracle.netstep import train_grads
    p, x, t = setup
    loss, out, g = train_grads(port, p, x, t)
    tt = lambda a: torch.tensor(np.asarray(a), dtype=torch.float64, requires_grad=True)  # noqa: E731
    P = {"stem_w": tt(p["stem_w"]), "stem_g": tt(p["stem_g"]), "stem_b": tt(p["stem_b"]),
         "dense_w": tt(p["dense_w"]), "dense_b": tt(p["dense_b"])}
    B = [{k: tt(v) for k, v in b.items()} for b in p["blocks"]]

    def conv(z, w, stride, groups=1):
        kh, kw = w.shape[0], w.shape[1]
        H, W = z.shape[2], z.shape[3]
        oh, ow = -(-H // stride[0]), -(-W // stride[1])
        ph = max((oh - 1) * stride[0] + kh - H, 0)
        pw = max((ow - 1) * stride[1] + kw - W, 0)
        z = torch.nn.functional.pad(z, (pw // 2, pw - pw // 2, ph // 2, ph - ph // 2))
        return torch.nn.functional.conv2d(z, w.permute(3, 2, 0, 1) if groups == 1 else w.permute(2, 3, 0, 1),
                                          stride=stride, groups=groups)

    def bn(z, gm, bt):
        m = z.mean(dim=(0, 2, 3), keepdim=True)
        v = (z * z).mean(dim=(0, 2, 3), keepdim=True) - m * m
        return gm.view(1, -1, 1, 1) * (z - m) / torch.sqrt(v + 1e-3) + bt.view(1, -1, 1, 1)

    z = torch.tensor(x, dtype=torch.float64).permute(0, 3, 1, 2)
    z = torch.relu(bn(conv(z, P["stem_w"], (1, 2)), P["stem_g"], P["stem_b"]))
    for b in B:
        z = torch.relu(bn(conv(z, b["dw"], (2, 2), groups=z.shape[1]), b["g1"], b["b1"]))
        z = torch.relu(bn(conv(z, b["pw"], (1, 1)), b["g2"], b["b2"]))
    z = z.permute(0, 2, 3, 1).reshape(1, -1)
    z = torch.relu(z @ P["dense_w"] + P["dense_b"]).reshape(1, 4, 4, 8).permute(0, 3, 1, 2)
    z = torch.nn.functional.interpolate(z, scale_factor=2, mode="bilinear", align_corners=False)
    o = torch.sigmoid(z).permute(0, 2, 3, 1)
    L = torch.mean((o - torch.tensor(t, dtype=torch.float64)) ** 2)
    L.backward()
    assert abs(loss - float(L)) < 1e-6 * abs(float(L))
    assert_close(out, o.detach().numpy(), 1e-5, 1e-6, "output")
    assert_close(g["stem_w"], P["stem_w"].grad.numpy(), 1e-3, 1e-4, "stem_w")
    assert_close(g["dense_w"], P["dense_w"].grad.numpy(), 1e-3, 1e-4, "dense_w")
    assert_close(g["blocks"][1]["pw"], B[1]["pw"].grad.numpy(), 1e-3, 1e-4, "pw2")


def test_keras_adam_restatement_against_float64():
    """The float32 Keras Adam restatement stays within fp32 rounding of the
    same formula in float64, over several steps."""
    from oracle.keras_step import adam_update_f32
    rng = np.random.default_rng(5)
    p = rng.standard_normal(1000).astype(np.float32)
    m = np.zeros_like(p)
    v = np.zeros_like(p)
    p64, m64, v64 = p.astype(np.float64), np.zeros(1000), np.zeros(1000)
    for step in range(5):
        g = rng.standard_normal(1000).astype(np.float32)
        p, m, v = adam_update_f32(p, g, m, v, step)
        t = step + 1
        alpha = 1e-3 * np.sqrt(1 - 0.999 ** t) / (1 - 0.9 ** t)
        m64 = m64 + (g - m64) * (1 - 0.9)
        v64 = v64 + (g.astype(np.float64) ** 2 - v64) * (1 - 0.999)
        p64 = p64 - m64 * alpha / (np.sqrt(v64) + 1e-7)
        assert np.abs(m - m64).max() <= 1e-6 * np.abs(m64).max()
        assert np.abs(v - v64).max() <= 1e-6 * np.abs(v64).max()
        assert np.abs(p - p64).max() <= 1e-6 * np.abs(p64).max()
    # the first step moves every parameter by about lr (Adam's normalised step)
    p0 = rng.standard_normal(100).astype(np.float32)
    g0 = rng.standard_normal(100).astype(np.float32)
    p1, _, _ = adam_update_f32(p0, g0, np.zeros(100, np.float32), np.zeros(100, np.float32), 0)
    assert np.allclose(np.abs(p1 - p0), 1e-3, rtol=1e-3)


def test_keras_mse_restatement():
    from oracle.keras_step import mse_loss_f64, mse_loss_grad_f64
    p = np.array([[1.0, 2.0], [3.0, 5.0]], np.float32)
    t = np.array([[0.0, 2.0], [1.0, 1.0]], np.float32)
    assert mse_loss_f64(p, t) == (1 + 0 + 4 + 16) / 4
    assert np.array_equal(mse_loss_grad_f64(p, t), 2 * (p - t) / 4)
