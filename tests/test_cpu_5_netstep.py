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


def _uwb_batch(n, seed=0):
    """The reference example's synthetic batch: IQ ~ N(0, 1), heatmap ~ U(0, 1)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n, 8, 6, 3, 16, 2)).astype(np.float32)
    t = rng.uniform(0, 1, (n, 36, 24, 1)).astype(np.float32)
    return x, t


@pytest.fixture(scope="module")
def uwb():
    from opencl_tf.model import build_uwb_loc_v3
    from oracle.netstep import seq_of
    torch.manual_seed(0)
    return seq_of(build_uwb_loc_v3())


def test_stage_composer_equals_readme_step(setup, port):
    """The generic stage-list composer reproduces the README step bit for bit."""
    from opencl_tf.model import build_model
    from oracle.netstep import seq_of, seq_train_grads, train_grads
    p, x, t = setup
    torch.manual_seed(0)
    seq = seq_of(build_model())
    l0, o0, g0 = train_grads(port, p, x, t)
    l1, o1, g1 = seq_train_grads(port, seq, x, t)
    assert l0 == l1
    assert_bitexact(o0, o1, "output")
    assert_bitexact(g1[0]["w"], g0["stem_w"], "stem_w")
    assert_bitexact(g1[1]["g"], g0["stem_g"], "stem_g")
    assert_bitexact(g1[-5]["w"], g0["dense_w"], "dense_w")
    for j, gb in enumerate(g0["blocks"]):
        k = 3 + 6 * j
        assert_bitexact(g1[k]["w"], gb["dw"], f"b{j}.dw")
        assert_bitexact(g1[k + 1]["b"], gb["b1"], f"b{j}.b1")
        assert_bitexact(g1[k + 3]["w"], gb["pw"], f"b{j}.pw")
        assert_bitexact(g1[k + 4]["g"], gb["g2"], f"b{j}.g2")


def test_uwb_step_port_equals_reference_kernels(uwb, port, ref):
    from oracle.netstep import seq_forward_inference, seq_train_grads, uwb_input
    x, t = _uwb_batch(4)
    xi = uwb_input(x)
    lp, op, gp = seq_train_grads(port, uwb, xi, t)
    lr, orf, gr = seq_train_grads(ref, uwb, xi, t)
    assert lp == lr
    assert_bitexact(op, orf, "output")
    for i, (a, b) in enumerate(zip(gp, gr)):
        for k in a:
            assert_bitexact(a[k], b[k], f"stage {i} {k}")
    assert_bitexact(seq_forward_inference(port, uwb, xi), seq_forward_inference(ref, uwb, xi), "inference")


def test_uwb_step_against_float64_autograd(uwb, port):
    """The uwb_loc_v3 wiring (permute, 1x1-spatial BatchNorms, the two-step
    upsampling head) against float64 torch autograd.  The oracle's serial fp32
    BatchNorm sums (the reference's order) leave ~2e-4 relative error in the
    gradients at this batch, growing with the count reduced; a wiring mistake
    is O(1)."""
    from oracle.netstep import seq_train_grads, seq_train_grads_f64, uwb_input
    x, t = _uwb_batch(16, seed=1)
    xi = uwb_input(x)
    loss, out, g = seq_train_grads(port, uwb, xi, t)
    e_loss, e_out, e_g = seq_train_grads_f64(uwb, xi, t)
    assert abs(loss - e_loss) < 1e-6 * abs(e_loss)
    assert_close(out, e_out, 1e-5, 1e-5, "output")
    for i, (a, b) in enumerate(zip(g, e_g)):
        for k in a:
            assert_close(a[k], b[k], 1e-3, 1e-3, f"stage {i} ({uwb[i][0]}) {k}")


def test_uwb_input_permute():
    """Permute((1, 4, 2, 3, 5)) + Reshape: element (n, t, s, a, b, c) lands at
    (n, t, b, s*6 + a*2 + c)."""
    from oracle.netstep import uwb_input
    x = np.arange(2 * 8 * 6 * 3 * 16 * 2, dtype=np.float32).reshape(2, 8, 6, 3, 16, 2)
    y = uwb_input(x)
    assert y.shape == (2, 8, 16, 36)
    assert y[1, 5, 11, 4 * 6 + 2 * 2 + 1] == x[1, 5, 4, 2, 11, 1]


@pytest.mark.parametrize("widened", [False, True])
def test_numpy_readme_params_match_the_model(widened):
    """The bench reference arm's numpy weights have the model's structure and
    shapes, and the Keras initial values (glorot-uniform bounds, gamma 1, beta
    0, zero bias)."""
    from opencl_tf.model import build_model
    from oracle.netstep import params_of, readme_params
    want = params_of(build_model(widened=widened))
    got = readme_params(widened=widened, seed=0)

    def flat(p, pre=""):
        out = {}
        for k, v in p.items():
            if isinstance(v, list):
                for i, d in enumerate(v):
                    out.update(flat(d, f"{pre}{k}{i}."))
            else:
                out[pre + k] = v
        return out

    fw, fg = flat(want), flat(got)
    assert sorted(fw) == sorted(fg)
    for k in fw:
        assert fw[k].shape == fg[k].shape and fg[k].dtype == np.float32, k
        if k.endswith(("_g", ".g1", ".g2")):
            assert (fg[k] == 1).all(), k
        elif k.endswith(("_b", ".b1", ".b2")):
            assert (fg[k] == 0).all(), k
        else:
            assert np.abs(fg[k]).max() <= np.abs(fw[k]).max() * 1.05 + 1e-6, k


def test_numpy_uwb_seq_matches_the_model(uwb):
    from oracle.netstep import uwb_seq
    got = uwb_seq(seed=0)
    assert [k for k, _, _ in got] == [k for k, _, _ in uwb]
    for (k, p, a), (_, q, b) in zip(got, uwb):
        assert sorted(p) == sorted(q), k
        for n in p:
            assert p[n].shape == q[n].shape, (k, n)
        assert a == b, (k, a, b)
