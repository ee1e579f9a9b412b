"""The reference's second end-to-end network, uwb_loc_v3
(examples/train_full_model.py:70-100), on the GPU: its training step against
the oracle composed from the restated kernels (oracle/netstep.py), the
inference forward with BatchNormalization on moving statistics for both
networks, fused against unfused layer pairs, and the example's own check that
a few Adam steps lower the loss."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import L2_REL, MAX_REL, assert_close, rel_errs, to_np
from oracle.netstep import (seq_forward_inference, seq_of, seq_train_grads, seq_train_grads_f64, uwb_input)

pytestmark = pytest.mark.gpu


def _uwb(seed=0, fuse=True):
    from opencl_tf.model import build_uwb_loc_v3
    torch.manual_seed(seed)
    return build_uwb_loc_v3(device="cuda", fuse_bn_relu=fuse)


def _batch(n, seed=0):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n, 8, 6, 3, 16, 2)).astype(np.float32)
    t = rng.uniform(0, 1, (n, 36, 24, 1)).astype(np.float32)
    return x, t


def _grads_of(model):
    """Weight gradients per stage, keyed like seq_train_grads()."""
    out = []
    for kind, layer, _ in model.stages():
        if kind in ("conv", "dw"):
            out.append({"w": layer.kernel.grad})
        elif kind == "bn":
            out.append({"g": layer.gamma.grad, "b": layer.beta.grad})
        elif kind == "dense":
            out.append({"w": layer.kernel.grad, "b": layer.bias.grad})
        else:
            out.append({})
    return out


@pytest.mark.parametrize("batch", [2, 16, 64])
def test_uwb_step_matches_oracle(otf, port, batch):
    """Loss, output and all 40 weight gradients.  Each gradient is within the
    contract tolerance of the oracle, or else within that tolerance of the
    float64 answer, or else no farther from float64 than the oracle is.  Below
    ten BatchNorms (two of them over 1x1 maps) the oracle and the GPU each
    carry ~1e-5..1e-4 of fp32 rounding in independent orders (the oracle's
    serial BatchNorm sums, the reference's order, lose ~count * 2^-24), so
    their difference can pass 1e-5 while both stay that close to float64."""
    from opencl_tf.train import mse
    m = _uwb()
    x, t = _batch(batch, seed=batch)
    seq = seq_of(m)
    out = m(torch.from_numpy(x).cuda(), training=True)
    loss = mse(out, torch.from_numpy(t).cuda())
    loss.backward()
    xi = uwb_input(x)
    r_loss, r_out, r_g = seq_train_grads(port, seq, xi, t)
    e_loss, e_out, e_g = seq_train_grads_f64(seq, xi, t, device="cuda")
    assert abs(float(loss.detach()) - r_loss) <= 1e-5 * abs(r_loss)
    assert_close(to_np(out), r_out, what="output")
    report = []
    for i, (got_d, want_d, exact_d) in enumerate(zip(_grads_of(m), r_g, e_g)):
        for k, g in got_d.items():
            got, want, exact = to_np(g), want_d[k], exact_d[k]
            name = f"{i}:{seq[i][0]}.{k}"
            vs_ref, ref_vs_exact, vs_exact = rel_errs(got, want), rel_errs(want, exact), rel_errs(got, exact)
            report.append((name, vs_ref, ref_vs_exact, vs_exact))
            if vs_ref[0] <= MAX_REL and vs_ref[1] <= L2_REL:
                continue
            within = vs_exact[0] <= MAX_REL and vs_exact[1] <= L2_REL
            assert within or vs_exact[1] <= ref_vs_exact[1], (name, vs_ref, vs_exact, ref_vs_exact)
    print("\n".join(f"{n:12s} gpu-vs-oracle {a[0]:.1e}/{a[1]:.1e}  oracle-vs-f64 {b[0]:.1e}/{b[1]:.1e}  "
                    f"gpu-vs-f64 {c[0]:.1e}/{c[1]:.1e}" for n, a, b, c in report))


def _trained(model, x, t, steps=2):
    """A few eager Adam steps, so weights and moving statistics are not the
    initial ones."""
    from opencl_tf.train import TrainStep
    step = TrainStep(model, graphed=False)
    xd, td = torch.from_numpy(x).cuda(), torch.from_numpy(t).cuda()
    for _ in range(steps):
        step(xd, td)
    torch.cuda.synchronize()
    return model


@pytest.mark.parametrize("batch", [2, 32])
def test_uwb_inference_matches_oracle(otf, port, batch):
    m = _trained(_uwb(1), *_batch(16, seed=7))
    x, _ = _batch(batch, seed=3)
    with torch.no_grad():
        got = m(torch.from_numpy(x).cuda(), training=False)
    want = seq_forward_inference(port, seq_of(m), uwb_input(x))
    assert_close(to_np(got), want, what="uwb inference")


def test_readme_inference_matches_oracle(otf, port):
    from opencl_tf.model import build_model
    torch.manual_seed(2)
    m = build_model(device="cuda")
    rng = np.random.default_rng(5)
    xt = rng.uniform(0, 1, (8, 64, 64, 3)).astype(np.float32)
    tt = rng.uniform(0, 1, (8, 8, 8, 8)).astype(np.float32)
    _trained(m, xt, tt)
    x = rng.uniform(0, 1, (4, 64, 64, 3)).astype(np.float32)
    with torch.no_grad():
        got = m(torch.from_numpy(x).cuda(), training=False)
    want = seq_forward_inference(port, seq_of(m), x)
    assert_close(to_np(got), want, what="README inference")


def test_uwb_fused_matches_unfused(otf):
    """BatchNorm -> ReLU and Dense -> ReLU fused against the layer pairs: the
    same output, loss and gradients bit for bit."""
    from opencl_tf.train import mse
    x, t = _batch(8, seed=11)
    xd, td = torch.from_numpy(x).cuda(), torch.from_numpy(t).cuda()
    fused, plain = _uwb(4, fuse=True), _uwb(4, fuse=False)
    outs = []
    for m in (fused, plain):
        out = m(xd, training=True)
        mse(out, td).backward()
        outs.append(out.detach())
    assert torch.equal(outs[0], outs[1])
    for a, b in zip(fused.parameters(), plain.parameters()):
        assert torch.equal(a.grad, b.grad)
    for (ka, la, _), (kb, lb, _) in zip(fused.stages(), plain.stages()):
        if ka == "bn":
            assert torch.equal(la.moving_mean, lb.moving_mean) and torch.equal(la.moving_var, lb.moving_var)


@pytest.mark.parametrize("graphed", [False, True])
def test_uwb_loss_decreases(otf, graphed):
    """The example's training check: a few Adam(1e-3) steps on one batch of 2
    lower the MSE."""
    from opencl_tf.train import TrainStep
    x, t = _batch(2, seed=1)
    xd, td = torch.from_numpy(x).cuda(), torch.from_numpy(t).cuda()
    step = TrainStep(_uwb(6), lr=1e-3, graphed=graphed)
    first = float(step(xd, td))
    for _ in range(9):
        last = float(step(xd, td))
    assert last < first, (first, last)
    assert tuple(step.model(xd, training=False).shape) == (2, 36, 24, 1)
