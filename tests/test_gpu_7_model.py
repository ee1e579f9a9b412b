"""End-to-end: the README build_model() network's training step on the GPU
against the oracle-composed step (tests/netoracle.py) -- loss, output and
every weight gradient -- plus the CUDA-graph step and convergence checks
(the reference's "loss decreases" integration tests)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_close, rel_errs, to_np
from oracle.netstep import params_of, train_grads

pytestmark = pytest.mark.gpu


def _model(seed=0):
    from opencl_tf.model import build_model
    torch.manual_seed(seed)
    return build_model(device="cuda")


def _batch(n, seed=1):
    rng = np.random.default_rng(seed)
    x = rng.uniform(0, 1, (n, 64, 64, 3)).astype(np.float32)
    t = rng.uniform(0, 1, (n, 8, 8, 8)).astype(np.float32)
    return x, t


def _grad_pairs(m, g):
    out = [("stem_w", m.stem_conv.kernel, g["stem_w"]), ("stem_g", m.stem_bn.gamma, g["stem_g"]),
           ("stem_b", m.stem_bn.beta, g["stem_b"]), ("dense_w", m.dense.kernel, g["dense_w"]),
           ("dense_b", m.dense.bias, g["dense_b"])]
    for i, (dw, bn1, _, pw, bn2, _) in enumerate(m.blocks):
        gb = g["blocks"][i]
        out += [(f"b{i}.dw", dw.kernel, gb["dw"]), (f"b{i}.g1", bn1.gamma, gb["g1"]), (f"b{i}.b1", bn1.beta, gb["b1"]),
                (f"b{i}.pw", pw.kernel, gb["pw"]), (f"b{i}.g2", bn2.gamma, gb["g2"]), (f"b{i}.b2", bn2.beta, gb["b2"])]
    return out


def _check_step(m, x, t, port, head=(4, 4, 8)):
    """Loss, output and all 17 weight gradients of one training step of `m`
    on (x, t) against the oracle-composed step.  Each gradient must be within
    the contract tolerance of the oracle (the reference's arithmetic).  Where
    the oracle itself is farther than that from the float64 answer (the stem
    and first depthwise filter gradients: BN backward amplifies the rounding
    of the reference's long serial sums), the GPU must instead be within the
    tolerance of float64 -- or, where no fp32 evaluation order can be (at
    batch 256 the stem filter gradient sums 524,288 products whose total
    nearly cancels: the reference's own result is ~7e-3 from float64), no
    farther from float64 than the oracle, in max and in L2 error."""
    from opencl_tf.train import mse
    from oracle.netstep import train_grads_f64
    p = params_of(m)
    out = m(torch.from_numpy(x).cuda(), training=True)
    loss = mse(out, torch.from_numpy(t).cuda())
    loss.backward()
    r_loss, r_out, r_g = train_grads(port, p, x, t, head=head)
    e_loss, e_out, e_g = train_grads_f64(p, x, t, head=head, device="cuda")
    assert abs(float(loss.detach()) - r_loss) <= 1e-5 * abs(r_loss)
    assert_close(to_np(out), r_out, what="output")
    report = []
    for (name, param, want), (_, _, exact) in zip(_grad_pairs(m, r_g), _grad_pairs(m, e_g)):
        got = to_np(param.grad)
        vs_ref, ref_vs_exact, vs_exact = rel_errs(got, want), rel_errs(want, exact), rel_errs(got, exact)
        report.append((name, vs_ref, ref_vs_exact, vs_exact))
        if vs_ref[0] <= 1e-4 and vs_ref[1] <= 1e-5:
            continue
        assert ref_vs_exact[0] > 1e-4 or ref_vs_exact[1] > 1e-5, (name, vs_ref, ref_vs_exact)
        if vs_exact[0] <= 1e-4 and vs_exact[1] <= 1e-5:
            assert vs_exact[1] <= ref_vs_exact[1], (name, vs_exact, ref_vs_exact)
        else:
            assert vs_exact[0] <= ref_vs_exact[0] and vs_exact[1] <= ref_vs_exact[1], (name, vs_exact, ref_vs_exact)
    print("\n".join(f"{n:8s} gpu-vs-oracle {a[0]:.1e}/{a[1]:.1e}  oracle-vs-f64 {b[0]:.1e}/{b[1]:.1e}  "
                    f"gpu-vs-f64 {c[0]:.1e}/{c[1]:.1e}" for n, a, b, c in report))


# 256 is the benchmarked batch (bench.py's README step): the BatchNorm
# statistics then run over 524,288 rows per channel at the stem.
@pytest.mark.parametrize("batch", [2, 4, 8, 256])
def test_build_model_step_matches_oracle(otf, port, batch):
    x, t = _batch(batch)
    _check_step(_model(), x, t, port)


def test_widened_build_model_step_matches_oracle(otf, port):
    """The widened variant's layer shapes (input 256x256x3, filters 96/192/288,
    Dense 589,824 x 512, head 8x8x8 -> 16x16x8) at batch 2: every op of its
    training step, composed, against the oracle."""
    from opencl_tf.model import build_model
    torch.manual_seed(0)
    m = build_model(widened=True, device="cuda")
    rng = np.random.default_rng(11)
    x = rng.uniform(0, 1, (2, 256, 256, 3)).astype(np.float32)
    t = rng.uniform(0, 1, (2, 16, 16, 8)).astype(np.float32)
    _check_step(m, x, t, port, head=(8, 8, 8))


def test_graphed_step_equals_eager_step(otf):
    from opencl_tf.train import TrainStep
    x, t = _batch(8, seed=2)
    xd, td = torch.from_numpy(x).cuda(), torch.from_numpy(t).cuda()
    m1, m2 = _model(3), _model(3)
    eager = TrainStep(m1, graphed=False)
    graphed = TrainStep(m2, graphed=True, warmup=3)
    for _ in range(3):
        eager(xd, td)
    l_g = graphed(xd, td)  # 3 warm-up steps + the captured step
    l_e = eager(xd, td)
    torch.cuda.synchronize()
    assert torch.equal(l_g, l_e)
    for a, b in zip(m1.parameters(), m2.parameters()):
        assert torch.equal(a, b)
    for _ in range(3):
        l_g, l_e = graphed(xd, td), eager(xd, td)
    assert torch.equal(l_g, l_e)


def test_loss_decreases(otf):
    from opencl_tf.train import TrainStep
    x, t = _batch(16, seed=4)
    xd, td = torch.from_numpy(x).cuda(), torch.from_numpy(t).cuda()
    step = TrainStep(_model(5), lr=1e-3, graphed=True)
    first = float(step(xd, td))
    for _ in range(20):
        last = float(step(xd, td))
    assert last < first, (first, last)


def test_bn_moving_stats_update(otf):
    bn = otf.layers.OpenCLBatchNormalization(momentum=0.5)
    _ = bn(torch.zeros(1, 2, 2, 3, device="cuda"), training=False)
    m0, v0 = bn.moving_mean.clone(), bn.moving_var.clone()
    rng = np.random.default_rng(0)
    for _ in range(4):
        bn(torch.from_numpy(rng.standard_normal((4, 3, 3, 3)).astype(np.float32) * 3 + 1).cuda(), training=True)
    assert not torch.allclose(bn.moving_mean, m0)
    assert not torch.allclose(bn.moving_var, v0)


@pytest.mark.parametrize("layer_fn", ["conv", "dw", "dense", "sigmoid", "bn"])
def test_keras_like_layers_train(otf, layer_fn):
    """Each layer inside an SGD step: loss decreases (reference
    test_keras_layer_trains pattern)."""
    L = otf.layers
    torch.manual_seed(42)
    if layer_fn == "conv":
        layer, x, tgt = L.OpenCLConv2D(4, 3), torch.randn(2, 8, 8, 3), torch.randn(2, 8, 8, 4)
    elif layer_fn == "dw":
        layer, x, tgt = L.OpenCLDepthwiseConv2D(3), torch.randn(2, 8, 8, 3), torch.randn(2, 8, 8, 3)
    elif layer_fn == "dense":
        layer, x, tgt = L.OpenCLDense(8), torch.randn(8, 16), torch.randn(8, 8)
    elif layer_fn == "sigmoid":
        layer, x, tgt = L.OpenCLSigmoid(), torch.randn(2, 4, 4, 8), torch.rand(2, 4, 4, 8)
        x.requires_grad_(True)
    else:
        layer, x, tgt = L.OpenCLBatchNormalization(), torch.randn(4, 5, 5, 3) * 2 + 1, torch.randn(4, 5, 5, 3)
    x, tgt = x.cuda(), tgt.cuda()
    if layer_fn == "sigmoid":
        x = x.detach().requires_grad_(True)
    _ = layer(x)
    params = list(layer.parameters()) or [x]
    opt = torch.optim.SGD(params, lr=1e-2 if layer_fn != "sigmoid" else 1.0)

    def step():
        opt.zero_grad()
        loss = torch.mean((layer(x) - tgt) ** 2)
        loss.backward()
        opt.step()
        return float(loss)

    l0 = step()
    for _ in range(5):
        l1 = step()
    assert l1 < l0


def test_fused_bn_relu_model_matches_unfused(otf):
    """The README model with its BatchNorm -> ReLU pairs fused gives the same
    loss, gradients and moving statistics as with the separate layers."""
    from opencl_tf.model import build_model
    from opencl_tf.train import mse
    torch.manual_seed(0)
    fused = build_model(device="cuda")
    plain = build_model(device="cuda", fuse_bn_relu=False)
    plain.load_state_dict(fused.state_dict())
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.rand(8, 64, 64, 3, device="cuda", generator=g)
    t = torch.rand(8, 8, 8, 8, device="cuda", generator=g)
    lf = mse(fused(x, training=True), t)
    lp = mse(plain(x, training=True), t)
    lf.backward()
    lp.backward()
    assert torch.equal(lf, lp)
    for (n, a), (_, b) in zip(fused.named_parameters(), plain.named_parameters()):
        assert torch.equal(a.grad, b.grad), n
    for (n, a), (_, b) in zip(fused.named_buffers(), plain.named_buffers()):
        assert torch.equal(a, b), n


def test_second_graph_equals_first(otf):
    """Two captured graphs of the step (graph 1 on its own input buffers, for an
    input pipeline) compute the same training steps: alternating them gives
    the same parameters, bit for bit, as replaying graph 0 only."""
    from opencl_tf.train import TrainStep
    batches = [_batch(8, seed=20 + i) for i in range(5)]
    m0, m1 = _model(9), _model(9)
    s0 = TrainStep(m0, graphed=True, warmup=3)
    s1 = TrainStep(m1, graphed=True, warmup=3)
    x, t = batches[0]
    xd, td = torch.from_numpy(x).cuda(), torch.from_numpy(t).cuda()
    s0(xd, td)
    s1(xd, td)  # both: warm-up steps + the capture of graph 0
    for i, (x, t) in enumerate(batches[1:]):
        xd, td = torch.from_numpy(x).cuda(), torch.from_numpy(t).cuda()
        l0 = s0(xd, td)
        bx, by = s1.graph_inputs(i % 2)
        bx.copy_(xd)
        by.copy_(td)
        l1 = s1.replay(i % 2)
        torch.cuda.synchronize()
        assert torch.equal(l0, l1), i
    for a, b in zip(m0.parameters(), m1.parameters()):
        assert torch.equal(a, b)
    s0.release()
    s1.release()
