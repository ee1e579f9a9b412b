"""The benchmark workloads of the hot path at full size.

c1  Conv2D fwd + dL/dx + dL/dw: x [8,64,64,3] ~N(0,1), w [3,7,3,48] He-normal,
    strides (1,1,2,1) SAME, upstream grad [8,64,32,48] ~N(0,1).
c2  depthwise-separable block fwd+bwd: x [64,32,16,48] -> DW 3x3 s2 SAME ->
    BN -> ReLU -> 1x1 48->96 -> BN -> ReLU, upstream grad ~N(0,1); ReLU masks
    bit-exact.
c3  Dense + head: x [1024,18432] ~U(-1,1), W Glorot-uniform, b = 0 -> ReLU ->
    [1024,4,4,8] -> bilinear x2 -> Sigmoid, upstream grad ~N(0,1); plus the
    stress GEMM fwd/bwd M=8192, K=4096, N=4096 ~N(0,1).

Checked against the oracle where it runs in seconds; the stress GEMM and the
long reductions are also checked against float64 on the GPU (the reference's
own serial fp32 sums are not exact there).  Tolerances as everywhere:
max-rel 1e-4, L2-rel 1e-5.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from helpers import assert_bitexact, assert_close, rel_errs, to_np

pytestmark = pytest.mark.gpu


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def _conv_f64(x, w, dy, strides, pads):
    """float64 conv forward / input grad / filter grad (NHWC, HWIO)."""
    xd = x.double().permute(0, 3, 1, 2)
    wd = w.double().permute(3, 2, 0, 1)
    xp = torch.nn.functional.pad(xd, pads)
    y = torch.nn.functional.conv2d(xp, wd, stride=strides).permute(0, 2, 3, 1)
    dyd = dy.double().permute(0, 3, 1, 2)
    dw = torch.nn.grad.conv2d_weight(xp, wd.shape, dyd, stride=strides).permute(2, 3, 1, 0)
    dxp = torch.nn.grad.conv2d_input(xp.shape, wd, dyd, stride=strides)
    H, W = xd.shape[2], xd.shape[3]
    dx = dxp[:, :, pads[2]:pads[2] + H, pads[0]:pads[0] + W].permute(0, 2, 3, 1)
    return y, dx, dw


def test_c1_conv2d_fwd_and_grads(otf, port):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((8, 64, 64, 3)).astype(np.float32)
    w = (rng.standard_normal((3, 7, 3, 48)) * math.sqrt(2.0 / 63)).astype(np.float32)
    dy = rng.standard_normal((8, 64, 32, 48)).astype(np.float32)
    st = (1, 1, 2, 1)
    y = otf.conv2d(_cuda(x), _cuda(w), strides=st, padding="SAME")
    dx = otf.conv2d_backprop_input([8, 64, 64, 3], _cuda(w), _cuda(dy), strides=st, padding="SAME")
    dw = otf.conv2d_backprop_filter(_cuda(x), [3, 7, 3, 48], _cuda(dy), strides=st, padding="SAME")
    assert_close(to_np(y), port.conv2d(x, w, st, "SAME"), what="y")
    assert_close(to_np(dx), port.conv2d_backprop_input(x.shape, w, dy, st, "SAME"), what="dx")
    ref_dw = port.conv2d_backprop_filter(x, w.shape, dy, st, "SAME")
    # SAME for (3,7) stride (1,2) on 64x64: pad rows 1/1, cols 2/3
    ey, edx, edw = _conv_f64(_cuda(x), _cuda(w), _cuda(dy), (1, 2), (2, 3, 1, 1))
    got = to_np(dw)
    vs_ref, vs_exact, ref_exact = rel_errs(got, ref_dw), rel_errs(got, edw.cpu().numpy()), \
        rel_errs(ref_dw, edw.cpu().numpy())
    assert vs_exact[0] <= 1e-4 and vs_exact[1] <= 1e-5, (vs_exact, ref_exact)
    assert vs_ref[0] <= 1e-4 and vs_ref[1] <= max(1e-5, 2 * ref_exact[1]), (vs_ref, ref_exact)
    assert_close(to_np(y), ey.cpu().numpy(), what="y vs f64")


def test_c2_depthwise_separable_block(otf, port):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((64, 32, 16, 48)).astype(np.float32)
    wd = (rng.standard_normal((3, 3, 48, 1)) * math.sqrt(2.0 / 9)).astype(np.float32)
    wp = (rng.standard_normal((1, 1, 48, 96)) * math.sqrt(2.0 / 48)).astype(np.float32)
    g1, b1 = np.ones(48, np.float32), np.zeros(48, np.float32)
    g2, b2 = np.ones(96, np.float32), np.zeros(96, np.float32)
    s2, s1 = (1, 2, 2, 1), (1, 1, 1, 1)
    # oracle forward
    a = port.depthwise_conv2d(x, wd, s2, "SAME")
    bn1, m1, v1 = port.batch_norm_training(a, g1, b1)
    r1 = port.relu(bn1)
    c = port.conv2d(r1, wp, s1, "SAME")
    bn2, m2, v2 = port.batch_norm_training(c, g2, b2)
    out = port.relu(bn2)
    dout = rng.standard_normal(out.shape).astype(np.float32)
    # GPU forward, op by op on the same inputs
    ga = otf.depthwise_conv2d(_cuda(x), _cuda(wd), strides=s2, padding="SAME")
    assert_bitexact(to_np(ga), a, "dw fwd")
    gbn1, gm1, gv1 = otf.batch_norm_training(ga, _cuda(g1), _cuda(b1))
    assert_close(to_np(gbn1), bn1, what="bn1")
    assert_bitexact(to_np(otf.relu(_cuda(bn1))), r1, "relu1 mask")
    gc = otf.conv2d(_cuda(r1), _cuda(wp), strides=s1, padding="SAME")
    assert_close(to_np(gc), c, what="pw fwd")
    gbn2, gm2, gv2 = otf.batch_norm_training(_cuda(c), _cuda(g2), _cuda(b2))
    assert_close(to_np(gbn2), bn2, what="bn2")
    assert_bitexact(to_np(otf.relu(_cuda(bn2))), out, "relu2 mask")
    # backward, op by op
    d = port.relu_grad(dout, bn2)
    assert_bitexact(to_np(otf.relu_grad(_cuda(dout), _cuda(bn2))), d, "relu2 grad")
    d2, dg2, db2 = port.batch_norm_grad(d, c, g2, m2, v2)
    gd2 = otf.batch_norm_grad(_cuda(d), _cuda(c), _cuda(g2), _cuda(m2), _cuda(v2))
    for got, want, n in zip(gd2, (d2, dg2, db2), ("bn2 dx", "bn2 dgamma", "bn2 dbeta")):
        assert_close(to_np(got), want, what=n)
    dwp = port.conv2d_backprop_filter(r1, wp.shape, d2, s1, "SAME")
    assert_close(to_np(otf.conv2d_backprop_filter(_cuda(r1), list(wp.shape), _cuda(d2), strides=s1,
                                                  padding="SAME")), dwp, what="pw wgrad")
    dr1 = port.conv2d_backprop_input(r1.shape, wp, d2, s1, "SAME")
    assert_close(to_np(otf.conv2d_backprop_input(list(r1.shape), _cuda(wp), _cuda(d2), strides=s1,
                                                 padding="SAME")), dr1, what="pw dgrad")
    d = port.relu_grad(dr1, bn1)
    d1, dg1, db1 = port.batch_norm_grad(d, a, g1, m1, v1)
    gd1 = otf.batch_norm_grad(_cuda(d), _cuda(a), _cuda(g1), _cuda(m1), _cuda(v1))
    for got, want, n in zip(gd1, (d1, dg1, db1), ("bn1 dx", "bn1 dgamma", "bn1 dbeta")):
        assert_close(to_np(got), want, what=n)
    assert_bitexact(to_np(otf.depthwise_conv2d_backprop_input(list(x.shape), _cuda(wd), _cuda(d1), strides=s2,
                                                              padding="SAME")),
                    port.depthwise_conv2d_backprop_input(x.shape, wd, d1, s2, "SAME"), "dw dgrad")
    assert_close(to_np(otf.depthwise_conv2d_backprop_filter(_cuda(x), list(wd.shape), _cuda(d1), strides=s2,
                                                            padding="SAME")),
                 port.depthwise_conv2d_backprop_filter(x, wd.shape, d1, s2, "SAME"), what="dw wgrad")


def test_c3_dense_head(otf, port):
    rng = np.random.default_rng(2)
    x = rng.uniform(-1, 1, (1024, 18432)).astype(np.float32)
    lim = math.sqrt(6.0 / (18432 + 128))
    W = rng.uniform(-lim, lim, (18432, 128)).astype(np.float32)
    b = np.zeros(128, np.float32)
    y = otf.dense(_cuda(x), _cuda(W), _cuda(b))
    ry = port.dense(x, W, b)
    assert_close(to_np(y), ry, what="dense fwd")
    r = port.relu(ry)
    h = r.reshape(1024, 4, 4, 8)
    u = port.upsampling_bilinear_2d(h, [2, 2])
    s = port.sigmoid(u)
    gs = otf.sigmoid(otf.upsampling_bilinear_2d(otf.relu(_cuda(ry)).reshape(1024, 4, 4, 8), size=[2, 2]))
    assert_close(to_np(gs), s, what="head")
    ds = rng.standard_normal(s.shape).astype(np.float32)
    du = port.sigmoid_grad(s, ds)
    dh = port.upsampling_bilinear_2d_grad(du, h.shape, [2, 2])
    dr = port.relu_grad(dh.reshape(1024, 128), ry)
    gdh = otf.upsampling_bilinear_2d_grad(_cuda(du), [1024, 4, 4, 8], size=[2, 2])
    assert_bitexact(to_np(gdh), dh, "upsampling grad")
    assert_bitexact(to_np(otf.relu_grad(_cuda(dh.reshape(1024, 128)), _cuda(ry))), dr, "relu grad")
    assert_close(to_np(otf.dense_backprop_input(_cuda(dr), _cuda(W))), port.dense_backprop_input(dr, W),
                 what="dense dgrad")
    assert_close(to_np(otf.dense_backprop_weight(_cuda(x), _cuda(dr))), port.dense_backprop_weight(x, dr),
                 what="dense wgrad")
    assert_bitexact(to_np(otf.dense_backprop_bias(_cuda(dr))), port.dense_backprop_bias(dr), "bias grad")


def test_c3_stress_gemm_fwd_bwd_against_float64(otf):
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(8192, 4096, device="cuda", generator=g)
    W = torch.randn(4096, 4096, device="cuda", generator=g)
    b = torch.zeros(4096, device="cuda")
    dy = torch.randn(8192, 4096, device="cuda", generator=g)
    y = otf.dense(x, W, b)
    xd, Wd, dyd = x.double(), W.double(), dy.double()
    for got, want, name in ((y, xd @ Wd, "fwd"), (otf.dense_backprop_input(dy, W), dyd @ Wd.T, "dgrad"),
                            (otf.dense_backprop_weight(x, dy), xd.T @ dyd, "wgrad")):
        mx, l2 = rel_errs(to_np(got), want.cpu().numpy())
        assert mx <= 1e-4 and l2 <= 1e-5, (name, mx, l2)


def test_long_reductions_against_float64(otf):
    """The README stem's filter gradient at batch 256 (K = 524288 pixels) and a
    K = 65536 dense product: fp32-class accuracy against float64."""
    torch.manual_seed(4)
    before = otf.device_timeouts()  # cumulative over the process
    x = torch.rand(256, 64, 64, 3, device="cuda")
    dy = torch.randn(256, 64, 32, 48, device="cuda")
    dw = otf.conv2d_backprop_filter(x, [3, 7, 3, 48], dy, strides=(1, 1, 2, 1), padding="SAME")
    _, _, edw = _conv_f64(x, torch.zeros(3, 7, 3, 48, device="cuda"), dy, (1, 2), (2, 3, 1, 1))
    mx, l2 = rel_errs(to_np(dw), edw.cpu().numpy())
    assert mx <= 1e-4 and l2 <= 1e-5, ("stem wgrad", mx, l2)
    a = torch.rand(512, 65536, device="cuda")
    w = torch.randn(65536, 256, device="cuda")
    y = otf.dense(a, w, torch.zeros(256, device="cuda"))
    mx, l2 = rel_errs(to_np(y), (a.double() @ w.double()).cpu().numpy())
    assert mx <= 1e-4 and l2 <= 1e-5, ("dense K=65536", mx, l2)
    assert otf.device_timeouts() == before


def test_full_size_ops_are_deterministic(otf):
    torch.manual_seed(5)
    x = torch.rand(256, 64, 64, 3, device="cuda")
    dy = torch.randn(256, 64, 32, 48, device="cuda")
    a = otf.conv2d_backprop_filter(x, [3, 7, 3, 48], dy, strides=(1, 1, 2, 1), padding="SAME")
    b = otf.conv2d_backprop_filter(x, [3, 7, 3, 48], dy, strides=(1, 1, 2, 1), padding="SAME")
    assert torch.equal(a, b)
    h = torch.randn(256, 64, 32, 48, device="cuda")
    g, z = torch.ones(48, device="cuda"), torch.zeros(48, device="cuda")
    r1, r2 = otf.batch_norm_training(h, g, z), otf.batch_norm_training(h, g, z)
    assert all(torch.equal(u, v) for u, v in zip(r1, r2))


@pytest.mark.parametrize("shape", [
    # pointwise input gradients of the README blocks (K = 96 / 144; N = 48 / 96) and the stem
    # forward: the GEMM shapes whose shared-memory ring depth is odd unless rounded
    ("dgrad", (256, 32, 16, 96), (1, 1, 48, 96), [256, 32, 16, 48]),
    ("dgrad", (256, 16, 8, 144), (1, 1, 96, 144), [256, 16, 8, 96]),
    ("fwd", (256, 64, 64, 3), (3, 7, 3, 48), None),
])
def test_tma_engine_repeated_standalone_calls(otf, shape):
    """The same contraction called 200 times on its own, with L2 flushed in
    between (as a per-op profiler replays it): every call returns the same
    bits and no pipeline wait of the tensor-core engine expires.  Guards the
    engine's barrier-phase bookkeeping, whose failures are timing-dependent."""
    kind, xs, ws, sizes = shape
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(*xs, device="cuda", generator=g)
    w = torch.randn(*ws, device="cuda", generator=g)
    flush = torch.empty(64 << 20, device="cuda")
    if kind == "dgrad":
        fn = lambda: otf.conv2d_backprop_input(sizes, w, x, (1, 1, 1, 1), "SAME")  # noqa: E731
    else:
        fn = lambda: otf.conv2d(x, w, (1, 1, 2, 1), "SAME")  # noqa: E731
    torch.cuda.synchronize()
    before = otf.device_timeouts()
    ref = fn().clone()
    bad = 0
    for _ in range(200):
        flush.fill_(1.0)
        bad += int(not torch.equal(fn(), ref))
    torch.cuda.synchronize()
    assert bad == 0
    assert otf.device_timeouts() == before


def test_widened_dense_wgrad_full_k_against_float64(otf):
    """The widened variant's Dense weight gradient at its full size: x
    [128, 589824] (the flattened 64x32x288 activations of 128 images), dy
    [128, 512] -> dW [589824, 512] (302 M entries, 1.2 GB) -- the step's
    largest gradient and its largest all-reduce -- against float64."""
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.rand(128, 589824, device="cuda", generator=g)  # post-ReLU activations are >= 0
    dy = torch.randn(128, 512, device="cuda", generator=g) * 1e-3
    dw = otf.dense_backprop_weight(x, dy)
    exact = x.double().t() @ dy.double()
    d = (dw.double() - exact)
    mx = float(d.abs().max() / exact.abs().max())
    l2 = float(torch.linalg.vector_norm(d) / torch.linalg.vector_norm(exact))
    assert mx <= 1e-4 and l2 <= 1e-5, (mx, l2)
