"""The stem's filter gradient on the CUDA cores (csrc/conv_wgrad.cu) and its
fusion with the BatchNorm -> ReLU backward.

* conv2d_backprop_filter of 7-wide, 3-channel, column-stride-2 filters with
  more than 32 output channels (the README stem: 3x7x3x48 over 64x64 images;
  the widened stem 3x7x3x96 over 256x256) against the oracle (the reference's
  arithmetic) and float64, with ragged shapes: units with unused columns,
  VALID padding, one image row, filter heights 1 and 5, an odd width that
  another engine takes;
* fused_ops.opencl_conv2d_batch_norm_relu_backprop_filter equal bit for bit
  to opencl_batch_norm_relu_grad followed by opencl_conv2d_backprop_filter,
  on the kernel's shapes and on a shape it does not take (the fallback);
* the README network with its stem fused still equals the unfused network.
Tolerances as everywhere: max-rel 1e-4, L2-rel 1e-5.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_close, rel_errs, to_np

pytestmark = pytest.mark.gpu


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def _wgrad_f64(x, dy, kshape, strides, padding):
    """float64 filter gradient (NHWC, HWIO), TF SAME/VALID padding."""
    import torch.nn.functional as F
    kh, kw = kshape[0], kshape[1]
    xd = torch.tensor(x, dtype=torch.float64, device="cuda").permute(0, 3, 1, 2)
    H, W = xd.shape[2], xd.shape[3]
    sh, sw = strides[1], strides[2]
    if padding == "SAME":
        oh, ow = -(-H // sh), -(-W // sw)
        ph, pw = max((oh - 1) * sh + kh - H, 0), max((ow - 1) * sw + kw - W, 0)
        xd = F.pad(xd, (pw // 2, pw - pw // 2, ph // 2, ph - ph // 2))
    dyd = torch.tensor(dy, dtype=torch.float64, device="cuda").permute(0, 3, 1, 2)
    wshape = (kshape[3], kshape[2], kh, kw)
    return torch.nn.grad.conv2d_weight(xd, wshape, dyd, stride=(sh, sw)).permute(2, 3, 1, 0).cpu().numpy()


CASES = [
    ((8, 64, 64, 3), (3, 7, 3, 48), "SAME"),    # the README stem at a small batch
    ((2, 9, 36, 3), (3, 7, 3, 48), "SAME"),     # 18 output columns of a 32-column unit
    ((3, 11, 28, 3), (5, 7, 3, 40), "VALID"),   # VALID, filter height 5, 20-column units (11 used)
    ((4, 1, 64, 3), (1, 7, 3, 96), "SAME"),     # one image row, filter height 1, 96 channels
    ((3, 5, 64, 3), (3, 7, 3, 96), "SAME"),     # 96 channels: two column chunks per output row
    ((2, 32, 256, 3), (3, 7, 3, 96), "SAME"),   # the widened stem's width and channels
    ((2, 9, 37, 3), (3, 7, 3, 48), "SAME"),     # odd width: not this kernel's (another engine)
]


@pytest.mark.parametrize("xs,ws,padding", CASES)
def test_stem_filter_gradient_matches_oracle(otf, port, xs, ws, padding):
    rng = np.random.default_rng(sum(xs) + sum(ws))
    strides = (1, 1, 2, 1)
    x = rng.uniform(0, 1, xs).astype(np.float32)
    out = otf.conv2d(_cuda(x), _cuda(np.zeros(ws, np.float32)), strides=strides, padding=padding)
    dy = rng.standard_normal(tuple(out.shape)).astype(np.float32)
    got = to_np(otf.conv2d_backprop_filter(_cuda(x), list(ws), _cuda(dy), strides=strides, padding=padding))
    want = port.conv2d_backprop_filter(x, ws, dy, strides, padding)
    exact = _wgrad_f64(x, dy, ws, strides, padding)
    vs_ref, ref_vs_exact, vs_exact = rel_errs(got, want), rel_errs(want, exact), rel_errs(got, exact)
    if not (vs_ref[0] <= 1e-4 and vs_ref[1] <= 1e-5):
        # the reference's serial sum is itself off: be exact-er than it
        assert vs_exact[0] <= 1e-4 and vs_exact[1] <= 1e-5, (vs_exact, ref_vs_exact)
        assert vs_exact[1] <= ref_vs_exact[1], (vs_exact, ref_vs_exact)


def test_stem_filter_gradient_readme_batch_256_against_float64(otf):
    """The benchmarked size: 524,288 output pixels per filter element."""
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.rand(256, 64, 64, 3, device="cuda", generator=g)
    dy = torch.randn(256, 64, 32, 48, device="cuda", generator=g)
    got = to_np(otf.conv2d_backprop_filter(x, [3, 7, 3, 48], dy, strides=(1, 1, 2, 1), padding="SAME"))
    exact = _wgrad_f64(to_np(x), to_np(dy), (3, 7, 3, 48), (1, 1, 2, 1), "SAME")
    assert_close(got, exact, what="stem wgrad vs float64")


def test_stem_filter_gradient_deterministic(otf):
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.rand(16, 64, 64, 3, device="cuda", generator=g)
    dy = torch.randn(16, 64, 32, 48, device="cuda", generator=g)
    a = otf.conv2d_backprop_filter(x, [3, 7, 3, 48], dy, strides=(1, 1, 2, 1), padding="SAME")
    b = otf.conv2d_backprop_filter(x, [3, 7, 3, 48], dy, strides=(1, 1, 2, 1), padding="SAME")
    assert torch.equal(a, b)


@pytest.mark.parametrize("xs,ws", [((8, 64, 64, 3), (3, 7, 3, 48)), ((2, 9, 36, 3), (3, 7, 3, 40)),
                                   ((2, 9, 37, 3), (3, 7, 3, 48)), ((2, 9, 36, 3), (3, 7, 3, 16)),
                                   ((2, 10, 12, 5), (3, 3, 5, 40))])
def test_fused_conv_bn_relu_filter_gradient_equals_the_ops(otf, xs, ws):
    """The fused op against ReluGrad -> BatchNormGrad -> Conv2DBackpropFilter
    (the last three shapes are not ones the fused kernel takes -- an odd
    width, 16 output channels (the narrow-filter kernel), 5 input channels
    (the GEMM engines): the fallback)."""
    from opencl_tf import fused_ops, raw_ops
    g = torch.Generator(device="cuda").manual_seed(6)
    x = torch.rand(*xs, device="cuda", generator=g)
    w = torch.randn(*ws, device="cuda", generator=g) * 0.2
    gamma = torch.rand(ws[3], device="cuda", generator=g) + 0.5
    beta = torch.randn(ws[3], device="cuda", generator=g) * 0.1
    st, pad = (1, 1, 2, 1), "SAME"
    z, y, mean, var = fused_ops.opencl_conv2d_batch_norm_relu_training(x, w, gamma, beta, st, pad)
    dz = torch.randn(z.shape, device="cuda", generator=g)
    dw, gg, gb = fused_ops.opencl_conv2d_batch_norm_relu_backprop_filter(x, list(ws), dz, y, gamma, beta, mean,
                                                                         var, st, pad)
    gy, gg2, gb2 = fused_ops.opencl_batch_norm_relu_grad(dz, y, gamma, beta, mean, var)
    dw2 = raw_ops.opencl_conv2d_backprop_filter(x, list(ws), gy, st, pad)
    assert torch.equal(gg, gg2) and torch.equal(gb, gb2)
    assert torch.equal(dw, dw2)
    # and the forward equals the ops in sequence
    y2 = raw_ops.opencl_conv2d(x, w, st, pad)
    z2, m2, v2 = fused_ops.opencl_batch_norm_relu_training(y2, gamma, beta)
    assert torch.equal(y, y2) and torch.equal(z, z2) and torch.equal(mean, m2) and torch.equal(var, v2)


def test_fused_stem_op_gradients_through_autograd(otf):
    """With the input needing a gradient the op's backward takes the unfused
    sequence (input gradient included); without, the fused filter gradient --
    both give the same filter, gamma and beta gradients."""
    from opencl_tf import fused_ops
    g = torch.Generator(device="cuda").manual_seed(8)
    x = torch.rand(4, 64, 64, 3, device="cuda", generator=g)
    w = (torch.randn(3, 7, 3, 48, device="cuda", generator=g) * 0.2)
    gamma = torch.rand(48, device="cuda", generator=g) + 0.5
    beta = torch.randn(48, device="cuda", generator=g) * 0.1
    dz = torch.randn(4, 64, 32, 48, device="cuda", generator=g)
    grads = []
    for need_x in (False, True):
        xs = x.clone().requires_grad_(need_x)
        ps = [t.clone().requires_grad_(True) for t in (w, gamma, beta)]
        z, _y, _m, _v = fused_ops.opencl_conv2d_batch_norm_relu_training(xs, *ps, (1, 1, 2, 1), "SAME")
        (z * dz).sum().backward()
        grads.append([p.grad for p in ps])
        assert (xs.grad is not None) == need_x
    for a, b in zip(*grads):
        assert torch.equal(a, b)
