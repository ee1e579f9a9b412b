"""The oracle pinned: the C restatement (oracle/port.c) against the reference's
own kernels -- their committed outputs (tests/golden, made by
tests/golden/make_golden.py from oracle/_ref) and, where oracle/_ref is
built, fresh runs at other shapes -- bit for bit; and both against float64."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from helpers import assert_bitexact, assert_close

GOLD = np.load(Path(__file__).parent / "golden" / "reference_kernels.npz")
CONV_CASES = [((1, 1, 1, 1), "SAME"), ((1, 2, 2, 1), "SAME"), ((1, 1, 1, 1), "VALID"), ((1, 2, 2, 1), "VALID")]


def _tag(strides, padding):
    return f"s{strides[1]}{strides[2]}_{padding}"


@pytest.mark.parametrize("strides,padding", CONV_CASES)
def test_golden_conv2d(port, strides, padding):
    t = "conv_" + _tag(strides, padding)
    x, w, y = GOLD[t + "_x"], GOLD[t + "_w"], GOLD[t + "_y"]
    assert_bitexact(port.conv2d(x, w, strides, padding), y, t)
    assert_bitexact(port.conv2d_backprop_input(x.shape, w, y, strides, padding), GOLD[t + "_dx"], t + " dx")
    assert_bitexact(port.conv2d_backprop_filter(x, w.shape, y, strides, padding), GOLD[t + "_dw"], t + " dw")


@pytest.mark.parametrize("dm", [1, 2])
@pytest.mark.parametrize("strides,padding", CONV_CASES)
def test_golden_depthwise(port, strides, padding, dm):
    t = f"dw{dm}_" + _tag(strides, padding)
    x, w, y = GOLD[t + "_x"], GOLD[t + "_w"], GOLD[t + "_y"]
    assert_bitexact(port.depthwise_conv2d(x, w, strides, padding), y, t)
    assert_bitexact(port.depthwise_conv2d_backprop_input(x.shape, w, y, strides, padding), GOLD[t + "_dx"], t)
    assert_bitexact(port.depthwise_conv2d_backprop_filter(x, w.shape, y, strides, padding), GOLD[t + "_dw"], t)


def test_golden_batchnorm(port):
    y, m, v = port.batch_norm_training(GOLD["bn_train_x"], GOLD["bn_train_g"], GOLD["bn_train_b"])
    assert_bitexact(y, GOLD["bn_train_y"], "y")
    assert_bitexact(m, GOLD["bn_train_mean"], "mean")
    assert_bitexact(v, GOLD["bn_train_var"], "var")
    yi = port.batch_norm_inference(*(GOLD["bn_inf_" + k] for k in ("x", "g", "b", "m", "v")))
    assert_bitexact(yi, GOLD["bn_inf_y"], "inference")
    x, g, b = GOLD["bn_grad_x"], GOLD["bn_grad_g"], GOLD["bn_grad_b"]
    y, m, v = port.batch_norm_training(x, g, b)
    dx, dg, db = port.batch_norm_grad(y, x, g, m, v)
    assert_bitexact(dx, GOLD["bn_grad_dx"], "dx")
    assert_bitexact(dg, GOLD["bn_grad_dg"], "dgamma")
    assert_bitexact(db, GOLD["bn_grad_db"], "dbeta")


def test_golden_relu_sigmoid(port):
    x = GOLD["relu_x"]
    assert_bitexact(port.relu(x), GOLD["relu_y"], "relu")
    assert_bitexact(port.relu_grad(port.relu(x), x), GOLD["relu_dx"], "relu grad")
    assert_bitexact(port.relu(GOLD["relu_edge_x"]), GOLD["relu_edge_y"], "relu edges")
    assert_bitexact(port.sigmoid(GOLD["sig_x"]), GOLD["sig_y"], "sigmoid")
    assert_bitexact(port.sigmoid_grad(GOLD["sig_y"], GOLD["sig_y"]), GOLD["sig_dx"], "sigmoid grad")
    assert_bitexact(port.sigmoid(GOLD["sig_ext_x"]), GOLD["sig_ext_y"], "sigmoid extremes")
    assert GOLD["sig_ext_y"][0, 0] == 0.0 and GOLD["sig_ext_y"][0, 1] == 1.0
    assert np.all(GOLD["relu_dx"][GOLD["relu_x"] == 0] == 0)


@pytest.mark.parametrize("shape", [(1, 1, 1), (8, 32, 64), (16, 64, 32), (3, 128, 10)])
def test_golden_dense(port, shape):
    t = "dense_%d_%d_%d" % shape
    x, w, b, y = (GOLD[t + s] for s in ("_x", "_w", "_b", "_y"))
    assert_bitexact(port.dense(x, w, b), y, t)
    assert_bitexact(port.dense_backprop_input(y, w), GOLD[t + "_dx"], t + " dx")
    assert_bitexact(port.dense_backprop_weight(x, y), GOLD[t + "_dw"], t + " dw")
    assert_bitexact(port.dense_backprop_bias(y), GOLD[t + "_db"], t + " db")


@pytest.mark.parametrize("sy,sx", [(2, 2), (3, 3), (2, 3), (4, 2), (1, 1)])
def test_golden_upsampling(port, sy, sx):
    t = f"up_{sy}{sx}"
    x, y = GOLD[t + "_x"], GOLD[t + "_y"]
    assert_bitexact(port.upsampling_bilinear_2d(x, [sy, sx]), y, t)
    assert_bitexact(port.upsampling_bilinear_2d_grad(y, x.shape, [sy, sx]), GOLD[t + "_dx"], t + " grad")
    if (sy, sx) == (1, 1):
        assert_bitexact(y, x, "identity")
    got = port.upsampling_bilinear_2d(GOLD["up_1px_x"], [3, 4])
    assert_bitexact(got, GOLD["up_1px_y"], "single pixel")
    # the reference's blend weights need not sum to exactly 1 in fp32; its own
    # test allows 1e-4 (tests/test_upsampling.py:61-67)
    np.testing.assert_allclose(got, np.broadcast_to(GOLD["up_1px_x"], got.shape), atol=1e-4)


RANDOM_CONV = [((3, 11, 13, 8), (3, 3, 8, 6), (1, 2, 2, 1), "SAME"), ((2, 10, 9, 5), (5, 3, 5, 7), (1, 3, 2, 1), "VALID"),
               ((2, 16, 16, 3), (3, 7, 3, 12), (1, 1, 2, 1), "SAME"), ((1, 1, 1, 1), (1, 1, 1, 1), (1, 1, 1, 1), "SAME")]


@pytest.mark.parametrize("xs,ws,strides,padding", RANDOM_CONV)
def test_port_equals_reference_kernels_conv(port, ref, xs, ws, strides, padding):
    rng = np.random.default_rng(11)
    x = rng.standard_normal(xs).astype(np.float32)
    w = rng.standard_normal(ws).astype(np.float32)
    y = ref.conv2d(x, w, strides, padding)
    assert_bitexact(port.conv2d(x, w, strides, padding), y, "fwd")
    assert_bitexact(port.conv2d_backprop_input(xs, w, y, strides, padding),
                    ref.conv2d_backprop_input(xs, w, y, strides, padding), "dgrad")
    assert_bitexact(port.conv2d_backprop_filter(x, ws, y, strides, padding),
                    ref.conv2d_backprop_filter(x, ws, y, strides, padding), "wgrad")
    wd = rng.standard_normal((ws[0], ws[1], xs[3], 2)).astype(np.float32)
    yd = ref.depthwise_conv2d(x, wd, strides, padding)
    assert_bitexact(port.depthwise_conv2d(x, wd, strides, padding), yd, "dw fwd")
    assert_bitexact(port.depthwise_conv2d_backprop_input(xs, wd, yd, strides, padding),
                    ref.depthwise_conv2d_backprop_input(xs, wd, yd, strides, padding), "dw dgrad")
    assert_bitexact(port.depthwise_conv2d_backprop_filter(x, wd.shape, yd, strides, padding),
                    ref.depthwise_conv2d_backprop_filter(x, wd.shape, yd, strides, padding), "dw wgrad")


def test_port_equals_reference_kernels_misc(port, ref):
    rng = np.random.default_rng(12)
    x = (rng.standard_normal((5, 9, 7, 13)) * 3 + 1).astype(np.float32)
    g = rng.standard_normal(13).astype(np.float32)
    b = rng.standard_normal(13).astype(np.float32)
    for a, c in zip(port.batch_norm_training(x, g, b), ref.batch_norm_training(x, g, b)):
        assert_bitexact(a, c, "bn")
    y, m, v = ref.batch_norm_training(x, g, b)
    for a, c in zip(port.batch_norm_grad(y, x, g, m, v), ref.batch_norm_grad(y, x, g, m, v)):
        assert_bitexact(a, c, "bn grad")
    xs = rng.standard_normal((3, 5, 7, 5)).astype(np.float32)
    for size in ([2, 2], [3, 5], [1, 4]):
        yu = ref.upsampling_bilinear_2d(xs, size)
        assert_bitexact(port.upsampling_bilinear_2d(xs, size), yu, "up")
        assert_bitexact(port.upsampling_bilinear_2d_grad(yu, xs.shape, size),
                        ref.upsampling_bilinear_2d_grad(yu, xs.shape, size), "up grad")
    X = rng.standard_normal((7, 300)).astype(np.float32)
    W = rng.standard_normal((300, 33)).astype(np.float32)
    B = rng.standard_normal(33).astype(np.float32)
    Y = ref.dense(X, W, B)
    assert_bitexact(port.dense(X, W, B), Y, "dense")
    assert_bitexact(port.dense_backprop_weight(X, Y), ref.dense_backprop_weight(X, Y), "dense dW")


@pytest.mark.parametrize("strides,padding", CONV_CASES)
def test_oracle_against_float64(port, strides, padding):
    from oracle.oracle import f64
    t = "conv_" + _tag(strides, padding)
    x, w, y = GOLD[t + "_x"], GOLD[t + "_w"], GOLD[t + "_y"]
    assert_close(y, f64.conv2d(x, w, strides, padding), 1e-5, 1e-6, "conv vs f64")
    assert_close(GOLD[t + "_dx"], f64.conv2d_backprop_input(x.shape, w, y, strides, padding), 1e-5, 1e-6, "dx")
    assert_close(GOLD[t + "_dw"], f64.conv2d_backprop_filter(x, w.shape, y, strides, padding), 1e-5, 1e-6, "dw")


def test_padding_resolution_matches_tf_rules():
    from oracle.oracle import resolve_padding
    for n in range(1, 20):
        for k in range(1, 8):
            for s in range(1, 5):
                out, pad = resolve_padding(n, k, s, "SAME")
                assert out == -(-n // s)
                assert pad == max((out - 1) * s + k - n, 0) // 2
                if n >= k:
                    assert resolve_padding(n, k, s, "VALID") == ((n - k) // s + 1, 0)


def test_reference_noise_floor_with_fma(ref):
    """The reference kernels contracted into FMAs (what -cl-mad-enable allows)
    differ from the uncontracted build by at most a few fp32 ulps of the
    result scale: the spread any fp32 implementation may show."""
    from oracle.oracle import Oracle, available
    if not available("ref_fma"):
        pytest.skip("oracle/_ref/libref_ocl_fma.so not built")
    fma = Oracle("ref_fma", threads=1)
    t = "conv_s11_SAME"
    x, w = GOLD[t + "_x"], GOLD[t + "_w"]
    a = ref.conv2d(x, w, (1, 1, 1, 1), "SAME")
    b = fma.conv2d(x, w, (1, 1, 1, 1), "SAME")
    assert_close(b, a, 1e-6, 1e-6, "fma vs plain")
