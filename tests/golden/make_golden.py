"""Generates tests/golden/*.npz: inputs and outputs of the reference's own
kernels (kernels/*.cl of OpenCL-Tensorflow 0.3.0, compiled for the host by
oracle/Makefile into oracle/_ref/, run single-threaded) at the seeds and
shapes of the reference's tests (tests/test_*.py).  The reference stores no
golden values of its own -- its tests compare against live TensorFlow,
which this image does not have -- so these fixtures are its kernels' outputs.

    make -C oracle ref && python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle.oracle import Oracle  # noqa: E402

CONV_CASES = [((1, 1, 1, 1), "SAME"), ((1, 2, 2, 1), "SAME"), ((1, 1, 1, 1), "VALID"), ((1, 2, 2, 1), "VALID")]


def tag(strides, padding):
    return f"s{strides[1]}{strides[2]}_{padding}"


def main() -> None:
    o = Oracle("ref", threads=1)
    out = {}

    # tests/test_conv2d.py:18-71 -- seeds 0 (forward) and 1 (gradients)
    for strides, padding in CONV_CASES:
        rng = np.random.default_rng(1)
        x = rng.standard_normal((2, 9, 9, 3)).astype(np.float32)
        w = rng.standard_normal((3, 3, 3, 5)).astype(np.float32)
        y = o.conv2d(x, w, strides, padding)
        t = "conv_" + tag(strides, padding)
        out[t + "_x"], out[t + "_w"], out[t + "_y"] = x, w, y
        out[t + "_dx"] = o.conv2d_backprop_input(x.shape, w, y, strides, padding)
        out[t + "_dw"] = o.conv2d_backprop_filter(x, w.shape, y, strides, padding)

    # tests/test_depthwise_conv2d.py:15-69 -- dm 1 and 2
    for dm in (1, 2):
        for strides, padding in CONV_CASES:
            rng = np.random.default_rng(1)
            x = rng.standard_normal((2, 9, 9, 4)).astype(np.float32)
            w = rng.standard_normal((3, 3, 4, dm)).astype(np.float32)
            y = o.depthwise_conv2d(x, w, strides, padding)
            t = f"dw{dm}_" + tag(strides, padding)
            out[t + "_x"], out[t + "_w"], out[t + "_y"] = x, w, y
            out[t + "_dx"] = o.depthwise_conv2d_backprop_input(x.shape, w, y, strides, padding)
            out[t + "_dw"] = o.depthwise_conv2d_backprop_filter(x, w.shape, y, strides, padding)

    # tests/test_batchnorm.py:36-101
    rng = np.random.default_rng(0)
    x = rng.standard_normal((4, 7, 7, 8)).astype(np.float32)
    g = (rng.standard_normal((8,)) + 1.0).astype(np.float32)
    b = (rng.standard_normal((8,)) * 0.1).astype(np.float32)
    out["bn_train_x"], out["bn_train_g"], out["bn_train_b"] = x, g, b
    out["bn_train_y"], out["bn_train_mean"], out["bn_train_var"] = o.batch_norm_training(x, g, b)
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 5, 5, 6)).astype(np.float32)
    g = (rng.standard_normal((6,)) + 1.0).astype(np.float32)
    b = (rng.standard_normal((6,)) * 0.1).astype(np.float32)
    m = (rng.standard_normal((6,)) * 0.5).astype(np.float32)
    v = (np.abs(rng.standard_normal((6,))) + 0.1).astype(np.float32)
    for k, a in zip(("x", "g", "b", "m", "v"), (x, g, b, m, v)):
        out["bn_inf_" + k] = a
    out["bn_inf_y"] = o.batch_norm_inference(x, g, b, m, v)
    rng = np.random.default_rng(2)
    x = rng.standard_normal((3, 5, 5, 4)).astype(np.float32)
    g = (rng.standard_normal((4,)) + 1.0).astype(np.float32)
    b = (rng.standard_normal((4,)) * 0.1).astype(np.float32)
    y, m, v = o.batch_norm_training(x, g, b)
    out["bn_grad_x"], out["bn_grad_g"], out["bn_grad_b"] = x, g, b
    out["bn_grad_dx"], out["bn_grad_dg"], out["bn_grad_db"] = o.batch_norm_grad(y, x, g, m, v)

    # tests/test_relu.py:14-48 (+ the x == 0 convention) and edge values
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 5, 5, 3)).astype(np.float32)
    x.flat[::5] = 0.0
    out["relu_x"] = x
    out["relu_y"] = o.relu(x)
    out["relu_dx"] = o.relu_grad(o.relu(x), x)
    edge = np.array([-100.0, 100.0, 0.0, -0.0, -30.0, 30.0, np.nan, np.inf, -np.inf, 1e-38], np.float32)
    out["relu_edge_x"], out["relu_edge_y"] = edge, o.relu(edge)

    # tests/test_sigmoid.py:18-76
    rng = np.random.default_rng(1)
    x = rng.standard_normal((3, 6, 6, 4)).astype(np.float32)
    out["sig_x"] = x
    out["sig_y"] = o.sigmoid(x)
    out["sig_dx"] = o.sigmoid_grad(out["sig_y"], out["sig_y"])
    ext = np.array([[-100.0, 100.0, 0.0, -30.0, 30.0]], np.float32)
    out["sig_ext_x"], out["sig_ext_y"] = ext, o.sigmoid(ext)

    # tests/test_dense.py:19-134
    for (B, I, O) in [(1, 1, 1), (8, 32, 64), (16, 64, 32), (3, 128, 10)]:
        rng = np.random.default_rng(42)
        x = rng.standard_normal((B, I)).astype(np.float32)
        W = rng.standard_normal((I, O)).astype(np.float32)
        bb = rng.standard_normal((O,)).astype(np.float32)
        y = o.dense(x, W, bb)
        t = f"dense_{B}_{I}_{O}"
        out[t + "_x"], out[t + "_w"], out[t + "_b"], out[t + "_y"] = x, W, bb, y
        out[t + "_dx"] = o.dense_backprop_input(y, W)
        out[t + "_dw"] = o.dense_backprop_weight(x, y)
        out[t + "_db"] = o.dense_backprop_bias(y)

    # tests/test_upsampling.py:28-111
    for sy, sx in [(2, 2), (3, 3), (2, 3), (4, 2), (1, 1)]:
        rng = np.random.default_rng(42)
        x = rng.standard_normal((2, 4, 6, 8)).astype(np.float32)
        y = o.upsampling_bilinear_2d(x, [sy, sx])
        t = f"up_{sy}{sx}"
        out[t + "_x"], out[t + "_y"] = x, y
        out[t + "_dx"] = o.upsampling_bilinear_2d_grad(y, x.shape, [sy, sx])
    x1 = np.array([[[[3.0, -1.0, 2.5]]]], np.float32)
    out["up_1px_x"], out["up_1px_y"] = x1, o.upsampling_bilinear_2d(x1, [3, 4])

    np.savez_compressed(HERE / "reference_kernels.npz", **out)
    print(f"wrote {len(out)} arrays to {HERE / 'reference_kernels.npz'}")


if __name__ == "__main__":
    main()
