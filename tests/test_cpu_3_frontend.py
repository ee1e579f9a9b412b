"""Host-side behaviour of the opencl_tf package that needs no GPU: the op
names, the gradient registry, layer configs and weight shapes, the README
network's structure, and argument checks that fail before any launch."""
from __future__ import annotations

import pytest
import torch

import opencl_tf
from opencl_tf import errors, initializers, layers
from opencl_tf._library import _GRADIENTS
from opencl_tf.model import build_model

REFERENCE_OPS = ["opencl_conv2d", "opencl_conv2d_backprop_input", "opencl_conv2d_backprop_filter",
                 "opencl_depthwise_conv2d", "opencl_depthwise_conv2d_backprop_input",
                 "opencl_depthwise_conv2d_backprop_filter", "opencl_relu", "opencl_relu_grad",
                 "opencl_batch_norm_training", "opencl_batch_norm_inference", "opencl_batch_norm_grad",
                 "opencl_sigmoid", "opencl_sigmoid_grad", "opencl_dense", "opencl_dense_backprop_input",
                 "opencl_dense_backprop_weight", "opencl_dense_backprop_bias", "opencl_upsampling_bilinear2d",
                 "opencl_upsampling_bilinear2d_grad"]


def test_raw_ops_are_the_reference_ops():
    assert sorted(vars(opencl_tf.raw_ops)) == sorted(REFERENCE_OPS)


def test_python_api_names():
    for n in ["conv2d", "conv2d_backprop_input", "conv2d_backprop_filter", "depthwise_conv2d",
              "depthwise_conv2d_backprop_input", "depthwise_conv2d_backprop_filter", "relu", "relu_grad",
              "batch_norm_training", "batch_norm_inference", "batch_norm_grad", "sigmoid", "sigmoid_grad", "dense",
              "dense_backprop_input", "dense_backprop_weight", "dense_backprop_bias", "upsampling_bilinear_2d",
              "upsampling_bilinear_2d_grad"]:
        assert callable(getattr(opencl_tf, n)), n


def test_gradient_registry_matches_reference_wiring():
    reference = {"OpenclConv2d", "OpenclDepthwiseConv2d", "OpenclRelu", "OpenclBatchNormTraining", "OpenclSigmoid",
                 "OpenclDense", "OpenclUpsamplingBilinear2d"}
    # the reference's registrations, plus the extensions (not reference ops): the fused
    # BatchNorm -> ReLU pair and the training step's MSE loss
    assert set(_GRADIENTS) == reference | {"OpenclBatchNormReluTraining", "OpenclDenseRelu", "OpenclMseLoss"}
    assert "OpenclBatchNormInference" not in _GRADIENTS


def test_gradient_functions_call_the_right_backward_ops(monkeypatch):
    calls = []
    for name in ("opencl_conv2d_backprop_input", "opencl_conv2d_backprop_filter", "opencl_relu_grad",
                 "opencl_sigmoid_grad", "opencl_dense_backprop_input", "opencl_dense_backprop_weight",
                 "opencl_dense_backprop_bias", "opencl_batch_norm_grad", "opencl_upsampling_bilinear2d_grad"):
        ret = (name,) * 3 if name == "opencl_batch_norm_grad" else name
        monkeypatch.setattr(opencl_tf.raw_ops, name, lambda *a, _n=name, _r=ret, **k: calls.append((_n, a, k)) or _r)
    from opencl_tf._library import Operation
    x, w = torch.zeros(2, 9, 9, 3), torch.zeros(3, 3, 3, 5)
    op = Operation("OpenclConv2d", (x, w), (torch.zeros(1),), {"strides": [1, 2, 2, 1], "padding": "SAME"},
                   (False, True))
    res = _GRADIENTS["OpenclConv2d"](op, "g")
    assert res == [None, "opencl_conv2d_backprop_filter"]
    assert calls[-1][1] == (x, [3, 3, 3, 5], "g") and calls[-1][2] == {"strides": [1, 2, 2, 1], "padding": "SAME"}
    op = Operation("OpenclRelu", (x,), (x,), {}, (True,))
    assert _GRADIENTS["OpenclRelu"](op, "g") == ["opencl_relu_grad"]
    assert calls[-1][1][1] is x  # the mask comes from the forward INPUT
    y = torch.ones(1)
    op = Operation("OpenclSigmoid", (x,), (y,), {}, (True,))
    _GRADIENTS["OpenclSigmoid"](op, "g")
    assert calls[-1][1] == (y, "g")  # from the forward OUTPUT
    op = Operation("OpenclBatchNormTraining", (x, "gamma", "beta"), ("y", "mean", "var"), {"epsilon": 1e-3},
                   (True, True, True))
    _GRADIENTS["OpenclBatchNormTraining"](op, "gy", "gm", "gv")
    assert calls[-1][1] == ("gy", x, "gamma", "mean", "var") and calls[-1][2] == {"epsilon": 1e-3}


def test_layer_configs_and_validation():
    c = layers.OpenCLConv2D(48, (3, 7), strides=(1, 2))
    assert c.get_config()["kernel_size"] == (3, 7) and c.get_config()["padding"] == "same"
    with pytest.raises(ValueError, match="padding"):
        layers.OpenCLConv2D(4, 3, padding="full")
    with pytest.raises(ValueError, match="bilinear"):
        layers.OpenCLUpSampling2D((2, 2), interpolation="nearest")
    d = layers.OpenCLDepthwiseConv2D(3, depth_multiplier=2)
    d.build((1, 8, 8, 5))
    assert tuple(d.kernel.shape) == (3, 3, 5, 2)
    bn = layers.OpenCLBatchNormalization(momentum=0.9)
    bn.build((1, 2, 2, 6))
    assert torch.equal(bn.gamma, torch.ones(6)) and torch.equal(bn.moving_var, torch.ones(6))
    assert {n for n, _ in bn.named_parameters()} == {"gamma", "beta"}
    assert {n for n, _ in bn.named_buffers()} == {"moving_mean", "moving_variance"}
    de = layers.OpenCLDense(7, use_bias=False)
    de.build((3, 11))
    assert de.bias is None and tuple(de.kernel.shape) == (11, 7)


def test_initializer_fans():
    torch.manual_seed(0)
    w = initializers.glorot_uniform((3, 7, 3, 48))
    lim = (6.0 / (63 + 7 * 3 * 48)) ** 0.5
    assert float(w.abs().max()) <= lim
    h = initializers.he_normal((3, 7, 3, 48))
    assert abs(float(h.std()) - (2.0 / 63) ** 0.5) < 0.02


def test_build_model_structure():
    m = build_model()
    assert sum(p.numel() for p in m.parameters()) == 2_383_040
    assert m.flat_features == 18432 and m.output_shape == (8, 8, 8)
    w = build_model(widened=True)
    assert sum(p.numel() for p in w.parameters()) == 302_074_496
    assert w.flat_features == 589_824 and w.output_shape == (16, 16, 8)


def test_cpu_tensors_are_rejected_before_any_launch():
    x = torch.zeros(1, 4, 4, 3)
    with pytest.raises(errors.InvalidArgumentError, match="CUDA device"):
        opencl_tf.relu(x)
    with pytest.raises(errors.InvalidArgumentError, match="CUDA device"):
        opencl_tf.conv2d(x, torch.zeros(3, 3, 3, 2))


def test_error_types():
    assert issubclass(errors.InvalidArgumentError, ValueError)
    assert isinstance(errors.from_status(1, "m"), errors.InvalidArgumentError)
    assert isinstance(errors.from_status(2, "m"), errors.InternalError)
    assert isinstance(errors.from_status(5, "m"), errors.DeadlineExceededError)
