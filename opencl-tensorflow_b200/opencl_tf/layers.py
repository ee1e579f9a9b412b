"""Layers over the seven ops, with the constructor arguments, weight names and
behaviour of the reference's Keras layers (opencl_tf/layers.py:33-328), as
``torch.nn.Module`` objects.

Like Keras layers they build their weights on the first call (or an explicit
``build(input_shape)``) from the input's channel count, keep NHWC
activations, and expose ``get_config()``.  ``OpenCLBatchNormalization`` takes
``training=`` per call (default: the module's train/eval mode) and updates
its moving statistics by the same exponential moving average of the biased
batch variance (opencl_tf/layers.py:185-195).
"""
from __future__ import annotations

from typing import Tuple, Union

import torch
from torch import nn

from . import initializers
from . import _library
from ._library import raw_ops
from .ops.conv2d import conv2d
from .ops.dense import dense
from .ops.depthwise_conv2d import depthwise_conv2d
from .ops.relu import relu
from .ops.sigmoid import sigmoid
from .ops.upsampling import upsampling_bilinear_2d


def _as_pair(v) -> Tuple[int, int]:
    return (int(v), int(v)) if isinstance(v, int) else (int(v[0]), int(v[1]))


class _Layer(nn.Module):
    """Keras-style lazy build: weights are created by ``build`` on first call."""

    def __init__(self, name: str | None = None, device=None):
        super().__init__()
        self.layer_name = name
        self._device = device
        self.built = False

    def build(self, input_shape) -> None:
        self.built = True

    def _weight(self, name, shape, init, trainable=True, device=None):
        t = initializers.get(init)(tuple(int(s) for s in shape))
        dev = device if device is not None else self._device
        if dev is not None:
            t = t.to(dev)
        if name in self.__dict__:  # the None placeholder set in __init__
            delattr(self, name)
        if trainable:
            p = nn.Parameter(t)
            self.register_parameter(name, p)
            return p
        self.register_buffer(name, t)
        return t

    def __call__(self, x, *args, **kwargs):
        if not self.built:
            if self._device is None and isinstance(x, torch.Tensor):
                self._device = x.device
            self.build(tuple(x.shape))
        return super().__call__(x, *args, **kwargs)

    def get_config(self) -> dict:
        return {"name": self.layer_name}


class OpenCLConv2D(_Layer):
    """Conv2D without bias (reference opencl_tf/layers.py:33-81)."""

    def __init__(self, filters: int, kernel_size: Union[int, Tuple[int, int]],
                 strides: Union[int, Tuple[int, int]] = (1, 1), padding: str = "same",
                 kernel_initializer="glorot_uniform", **kwargs):
        super().__init__(**kwargs)
        self.filters = int(filters)
        self.kernel_size = _as_pair(kernel_size)
        self.strides = _as_pair(strides)
        self.padding = padding.upper()
        if self.padding not in ("SAME", "VALID"):
            raise ValueError(f"padding must be 'same' or 'valid', got {padding!r}")
        self.kernel_initializer = initializers.get(kernel_initializer)
        self.kernel = None

    def build(self, input_shape):
        self.kernel = self._weight("kernel", (*self.kernel_size, int(input_shape[-1]), self.filters),
                                   self.kernel_initializer)
        super().build(input_shape)

    def forward(self, x):
        return conv2d(x, self.kernel, strides=(1, self.strides[0], self.strides[1], 1), padding=self.padding)

    def get_config(self):
        cfg = super().get_config()
        cfg.update(filters=self.filters, kernel_size=self.kernel_size, strides=self.strides,
                   padding=self.padding.lower(), kernel_initializer=initializers.serialize(self.kernel_initializer))
        return cfg


class OpenCLDepthwiseConv2D(_Layer):
    """DepthwiseConv2D without bias (reference opencl_tf/layers.py:87-135)."""

    def __init__(self, kernel_size: Union[int, Tuple[int, int]], strides: Union[int, Tuple[int, int]] = (1, 1),
                 padding: str = "same", depth_multiplier: int = 1, depthwise_initializer="glorot_uniform",
                 **kwargs):
        super().__init__(**kwargs)
        self.kernel_size = _as_pair(kernel_size)
        self.strides = _as_pair(strides)
        self.padding = padding.upper()
        if self.padding not in ("SAME", "VALID"):
            raise ValueError(f"padding must be 'same' or 'valid', got {padding!r}")
        self.depth_multiplier = int(depth_multiplier)
        self.depthwise_initializer = initializers.get(depthwise_initializer)
        self.kernel = None

    def build(self, input_shape):
        self.kernel = self._weight("depthwise_kernel",
                                   (*self.kernel_size, int(input_shape[-1]), self.depth_multiplier),
                                   self.depthwise_initializer)
        super().build(input_shape)

    def forward(self, x):
        return depthwise_conv2d(x, self.kernel, strides=(1, self.strides[0], self.strides[1], 1),
                                padding=self.padding)

    def get_config(self):
        cfg = super().get_config()
        cfg.update(kernel_size=self.kernel_size, strides=self.strides, padding=self.padding.lower(),
                   depth_multiplier=self.depth_multiplier,
                   depthwise_initializer=initializers.serialize(self.depthwise_initializer))
        return cfg


class OpenCLBatchNormalization(_Layer):
    """BatchNorm over the channel (last) axis with trainable gamma/beta and EMA
    moving statistics (reference opencl_tf/layers.py:141-205)."""

    def __init__(self, momentum: float = 0.99, epsilon: float = 1e-3, **kwargs):
        super().__init__(**kwargs)
        self.momentum = float(momentum)
        self.epsilon = float(epsilon)
        self.gamma = self.beta = None
        self.moving_mean = self.moving_var = None

    def build(self, input_shape):
        C = int(input_shape[-1])
        self.gamma = self._weight("gamma", (C,), "ones")
        self.beta = self._weight("beta", (C,), "zeros")
        self.moving_mean = self._weight("moving_mean", (C,), "zeros", trainable=False)
        self.moving_var = self._weight("moving_variance", (C,), "ones", trainable=False)
        super().build(input_shape)

    def forward(self, x, training=None):
        if training is None:
            training = self.training
        if bool(training):
            y, batch_mean, batch_var = raw_ops.opencl_batch_norm_training(x, self.gamma, self.beta,
                                                                          epsilon=self.epsilon)
            with torch.no_grad():
                _library.batch_norm_update_moving(self.moving_mean, self.moving_var, batch_mean.detach(),
                                                  batch_var.detach(), self.momentum)
            return y
        return raw_ops.opencl_batch_norm_inference(x, self.gamma, self.beta, self.moving_mean, self.moving_var,
                                                   epsilon=self.epsilon)

    def forward_relu(self, x, training=None):
        """relu(self(x)): this layer followed by an OpenCLReLU, the pair the
        reference's networks chain, as one fused op when training (bit-identical
        values and gradients, one pass over x and no intermediate tensor)."""
        if training is None:
            training = self.training
        if bool(training):
            # the moving-average update runs in the op's statistics pass
            z, _mean, _var = _library.fused_ops.opencl_batch_norm_relu_training(
                x, self.gamma, self.beta, epsilon=self.epsilon,
                moving=(self.moving_mean, self.moving_var, self.momentum))
            return z
        return relu(self.forward(x, training=False))

    def get_config(self):
        cfg = super().get_config()
        cfg.update(momentum=self.momentum, epsilon=self.epsilon)
        return cfg


class OpenCLReLU(_Layer):
    """ReLU (reference opencl_tf/layers.py:211-218)."""

    def forward(self, x):
        return relu(x)


class OpenCLSigmoid(_Layer):
    """Sigmoid activation (reference opencl_tf/layers.py:224-231)."""

    def forward(self, x):
        return sigmoid(x)


class OpenCLDense(_Layer):
    """Dense without an activation argument; a zero bias is synthesised when
    ``use_bias=False`` so the op is always (x, W, b) (reference
    opencl_tf/layers.py:237-292)."""

    def __init__(self, units: int, use_bias: bool = True, kernel_initializer="glorot_uniform",
                 bias_initializer="zeros", **kwargs):
        super().__init__(**kwargs)
        self.units = int(units)
        self.use_bias = bool(use_bias)
        self.kernel_initializer = initializers.get(kernel_initializer)
        self.bias_initializer = initializers.get(bias_initializer)
        self.kernel = None
        self.bias = None

    def build(self, input_shape):
        self.kernel = self._weight("kernel", (int(input_shape[-1]), self.units), self.kernel_initializer)
        if self.use_bias:
            self.bias = self._weight("bias", (self.units,), self.bias_initializer)
        super().build(input_shape)

    def _b(self, x):
        return self.bias if self.use_bias else torch.zeros((self.units,), dtype=x.dtype, device=x.device)

    def forward(self, x):
        return dense(x, self.kernel, self._b(x))

    def forward_relu(self, x):
        """relu(self(x)): this layer followed by an OpenCLReLU as one op, the
        ReLU applied in the GEMM's epilogue (bit-identical values and
        gradients, one launch and one pass over the output fewer)."""
        return _library.fused_ops.opencl_dense_relu(x, self.kernel, self._b(x))

    def get_config(self):
        cfg = super().get_config()
        cfg.update(units=self.units, use_bias=self.use_bias,
                   kernel_initializer=initializers.serialize(self.kernel_initializer),
                   bias_initializer=initializers.serialize(self.bias_initializer))
        return cfg


class OpenCLUpSampling2D(_Layer):
    """Bilinear 2-D upsampling; only 'bilinear' is supported (reference
    opencl_tf/layers.py:298-328)."""

    def __init__(self, size=(2, 2), interpolation: str = "bilinear", **kwargs):
        super().__init__(**kwargs)
        if interpolation != "bilinear":
            raise ValueError(
                f"OpenCLUpSampling2D only supports interpolation='bilinear', got {interpolation!r}. "
                "Use a stock upsampling layer for other methods.")
        self.size = _as_pair(size)
        self.interpolation = interpolation

    def forward(self, x):
        return upsampling_bilinear_2d(x, size=list(self.size))

    def get_config(self):
        cfg = super().get_config()
        cfg.update(size=self.size, interpolation=self.interpolation)
        return cfg


__all__ = ["OpenCLConv2D", "OpenCLDepthwiseConv2D", "OpenCLBatchNormalization", "OpenCLReLU", "OpenCLSigmoid",
           "OpenCLDense", "OpenCLUpSampling2D"]
