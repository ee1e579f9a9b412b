"""The network of the reference README's ``build_model()`` (README.md:162-183),
built from this package's layers:

    conv_bn_relu(48, (3, 7), strides=(1, 2))
    dsconv_block(96,  strides=2)    DW 3x3 -> BN -> ReLU -> 1x1 conv -> BN -> ReLU
    dsconv_block(144, strides=2)
    Flatten -> Dense(128) -> ReLU -> Reshape(4, 4, 8) -> UpSampling2D(2x) -> Sigmoid

Each BatchNormalization -> ReLU pair runs as one fused op in training, and
Dense -> ReLU as one GEMM with the ReLU in its epilogue (``fuse_bn_relu=True``,
the default): the same values and gradients bit for bit as the layers in
sequence, one activation pass fewer each way.

``build_model(widened=True)`` gives the larger variant used for scaling runs:
input 256x256x3, filters 96/192/288, Dense 512, Reshape(8, 8, 8) -> 16x16x8.
All activations are NHWC float32 on the GPU; Flatten/Reshape are free views.
"""
from __future__ import annotations

from typing import Sequence

import torch
from torch import nn

from .layers import (OpenCLBatchNormalization, OpenCLConv2D, OpenCLDense, OpenCLDepthwiseConv2D, OpenCLReLU,
                     OpenCLSigmoid, OpenCLUpSampling2D)


def _same_out(n: int, s: int) -> int:
    return (n + s - 1) // s


class BuildModel(nn.Module):
    def __init__(self, input_shape: Sequence[int] = (64, 64, 3), filters: Sequence[int] = (48, 96, 144),
                 dense_units: int = 128, head: Sequence[int] = (4, 4, 8), upsample=(2, 2), device=None,
                 fuse_bn_relu: bool = True):
        super().__init__()
        self.fuse_bn_relu = bool(fuse_bn_relu)
        H, W, C = (int(v) for v in input_shape)
        self.input_shape = (H, W, C)
        self.head = tuple(int(v) for v in head)
        if self.head[0] * self.head[1] * self.head[2] != dense_units:
            raise ValueError("head must reshape the dense output exactly")
        dev = torch.device(device) if device is not None else None

        def built(layer, shape):
            layer._device = dev
            layer.build(shape)
            return layer

        f0 = int(filters[0])
        self.stem_conv = built(OpenCLConv2D(f0, (3, 7), strides=(1, 2), padding="same"), (1, H, W, C))
        H, W, C = _same_out(H, 1), _same_out(W, 2), f0
        self.stem_bn = built(OpenCLBatchNormalization(), (1, H, W, C))
        self.stem_relu = OpenCLReLU()
        blocks = []
        for f in filters[1:]:
            dw = built(OpenCLDepthwiseConv2D(3, strides=(2, 2), padding="same"), (1, H, W, C))
            H, W = _same_out(H, 2), _same_out(W, 2)
            bn1 = built(OpenCLBatchNormalization(), (1, H, W, C))
            pw = built(OpenCLConv2D(int(f), 1), (1, H, W, C))
            C = int(f)
            bn2 = built(OpenCLBatchNormalization(), (1, H, W, C))
            blocks.append(nn.ModuleList([dw, bn1, OpenCLReLU(), pw, bn2, OpenCLReLU()]))
        self.blocks = nn.ModuleList(blocks)
        self.flat_features = H * W * C
        self.dense = built(OpenCLDense(int(dense_units)), (1, self.flat_features))
        self.dense_relu = OpenCLReLU()
        self.up = OpenCLUpSampling2D(upsample)
        self.sigmoid = OpenCLSigmoid()
        self.output_shape = (self.head[0] * self.up.size[0], self.head[1] * self.up.size[1], self.head[2])

    def _bn_relu(self, bn, relu, x, training):
        if self.fuse_bn_relu:
            return bn.forward_relu(x, training=training)
        return relu(bn(x, training=training))

    def forward(self, x, training=None):
        x = self._bn_relu(self.stem_bn, self.stem_relu, self.stem_conv(x), training)
        for dw, bn1, r1, pw, bn2, r2 in self.blocks:
            x = self._bn_relu(bn1, r1, dw(x), training)
            x = self._bn_relu(bn2, r2, pw(x), training)
        x = x.reshape(x.shape[0], -1)
        x = self.dense.forward_relu(x) if self.fuse_bn_relu else self.dense_relu(self.dense(x))
        x = x.reshape(x.shape[0], *self.head)
        return self.sigmoid(self.up(x))


def build_model(widened: bool = False, device=None, fuse_bn_relu: bool = True) -> BuildModel:
    """The README model; ``widened=True`` for the 256x256 / 96-192-288 / Dense 512 variant."""
    if widened:
        return BuildModel((256, 256, 3), (96, 192, 288), 512, (8, 8, 8), device=device, fuse_bn_relu=fuse_bn_relu)
    return BuildModel(device=device, fuse_bn_relu=fuse_bn_relu)
