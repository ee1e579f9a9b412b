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

``build_uwb_loc_v3()`` is the reference's second end-to-end network, the
``uwb_loc_v3`` model of examples/train_full_model.py:70-100: stacked radar IQ
[T, 6, 3, bins, 2] permuted to a [T, bins, 36] image, a stem, three
depthwise-separable blocks down to 1x1, a 1x1 neck, then a Dense heatmap head
upsampled twice with a 3x3 conv refinement after each step and a 1x1 conv to
one sigmoid channel.

Both networks list their layers with ``stages()`` as (kind, layer, arg)
triples in execution order; ``run_stages`` executes such a list, fusing each
BatchNormalization -> ReLU and Dense -> ReLU pair when asked.  In inference
(``training=False``) BatchNormalization uses its moving statistics
(OpenclBatchNormInference).
"""
from __future__ import annotations

from typing import Sequence

import torch
from torch import nn

from .layers import (OpenCLBatchNormalization, OpenCLConv2D, OpenCLDense, OpenCLDepthwiseConv2D, OpenCLReLU,
                     OpenCLSigmoid, OpenCLUpSampling2D)


def _same_out(n: int, s: int) -> int:
    return (n + s - 1) // s


def run_stages(stages, x, training=None, fuse: bool = True):
    """Runs (kind, layer, arg) stages in order.  kinds: conv, dw, bn, relu,
    dense, flatten, reshape (arg = the per-sample shape), up, sigmoid."""
    i, n = 0, len(stages)
    while i < n:
        kind, layer, arg = stages[i]
        nxt = stages[i + 1][0] if i + 1 < n else None
        if fuse and nxt == "relu" and kind == "bn":
            x = layer.forward_relu(x, training=training)
            i += 2
            continue
        if fuse and nxt == "relu" and kind == "dense":
            x = layer.forward_relu(x)
            i += 2
            continue
        if kind == "bn":
            x = layer(x, training=training)
        elif kind == "flatten":
            x = x.reshape(x.shape[0], -1)
        elif kind == "reshape":
            x = x.reshape(x.shape[0], *arg)
        else:
            x = layer(x)
        i += 1
    return x


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

    def stages(self):
        st = [("conv", self.stem_conv, None), ("bn", self.stem_bn, None), ("relu", self.stem_relu, None)]
        for dw, bn1, r1, pw, bn2, r2 in self.blocks:
            st += [("dw", dw, None), ("bn", bn1, None), ("relu", r1, None), ("conv", pw, None), ("bn", bn2, None),
                   ("relu", r2, None)]
        return st + [("flatten", None, None), ("dense", self.dense, None), ("relu", self.dense_relu, None),
                     ("reshape", None, self.head), ("up", self.up, None), ("sigmoid", self.sigmoid, None)]


class UwbLocV3(nn.Module):
    """examples/train_full_model.py:70-100 with this package's layers.  Input
    [N, t_ctx, 6, 3, n_bins, 2] (stacked IQ); output [N, 4*head_h, 4*head_w, 1]."""

    def __init__(self, t_ctx: int = 8, n_bins: int = 16, head: Sequence[int] = (9, 6, 8), device=None,
                 fuse_bn_relu: bool = True):
        super().__init__()
        self.fuse_bn_relu = bool(fuse_bn_relu)
        self.t_ctx, self.n_bins = int(t_ctx), int(n_bins)
        self.head = tuple(int(v) for v in head)
        self.input_shape = (self.t_ctx, 6, 3, self.n_bins, 2)
        dev = torch.device(device) if device is not None else None
        H, W, C = self.t_ctx, self.n_bins, 36
        st = []
        mods = nn.ModuleList()

        def add(kind, layer=None, arg=None, shape=None):
            if layer is not None:
                layer._device = dev
                if shape is not None:
                    layer.build(shape)
                mods.append(layer)
            st.append((kind, layer, arg))

        def conv_bn_relu(f, k, strides=(1, 1)):
            nonlocal H, W, C
            add("conv", OpenCLConv2D(f, k, strides=strides, padding="same"), shape=(1, H, W, C))
            H, W, C = _same_out(H, strides[0]), _same_out(W, strides[1]), f
            add("bn", OpenCLBatchNormalization(), shape=(1, H, W, C))
            add("relu", OpenCLReLU())

        def dsconv(f, strides):
            nonlocal H, W, C
            add("dw", OpenCLDepthwiseConv2D(3, strides=strides, padding="same"), shape=(1, H, W, C))
            H, W = _same_out(H, strides[0]), _same_out(W, strides[1])
            add("bn", OpenCLBatchNormalization(), shape=(1, H, W, C))
            add("relu", OpenCLReLU())
            conv_bn_relu(f, 1)

        conv_bn_relu(48, (3, 7), strides=(1, 2))     # stem
        for f in (96, 144, 192):                     # b1, b2, b3
            dsconv(f, (2, 2))
        conv_bn_relu(64, (1, 1))                     # neck
        hh, hw, hc = self.head
        add("flatten")
        add("dense", OpenCLDense(hh * hw * hc), shape=(1, H * W * C))
        add("relu", OpenCLReLU())
        add("reshape", arg=self.head)
        H, W, C = hh, hw, hc
        for _ in range(2):                           # hm_up1 / hm_refine1, hm_up2 / hm_refine2
            add("up", OpenCLUpSampling2D((2, 2)))
            H, W = 2 * H, 2 * W
            conv_bn_relu(16, (3, 3))
        add("conv", OpenCLConv2D(1, (1, 1)), shape=(1, H, W, C))  # heatmap_conv
        add("sigmoid", OpenCLSigmoid())
        self.layers_ = mods
        self._stages = st
        self.output_shape = (H, W, 1)

    def stages(self):
        return list(self._stages)

    def forward(self, x, training=None):
        # Permute((1, 4, 2, 3, 5)) then Reshape((t_ctx, n_bins, 36)): [N, T, 6, 3, B, 2] -> [N, T, B, 36]
        n = x.shape[0]
        x = x.permute(0, 1, 4, 2, 3, 5).reshape(n, self.t_ctx, self.n_bins, 36)
        return run_stages(self._stages, x, training=training, fuse=self.fuse_bn_relu)


def build_model(widened: bool = False, device=None, fuse_bn_relu: bool = True) -> BuildModel:
    """The README model; ``widened=True`` for the 256x256 / 96-192-288 / Dense 512 variant."""
    if widened:
        return BuildModel((256, 256, 3), (96, 192, 288), 512, (8, 8, 8), device=device, fuse_bn_relu=fuse_bn_relu)
    return BuildModel(device=device, fuse_bn_relu=fuse_bn_relu)


def build_uwb_loc_v3(device=None, fuse_bn_relu: bool = True) -> UwbLocV3:
    """The reference example's uwb_loc_v3 network (T_CTX 8, 16 range bins, 9x6x8 head)."""
    return UwbLocV3(device=device, fuse_bn_relu=fuse_bn_relu)
