"""TEST INFRASTRUCTURE -- the parity oracle for the seven ops.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg import this module.  It is what the GPU results are compared with,
never the thing measured on the GPU path and never a fallback for it.

Three arbiters, all on host numpy arrays:

* ``Oracle("ref")``  -- the reference's own ``kernels/*.cl`` compiled as C++
  through ``cl_shim.h`` and driven like ``src/ops/*.cc`` (``oracle/_ref/``).
* ``Oracle("port")`` -- ``port.c``, a plain-C restatement of the same
  arithmetic in the same accumulation order.  It is pinned bit for bit
  against ``"ref"`` by ``tests/test_oracle_pin.py`` and by the committed
  golden vectors in ``tests/golden/``.
* ``f64``            -- float64 numpy restatements of the same maths, used to
  measure how far each fp32 implementation is from the exact result.

Function names and argument meaning follow the reference's Python API
(``opencl_tf/ops/*.py``): NHWC activations, HWIO filters, ``strides`` as an
NHWC 4-list, ``padding`` "SAME"/"VALID", ``size`` = [sy, sx].
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIBS = {
    "port": HERE / "liboracle_port.so",
    "ref": HERE / "_ref" / "libref_ocl.so",
    "ref_fma": HERE / "_ref" / "libref_ocl_fma.so",
}
PREFIX = {"port": "port_", "ref": "ref_", "ref_fma": "ref_"}

_F = ctypes.POINTER(ctypes.c_float)
_I = ctypes.c_int
_L = ctypes.c_long


def build(quiet: bool = True) -> None:
    """Compile the oracle libraries (``make -C oracle``)."""
    out = subprocess.run(["make", "-C", str(HERE)], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def available(impl: str) -> bool:
    return LIBS[impl].exists()


def _fp(a: np.ndarray):
    return a.ctypes.data_as(_F)


def _c32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _same(padding: str) -> int:
    if padding not in ("SAME", "VALID"):
        raise ValueError(f"padding must be SAME or VALID, got {padding!r}")
    return 1 if padding == "SAME" else 0


def _cdiv(a: int, b: int) -> int:
    """C integer division (truncates toward zero)."""
    q = abs(a) // abs(b)
    return q if (a >= 0) == (b > 0) else -q


def resolve_padding(in_size: int, k: int, stride: int, padding: str):
    """src/padding_utils.h:22-33 (TF SAME/VALID), with C integer division."""
    if padding == "SAME":
        out = _cdiv(in_size + stride - 1, stride)
        pad = _cdiv(max((out - 1) * stride + k - in_size, 0), 2)
    else:
        out = _cdiv(in_size - k + stride, stride)
        pad = 0
    return out, pad


class Oracle:
    """fp32 oracle over one of the compiled libraries ("ref" or "port")."""

    def __init__(self, impl: str = "port", threads: int | None = None):
        path = LIBS[impl]
        if not path.exists():
            raise FileNotFoundError(f"oracle library {path} is not built (make -C oracle)")
        self.impl = impl
        self.lib = ctypes.CDLL(str(path))
        self.p = PREFIX[impl]
        for name in ("conv2d", "conv2d_backprop_input", "conv2d_backprop_filter",
                     "depthwise_conv2d", "depthwise_conv2d_backprop_input",
                     "depthwise_conv2d_backprop_filter"):
            getattr(self.lib, self.p + name).argtypes = [_F, _F, _F] + [_I] * 10
        for name in ("relu", "sigmoid"):
            getattr(self.lib, self.p + name).argtypes = [_F, _F, _L]
        for name in ("relu_grad", "sigmoid_grad"):
            getattr(self.lib, self.p + name).argtypes = [_F, _F, _F, _L]
        getattr(self.lib, self.p + "batch_norm_training").argtypes = [_F] * 6 + [_I] * 4 + [ctypes.c_float]
        getattr(self.lib, self.p + "batch_norm_inference").argtypes = [_F] * 6 + [_I] * 4 + [ctypes.c_float]
        getattr(self.lib, self.p + "batch_norm_grad").argtypes = [_F] * 8 + [_I] * 4 + [ctypes.c_float]
        getattr(self.lib, self.p + "dense").argtypes = [_F] * 4 + [_I] * 3
        getattr(self.lib, self.p + "dense_backprop_input").argtypes = [_F] * 3 + [_I] * 3
        getattr(self.lib, self.p + "dense_backprop_weight").argtypes = [_F] * 3 + [_I] * 3
        getattr(self.lib, self.p + "dense_backprop_bias").argtypes = [_F] * 2 + [_I] * 2
        getattr(self.lib, self.p + "upsampling_bilinear2d").argtypes = [_F] * 2 + [_I] * 6
        getattr(self.lib, self.p + "upsampling_bilinear2d_grad").argtypes = [_F] * 2 + [_I] * 6
        getattr(self.lib, self.p + "set_threads").argtypes = [_I]
        if threads is not None:
            self.set_threads(threads)

    def _fn(self, name):
        return getattr(self.lib, self.p + name)

    def set_threads(self, n: int) -> None:
        self._fn("set_threads")(int(n))

    def threads(self) -> int:
        return int(self._fn("get_threads")())

    # ------------------------------------------------------------ conv2d
    def _conv_dims(self, x_shape, w_shape, strides, padding):
        N, H, W, Ci = x_shape
        kH, kW, wci, Co = w_shape
        if wci != Ci:
            raise ValueError("filter[2] must equal input channels")
        sH, sW = int(strides[1]), int(strides[2])
        Ho, _ = resolve_padding(H, kH, sH, padding)
        Wo, _ = resolve_padding(W, kW, sW, padding)
        return N, H, W, Ci, kH, kW, Co, sH, sW, Ho, Wo

    def conv2d(self, x, w, strides=(1, 1, 1, 1), padding="SAME"):
        x, w = _c32(x), _c32(w)
        N, H, W, Ci, kH, kW, Co, sH, sW, Ho, Wo = self._conv_dims(x.shape, w.shape, strides, padding)
        y = np.empty((N, Ho, Wo, Co), np.float32)
        self._fn("conv2d")(_fp(x), _fp(w), _fp(y), N, H, W, Ci, kH, kW, Co, sH, sW, _same(padding))
        return y

    def conv2d_backprop_input(self, input_sizes, w, grad_out, strides, padding):
        w, dy = _c32(w), _c32(grad_out)
        N, H, W, Ci = (int(v) for v in input_sizes)
        _, _, _, _, kH, kW, Co, sH, sW, Ho, Wo = self._conv_dims((N, H, W, Ci), w.shape, strides, padding)
        assert dy.shape == (N, Ho, Wo, Co), "out_backprop shape mismatch"
        dx = np.empty((N, H, W, Ci), np.float32)
        self._fn("conv2d_backprop_input")(_fp(dy), _fp(w), _fp(dx), N, H, W, Ci, kH, kW, Co, sH, sW,
                                          _same(padding))
        return dx

    def conv2d_backprop_filter(self, x, filter_sizes, grad_out, strides, padding):
        x, dy = _c32(x), _c32(grad_out)
        kH, kW, Ci, Co = (int(v) for v in filter_sizes)
        N, H, W, _, _, _, _, sH, sW, Ho, Wo = self._conv_dims(x.shape, (kH, kW, Ci, Co), strides, padding)
        assert dy.shape == (N, Ho, Wo, Co), "out_backprop shape mismatch"
        dw = np.empty((kH, kW, Ci, Co), np.float32)
        self._fn("conv2d_backprop_filter")(_fp(x), _fp(dy), _fp(dw), N, H, W, Ci, kH, kW, Co, sH, sW,
                                           _same(padding))
        return dw

    # --------------------------------------------------- depthwise conv2d
    def depthwise_conv2d(self, x, w, strides=(1, 1, 1, 1), padding="SAME"):
        x, w = _c32(x), _c32(w)
        N, H, W, C = x.shape
        kH, kW, wc, dm = w.shape
        assert wc == C
        sH, sW = int(strides[1]), int(strides[2])
        Ho, _ = resolve_padding(H, kH, sH, padding)
        Wo, _ = resolve_padding(W, kW, sW, padding)
        y = np.empty((N, Ho, Wo, C * dm), np.float32)
        self._fn("depthwise_conv2d")(_fp(x), _fp(w), _fp(y), N, H, W, C, kH, kW, dm, sH, sW, _same(padding))
        return y

    def depthwise_conv2d_backprop_input(self, input_sizes, w, grad_out, strides, padding):
        w, dy = _c32(w), _c32(grad_out)
        N, H, W, C = (int(v) for v in input_sizes)
        kH, kW, _, dm = w.shape
        sH, sW = int(strides[1]), int(strides[2])
        dx = np.empty((N, H, W, C), np.float32)
        self._fn("depthwise_conv2d_backprop_input")(_fp(dy), _fp(w), _fp(dx), N, H, W, C, kH, kW, dm, sH, sW,
                                                    _same(padding))
        return dx

    def depthwise_conv2d_backprop_filter(self, x, filter_sizes, grad_out, strides, padding):
        x, dy = _c32(x), _c32(grad_out)
        kH, kW, C, dm = (int(v) for v in filter_sizes)
        N, H, W, _ = x.shape
        sH, sW = int(strides[1]), int(strides[2])
        dw = np.empty((kH, kW, C, dm), np.float32)
        self._fn("depthwise_conv2d_backprop_filter")(_fp(x), _fp(dy), _fp(dw), N, H, W, C, kH, kW, dm, sH,
                                                     sW, _same(padding))
        return dw

    # --------------------------------------------------------- elementwise
    def relu(self, x):
        x = _c32(x)
        y = np.empty_like(x)
        self._fn("relu")(_fp(x), _fp(y), x.size)
        return y

    def relu_grad(self, gradients, features):
        g, f = _c32(gradients), _c32(features)
        out = np.empty_like(g)
        self._fn("relu_grad")(_fp(g), _fp(f), _fp(out), g.size)
        return out

    def sigmoid(self, x):
        x = _c32(x)
        y = np.empty_like(x)
        self._fn("sigmoid")(_fp(x), _fp(y), x.size)
        return y

    def sigmoid_grad(self, y, dy):
        y, dy = _c32(y), _c32(dy)
        out = np.empty_like(y)
        self._fn("sigmoid_grad")(_fp(y), _fp(dy), _fp(out), y.size)
        return out

    # ----------------------------------------------------------- batchnorm
    def batch_norm_training(self, x, gamma, beta, epsilon=1e-3):
        x, g, b = _c32(x), _c32(gamma), _c32(beta)
        N, H, W, C = x.shape
        y = np.empty_like(x)
        m = np.empty(C, np.float32)
        v = np.empty(C, np.float32)
        self._fn("batch_norm_training")(_fp(x), _fp(g), _fp(b), _fp(y), _fp(m), _fp(v), N, H, W, C,
                                        float(epsilon))
        return y, m, v

    def batch_norm_inference(self, x, gamma, beta, mean, var, epsilon=1e-3):
        x, g, b, m, v = (_c32(a) for a in (x, gamma, beta, mean, var))
        N, H, W, C = x.shape
        y = np.empty_like(x)
        self._fn("batch_norm_inference")(_fp(x), _fp(g), _fp(b), _fp(m), _fp(v), _fp(y), N, H, W, C,
                                         float(epsilon))
        return y

    def batch_norm_grad(self, grad_y, x, gamma, saved_mean, saved_var, epsilon=1e-3):
        dy, x, g, m, v = (_c32(a) for a in (grad_y, x, gamma, saved_mean, saved_var))
        N, H, W, C = x.shape
        dx = np.empty_like(x)
        dg = np.empty(C, np.float32)
        db = np.empty(C, np.float32)
        self._fn("batch_norm_grad")(_fp(dy), _fp(x), _fp(g), _fp(m), _fp(v), _fp(dx), _fp(dg), _fp(db),
                                    N, H, W, C, float(epsilon))
        return dx, dg, db

    # --------------------------------------------------------------- dense
    def dense(self, x, w, b):
        x, w, b = _c32(x), _c32(w), _c32(b)
        batch, in_f = x.shape
        out_f = w.shape[1]
        y = np.empty((batch, out_f), np.float32)
        self._fn("dense")(_fp(x), _fp(w), _fp(b), _fp(y), batch, in_f, out_f)
        return y

    def dense_backprop_input(self, grad_y, w):
        dy, w = _c32(grad_y), _c32(w)
        batch, out_f = dy.shape
        in_f = w.shape[0]
        dx = np.empty((batch, in_f), np.float32)
        self._fn("dense_backprop_input")(_fp(dy), _fp(w), _fp(dx), batch, in_f, out_f)
        return dx

    def dense_backprop_weight(self, x, grad_y):
        x, dy = _c32(x), _c32(grad_y)
        batch, in_f = x.shape
        out_f = dy.shape[1]
        dw = np.empty((in_f, out_f), np.float32)
        self._fn("dense_backprop_weight")(_fp(x), _fp(dy), _fp(dw), batch, in_f, out_f)
        return dw

    def dense_backprop_bias(self, grad_y):
        dy = _c32(grad_y)
        batch, out_f = dy.shape
        db = np.empty(out_f, np.float32)
        self._fn("dense_backprop_bias")(_fp(dy), _fp(db), batch, out_f)
        return db

    # ---------------------------------------------------------- upsampling
    def upsampling_bilinear_2d(self, x, size):
        x = _c32(x)
        N, H, W, C = x.shape
        sy, sx = (int(s) for s in size)
        y = np.empty((N, H * sy, W * sx, C), np.float32)
        self._fn("upsampling_bilinear2d")(_fp(x), _fp(y), N, H, W, C, sy, sx)
        return y

    def upsampling_bilinear_2d_grad(self, grad_out, input_sizes, size):
        dy = _c32(grad_out)
        N, H, W, C = (int(v) for v in input_sizes)
        sy, sx = (int(s) for s in size)
        dx = np.empty((N, H, W, C), np.float32)
        self._fn("upsampling_bilinear2d_grad")(_fp(dy), _fp(dx), N, H, W, C, sy, sx)
        return dx


# ----------------------------------------------------------------------------
# float64 arbiter: the same maths in double precision (vectorised numpy).
# ----------------------------------------------------------------------------
class f64:
    """Float64 restatements; inputs are promoted, outputs are float64."""

    @staticmethod
    def _pad_geom(H, W, kH, kW, sH, sW, padding):
        Ho, pH = resolve_padding(H, kH, sH, padding)
        Wo, pW = resolve_padding(W, kW, sW, padding)
        Hp = max(H + pH, (Ho - 1) * sH + kH)
        Wp = max(W + pW, (Wo - 1) * sW + kW)
        return Ho, Wo, pH, pW, Hp, Wp

    @staticmethod
    def conv2d(x, w, strides, padding):
        x = np.asarray(x, np.float64)
        w = np.asarray(w, np.float64)
        N, H, W, Ci = x.shape
        kH, kW, _, Co = w.shape
        sH, sW = strides[1], strides[2]
        Ho, Wo, pH, pW, Hp, Wp = f64._pad_geom(H, W, kH, kW, sH, sW, padding)
        xp = np.zeros((N, Hp, Wp, Ci))
        xp[:, pH:pH + H, pW:pW + W] = x
        y = np.zeros((N, Ho, Wo, Co))
        for kh in range(kH):
            for kw in range(kW):
                patch = xp[:, kh:kh + sH * (Ho - 1) + 1:sH, kw:kw + sW * (Wo - 1) + 1:sW]
                y += patch @ w[kh, kw]
        return y

    @staticmethod
    def conv2d_backprop_input(input_sizes, w, dy, strides, padding):
        w = np.asarray(w, np.float64)
        dy = np.asarray(dy, np.float64)
        N, H, W, Ci = (int(v) for v in input_sizes)
        kH, kW, _, Co = w.shape
        sH, sW = strides[1], strides[2]
        Ho, Wo, pH, pW, Hp, Wp = f64._pad_geom(H, W, kH, kW, sH, sW, padding)
        dxp = np.zeros((N, Hp, Wp, Ci))
        for kh in range(kH):
            for kw in range(kW):
                dxp[:, kh:kh + sH * (Ho - 1) + 1:sH, kw:kw + sW * (Wo - 1) + 1:sW] += dy @ w[kh, kw].T
        return dxp[:, pH:pH + H, pW:pW + W]

    @staticmethod
    def conv2d_backprop_filter(x, filter_sizes, dy, strides, padding):
        x = np.asarray(x, np.float64)
        dy = np.asarray(dy, np.float64)
        N, H, W, Ci = x.shape
        kH, kW, _, Co = (int(v) for v in filter_sizes)
        sH, sW = strides[1], strides[2]
        Ho, Wo, pH, pW, Hp, Wp = f64._pad_geom(H, W, kH, kW, sH, sW, padding)
        xp = np.zeros((N, Hp, Wp, Ci))
        xp[:, pH:pH + H, pW:pW + W] = x
        dw = np.zeros((kH, kW, Ci, Co))
        dyf = dy.reshape(-1, Co)
        for kh in range(kH):
            for kw in range(kW):
                patch = xp[:, kh:kh + sH * (Ho - 1) + 1:sH, kw:kw + sW * (Wo - 1) + 1:sW]
                dw[kh, kw] = patch.reshape(-1, Ci).T @ dyf
        return dw

    @staticmethod
    def depthwise_conv2d(x, w, strides, padding):
        x = np.asarray(x, np.float64)
        w = np.asarray(w, np.float64)
        N, H, W, C = x.shape
        kH, kW, _, dm = w.shape
        sH, sW = strides[1], strides[2]
        Ho, Wo, pH, pW, Hp, Wp = f64._pad_geom(H, W, kH, kW, sH, sW, padding)
        xp = np.zeros((N, Hp, Wp, C))
        xp[:, pH:pH + H, pW:pW + W] = x
        y = np.zeros((N, Ho, Wo, C, dm))
        for kh in range(kH):
            for kw in range(kW):
                patch = xp[:, kh:kh + sH * (Ho - 1) + 1:sH, kw:kw + sW * (Wo - 1) + 1:sW]
                y += patch[..., None] * w[kh, kw]
        return y.reshape(N, Ho, Wo, C * dm)

    @staticmethod
    def depthwise_conv2d_backprop_input(input_sizes, w, dy, strides, padding):
        w = np.asarray(w, np.float64)
        dy = np.asarray(dy, np.float64)
        N, H, W, C = (int(v) for v in input_sizes)
        kH, kW, _, dm = w.shape
        sH, sW = strides[1], strides[2]
        Ho, Wo, pH, pW, Hp, Wp = f64._pad_geom(H, W, kH, kW, sH, sW, padding)
        dy5 = dy.reshape(N, Ho, Wo, C, dm)
        dxp = np.zeros((N, Hp, Wp, C))
        for kh in range(kH):
            for kw in range(kW):
                dxp[:, kh:kh + sH * (Ho - 1) + 1:sH, kw:kw + sW * (Wo - 1) + 1:sW] += (dy5 * w[kh, kw]).sum(-1)
        return dxp[:, pH:pH + H, pW:pW + W]

    @staticmethod
    def depthwise_conv2d_backprop_filter(x, filter_sizes, dy, strides, padding):
        x = np.asarray(x, np.float64)
        dy = np.asarray(dy, np.float64)
        N, H, W, C = x.shape
        kH, kW, _, dm = (int(v) for v in filter_sizes)
        sH, sW = strides[1], strides[2]
        Ho, Wo, pH, pW, Hp, Wp = f64._pad_geom(H, W, kH, kW, sH, sW, padding)
        xp = np.zeros((N, Hp, Wp, C))
        xp[:, pH:pH + H, pW:pW + W] = x
        dy5 = dy.reshape(N, Ho, Wo, C, dm)
        dw = np.zeros((kH, kW, C, dm))
        for kh in range(kH):
            for kw in range(kW):
                patch = xp[:, kh:kh + sH * (Ho - 1) + 1:sH, kw:kw + sW * (Wo - 1) + 1:sW]
                dw[kh, kw] = np.einsum("nhwc,nhwcd->cd", patch, dy5)
        return dw

    @staticmethod
    def sigmoid(x):
        return 1.0 / (1.0 + np.exp(-np.asarray(x, np.float64)))

    @staticmethod
    def sigmoid_grad(y, dy):
        y = np.asarray(y, np.float64)
        return np.asarray(dy, np.float64) * y * (1.0 - y)

    @staticmethod
    def batch_norm_training(x, gamma, beta, epsilon=1e-3):
        x = np.asarray(x, np.float64)
        C = x.shape[-1]
        xf = x.reshape(-1, C)
        mean = xf.mean(0)
        var = (xf * xf).mean(0) - mean * mean
        y = np.asarray(gamma, np.float64) * (x - mean) / np.sqrt(var + epsilon) + np.asarray(beta, np.float64)
        return y, mean, var

    @staticmethod
    def batch_norm_inference(x, gamma, beta, mean, var, epsilon=1e-3):
        x = np.asarray(x, np.float64)
        return (np.asarray(gamma, np.float64) * (x - np.asarray(mean, np.float64))
                / np.sqrt(np.asarray(var, np.float64) + epsilon) + np.asarray(beta, np.float64))

    @staticmethod
    def batch_norm_grad(dy, x, gamma, mean, var, epsilon=1e-3):
        dy = np.asarray(dy, np.float64)
        x = np.asarray(x, np.float64)
        C = x.shape[-1]
        inv = 1.0 / np.sqrt(np.asarray(var, np.float64) + epsilon)
        xh = (x - np.asarray(mean, np.float64)) * inv
        dbeta = dy.reshape(-1, C).sum(0)
        dgamma = (dy * xh).reshape(-1, C).sum(0)
        nhw = x.size // C
        dx = (np.asarray(gamma, np.float64) * inv / nhw) * (nhw * dy - dbeta - xh * dgamma)
        return dx, dgamma, dbeta

    @staticmethod
    def dense(x, w, b):
        return np.asarray(x, np.float64) @ np.asarray(w, np.float64) + np.asarray(b, np.float64)

    @staticmethod
    def dense_backprop_input(dy, w):
        return np.asarray(dy, np.float64) @ np.asarray(w, np.float64).T

    @staticmethod
    def dense_backprop_weight(x, dy):
        return np.asarray(x, np.float64).T @ np.asarray(dy, np.float64)

    @staticmethod
    def dense_backprop_bias(dy):
        return np.asarray(dy, np.float64).sum(0)

    @staticmethod
    def upsample_coords(in_size: int, out_size: int):
        """Per-axis clamped corners and fraction, computed in float32 exactly
        as kernels/upsampling_bilinear_kernels.cl:51-64 writes them."""
        o = np.arange(out_size, dtype=np.int64)
        f = ((o.astype(np.float32) + np.float32(0.5)) * np.float32(in_size)) / np.float32(out_size) - np.float32(0.5)
        f = f.astype(np.float32)
        i0 = np.floor(f).astype(np.int64)
        frac = (f - i0.astype(np.float32)).astype(np.float32)
        i1 = i0 + 1
        return np.clip(i0, 0, in_size - 1), np.clip(i1, 0, in_size - 1), frac

    @staticmethod
    def upsampling_bilinear_2d(x, size):
        x = np.asarray(x, np.float64)
        N, H, W, C = x.shape
        Ho, Wo = H * size[0], W * size[1]
        h0, h1, dh = f64.upsample_coords(H, Ho)
        w0, w1, dw = f64.upsample_coords(W, Wo)
        dh = dh.astype(np.float64)[None, :, None, None]
        dw = dw.astype(np.float64)[None, None, :, None]
        v00 = x[:, h0][:, :, w0]
        v01 = x[:, h0][:, :, w1]
        v10 = x[:, h1][:, :, w0]
        v11 = x[:, h1][:, :, w1]
        return (1 - dh) * (1 - dw) * v00 + (1 - dh) * dw * v01 + dh * (1 - dw) * v10 + dh * dw * v11

    @staticmethod
    def upsampling_bilinear_2d_grad(dy, input_sizes, size):
        dy = np.asarray(dy, np.float64)
        N, H, W, C = (int(v) for v in input_sizes)
        Ho, Wo = H * size[0], W * size[1]
        h0, h1, dh = f64.upsample_coords(H, Ho)
        w0, w1, dw = f64.upsample_coords(W, Wo)
        Ah = np.zeros((H, Ho))
        Aw = np.zeros((W, Wo))
        np.add.at(Ah, (h0, np.arange(Ho)), 1 - dh.astype(np.float64))
        np.add.at(Ah, (h1, np.arange(Ho)), dh.astype(np.float64))
        np.add.at(Aw, (w0, np.arange(Wo)), 1 - dw.astype(np.float64))
        np.add.at(Aw, (w1, np.arange(Wo)), dw.astype(np.float64))
        return np.einsum("ho,nopc,wp->nhwc", Ah, dy, Aw)


def rel_err(got, want):
    """(max |got-want| / max |want|, ||got-want||_2 / ||want||_2) in float64."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    d = got - want
    scale = np.abs(want).max() if want.size else 0.0
    nrm = np.linalg.norm(want.ravel())
    mx = float(np.abs(d).max() / scale) if scale > 0 else float(np.abs(d).max() if d.size else 0.0)
    l2 = float(np.linalg.norm(d.ravel()) / nrm) if nrm > 0 else float(np.linalg.norm(d.ravel()))
    return mx, l2


if os.environ.get("B2_ORACLE_AUTOBUILD", "0") == "1" and not LIBS["port"].exists():
    build()
