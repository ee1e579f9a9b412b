"""Loads the B200 backend library (``libb2ocl.so``) and exposes the 19 ops.

This module plays the role of the reference's ``opencl_tf/_library.py`` (which
calls ``tf.load_op_library``, opencl_tf/_library.py:25-34): it loads the
compiled op library, fails with ``ImportError`` when it is missing, and
publishes ``raw_ops``, a namespace holding one function per reference op under
TF's snake_case op names (``opencl_conv2d``, ``opencl_batch_norm_grad``, ...).

Tensors are torch CUDA tensors (float32, NHWC / HWIO like the reference);
shape arguments the reference marks ``HostMemory`` (``input_sizes``,
``filter_sizes``) are host values (list, tuple, ``torch.Size`` or a CPU
tensor).  Every op runs asynchronously on torch's current CUDA stream, writes
into outputs allocated here (as ``allocate_output`` does in the reference),
and raises :class:`opencl_tf.errors.InvalidArgumentError` /
:class:`~opencl_tf.errors.InternalError` where the reference op returns
``InvalidArgument`` / ``Internal``.  There is no CPU or fallback path: without
the library, importing ``opencl_tf`` fails.

Gradients follow the TF model: ``RegisterGradient(op_type)`` attaches a
gradient function ``fn(op, *grads)`` to an op type (see ``gradients.py``), and
any raw op whose inputs require grad records an autograd node that calls it.
"""
from __future__ import annotations

import ctypes
import os
import types
from pathlib import Path

import torch

from . import errors

_HERE = Path(__file__).resolve().parent
_LIB_PATH = Path(os.environ.get("B2_LIBRARY", _HERE / "libb2ocl.so"))

if not _LIB_PATH.exists():
    raise ImportError(
        f"libb2ocl.so not found at {_LIB_PATH}.\n"
        "Build it first:\n"
        "    python opencl-tensorflow_b200/build.py")

_lib = ctypes.CDLL(str(_LIB_PATH))

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F32 = ctypes.c_float
_S = ctypes.c_char_p
_I64x4 = _I64 * 4
_I64x2 = _I64 * 2
_I32x4 = ctypes.c_int32 * 4

_SIGS = {
    "b2_init": [_I],
    "b2_abi_version": [],
    "b2_resolve_padding": [_I64, _I64, _I64, _S, ctypes.POINTER(_I64), ctypes.POINTER(_I64)],
    "b2_conv2d_output_shape": [_P, _P, _P, _I, _S, _P],
    "b2_depthwise_conv2d_output_shape": [_P, _P, _P, _I, _S, _P],
    "b2_conv2d": [_P, _P, _P, _P, _P, _P, _I, _S, _P, _P],
    "b2_conv2d_backprop_input": [_P, _P, _P, _P, _P, _P, _P, _I, _S, _P],
    "b2_conv2d_backprop_filter": [_P, _P, _P, _P, _P, _P, _P, _I, _S, _P],
    "b2_depthwise_conv2d": [_P, _P, _P, _P, _P, _P, _I, _S, _P, _P],
    "b2_depthwise_conv2d_backprop_input": [_P, _P, _P, _P, _P, _P, _P, _I, _S, _P],
    "b2_depthwise_conv2d_backprop_filter": [_P, _P, _P, _P, _P, _P, _P, _I, _S, _P],
    "b2_relu": [_P, _P, _P, _I64],
    "b2_relu_grad": [_P, _P, _P, _P, _I64],
    "b2_sigmoid": [_P, _P, _P, _I64],
    "b2_sigmoid_grad": [_P, _P, _P, _P, _I64],
    "b2_batch_norm_training": [_P, _P, _P, _P, _I64, _P, _I64, _F32, _P, _P, _P],
    "b2_batch_norm_inference": [_P, _P, _P, _P, _I64, _P, _I64, _P, _I64, _P, _I64, _F32, _P],
    "b2_batch_norm_grad": [_P, _P, _P, _P, _P, _P, _P, _P, _F32, _P, _P, _P],
    "b2_batch_norm_update_moving": [_P, _P, _P, _P, _P, _I64, _F32, _F32],
    "b2_batch_norm_relu_training": [_P, _P, _P, _P, _I64, _P, _I64, _F32, _P, _P, _P, _P, _P, _F32, _F32],
    "b2_batch_norm_relu_grad": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _F32, _P, _P, _P],
    "b2_dense": [_P, _P, _P, _P, _P, _P, _I64, _P],
    "b2_dense_relu": [_P, _P, _P, _P, _P, _P, _I64, _P],
    "b2_dense_backprop_input": [_P, _P, _P, _P, _P, _P],
    "b2_dense_backprop_weight": [_P, _P, _P, _P, _P, _P],
    "b2_dense_backprop_bias": [_P, _P, _P, _P],
    "b2_upsampling_bilinear2d": [_P, _P, _P, _P, _I, _P],
    "b2_upsampling_bilinear2d_grad": [_P, _P, _P, _P, _P, _I, _P],
    "b2_upsampling_coords": [_P, ctypes.c_int32, ctypes.c_int32, _P, _P, _P],
    "b2_mse_loss": [_P, _P, _P, _I64, _P],
    "b2_mse_loss_grad": [_P, _P, _P, _I64, _P, _P],
    "b2_adam_update": [_P, _I, _P, _P, _P, _P, _P, _F32, _F32, _F32, _F32, _F32, _F32, _P, _P],
    "b2_pool_trim": [],
    "b2_device_timeouts": [ctypes.POINTER(ctypes.c_uint)],
    "b2_stream_status": [_P],
    "b2_set_wait_limit_ns": [ctypes.c_uint64],
    "b2_set_reserved_sms": [_I],
    "b2_kernel_launch_count": [ctypes.POINTER(ctypes.c_uint64)],
}
for _name, _args in _SIGS.items():
    _fn = getattr(_lib, _name)
    _fn.argtypes = _args
    _fn.restype = _I
_lib.b2_last_error.restype = ctypes.c_char_p
_lib.b2_last_error.argtypes = []
_U8P = ctypes.POINTER(ctypes.c_ubyte)
_VPP = ctypes.POINTER(ctypes.c_void_p)
_lib.b2_peer_exchange_bytes.restype = ctypes.c_size_t
_lib.b2_peer_exchange_bytes.argtypes = [_I64, _I]
for _name, _args in {"b2_peer_buffer_create": [ctypes.c_size_t, _VPP, _U8P],
                     "b2_peer_buffer_open": [_U8P, _VPP],
                     "b2_peer_buffer_close": [_P], "b2_peer_buffer_free": [_P],
                     "b2_peer_allreduce_avg": [_P, _P, _I64, _I, _I, _VPP, _P]}.items():
    getattr(_lib, _name).argtypes = _args
    getattr(_lib, _name).restype = _I


class PoolStats(ctypes.Structure):
    _fields_ = [("bytes_in_use", ctypes.c_uint64), ("bytes_reserved", ctypes.c_uint64),
                ("peak_in_use", ctypes.c_uint64), ("num_allocs", ctypes.c_uint64)]


_lib.b2_pool_stats.argtypes = [ctypes.POINTER(PoolStats)]
_lib.b2_pool_stats.restype = _I

library_path = str(_LIB_PATH)


def _check(rc: int) -> None:
    if rc != 0:
        raise errors.from_status(rc, _lib.b2_last_error().decode(errors="replace"))


# ---------------------------------------------------------------- helpers

def _stream(t: torch.Tensor):
    return torch.cuda.current_stream(t.device).cuda_stream


def _input(t, what: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise errors.InvalidArgumentError(f"{what} must be a torch tensor on a CUDA device")
    if not t.is_cuda:
        raise errors.InvalidArgumentError(
            f"{what} must live on a CUDA device (this backend has no CPU path)")
    if t.dtype != torch.float32:
        raise errors.InvalidArgumentError(f"{what} must be float32, got {t.dtype}")
    return t if t.is_contiguous() else t.contiguous()


def _rank(t: torch.Tensor, r: int, msg: str) -> None:
    if t.dim() != r:
        raise errors.InvalidArgumentError(msg)


def _host_ints(v, n: int, what: str) -> list[int]:
    if isinstance(v, torch.Tensor):
        v = v.detach().cpu().tolist()
    v = [int(a) for a in v]
    if len(v) != n:
        raise errors.InvalidArgumentError(f"{what} must have {n} elements")
    return v


def _strides_arr(strides):
    s = [int(a) for a in strides]
    return (ctypes.c_int32 * len(s))(*s), len(s)


def _padding(padding) -> bytes:
    if isinstance(padding, bytes):
        padding = padding.decode()
    return str(padding).encode()


class _on_device:
    """Makes ``t``'s device current for the C library (it uses the calling
    thread's current device)."""

    __slots__ = ("idx", "prev")

    def __init__(self, t: torch.Tensor):
        self.idx = t.device.index if t.device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


def _p(t: torch.Tensor) -> int:
    return t.data_ptr()


# ------------------------------------------------------------ raw kernels
# One function per reference op, no autograd.  Argument names follow the
# REGISTER_OP input names.

def _k_conv2d(input, filter, strides, padding):
    x = _input(input, "input")
    w = _input(filter, "filter")
    _rank(x, 4, "input must be rank 4")
    _rank(w, 4, "filter must be rank 4")
    st, ns = _strides_arr(strides)
    xs, ws, ys = _I64x4(*x.shape), _I64x4(*w.shape), _I64x4()
    pad = _padding(padding)
    _check(_lib.b2_conv2d_output_shape(xs, ws, st, ns, pad, ys))
    y = torch.empty(tuple(ys), device=x.device, dtype=torch.float32)
    with _on_device(x):
        _check(_lib.b2_conv2d(_stream(x), _p(x), xs, _p(w), ws, st, ns, pad, _p(y), ys))
    return y


def _k_conv2d_backprop_input(input_sizes, filter, out_backprop, strides, padding):
    sizes = _host_ints(input_sizes, 4, "input_sizes")
    w = _input(filter, "filter")
    dy = _input(out_backprop, "out_backprop")
    _rank(w, 4, "filter must be rank 4")
    _rank(dy, 4, "out_backprop must be rank 4")
    st, ns = _strides_arr(strides)
    dx = torch.empty(tuple(sizes), device=w.device, dtype=torch.float32)
    with _on_device(w):
        _check(_lib.b2_conv2d_backprop_input(_stream(w), _I32x4(*sizes), _p(w), _I64x4(*w.shape), _p(dy),
                                             _I64x4(*dy.shape), st, ns, _padding(padding), _p(dx)))
    return dx


def _k_conv2d_backprop_filter(input, filter_sizes, out_backprop, strides, padding):
    x = _input(input, "input")
    sizes = _host_ints(filter_sizes, 4, "filter_sizes")
    dy = _input(out_backprop, "out_backprop")
    _rank(x, 4, "input must be rank 4")
    _rank(dy, 4, "out_backprop must be rank 4")
    st, ns = _strides_arr(strides)
    dw = torch.empty(tuple(sizes), device=x.device, dtype=torch.float32)
    with _on_device(x):
        _check(_lib.b2_conv2d_backprop_filter(_stream(x), _p(x), _I64x4(*x.shape), _I32x4(*sizes), _p(dy),
                                              _I64x4(*dy.shape), st, ns, _padding(padding), _p(dw)))
    return dw


def _k_depthwise_conv2d(input, filter, strides, padding):
    x = _input(input, "input")
    w = _input(filter, "filter")
    _rank(x, 4, "input must be rank 4")
    _rank(w, 4, "filter must be rank 4")
    st, ns = _strides_arr(strides)
    xs, ws, ys = _I64x4(*x.shape), _I64x4(*w.shape), _I64x4()
    pad = _padding(padding)
    _check(_lib.b2_depthwise_conv2d_output_shape(xs, ws, st, ns, pad, ys))
    y = torch.empty(tuple(ys), device=x.device, dtype=torch.float32)
    with _on_device(x):
        _check(_lib.b2_depthwise_conv2d(_stream(x), _p(x), xs, _p(w), ws, st, ns, pad, _p(y), ys))
    return y


def _k_depthwise_conv2d_backprop_input(input_sizes, filter, out_backprop, strides, padding):
    sizes = _host_ints(input_sizes, 4, "input_sizes")
    w = _input(filter, "filter")
    dy = _input(out_backprop, "out_backprop")
    _rank(w, 4, "filter must be rank 4")
    _rank(dy, 4, "out_backprop must be rank 4")
    st, ns = _strides_arr(strides)
    dx = torch.empty(tuple(sizes), device=w.device, dtype=torch.float32)
    with _on_device(w):
        _check(_lib.b2_depthwise_conv2d_backprop_input(_stream(w), _I32x4(*sizes), _p(w), _I64x4(*w.shape),
                                                       _p(dy), _I64x4(*dy.shape), st, ns, _padding(padding),
                                                       _p(dx)))
    return dx


def _k_depthwise_conv2d_backprop_filter(input, filter_sizes, out_backprop, strides, padding):
    x = _input(input, "input")
    sizes = _host_ints(filter_sizes, 4, "filter_sizes")
    dy = _input(out_backprop, "out_backprop")
    _rank(x, 4, "input must be rank 4")
    _rank(dy, 4, "out_backprop must be rank 4")
    st, ns = _strides_arr(strides)
    dw = torch.empty(tuple(sizes), device=x.device, dtype=torch.float32)
    with _on_device(x):
        _check(_lib.b2_depthwise_conv2d_backprop_filter(_stream(x), _p(x), _I64x4(*x.shape), _I32x4(*sizes),
                                                        _p(dy), _I64x4(*dy.shape), st, ns, _padding(padding),
                                                        _p(dw)))
    return dw


def _k_relu(input):
    x = _input(input, "input")
    y = torch.empty_like(x)
    with _on_device(x):
        _check(_lib.b2_relu(_stream(x), _p(x), _p(y), x.numel()))
    return y


def _k_relu_grad(gradients, features):
    g = _input(gradients, "gradients")
    f = _input(features, "features")
    if g.shape != f.shape:
        raise errors.InvalidArgumentError("gradients and features must have equal shape")
    out = torch.empty_like(g)
    with _on_device(g):
        _check(_lib.b2_relu_grad(_stream(g), _p(g), _p(f), _p(out), g.numel()))
    return out


def _k_sigmoid(input):
    x = _input(input, "input")
    y = torch.empty_like(x)
    with _on_device(x):
        _check(_lib.b2_sigmoid(_stream(x), _p(x), _p(y), x.numel()))
    return y


def _k_sigmoid_grad(y, dy):
    y = _input(y, "y")
    dy = _input(dy, "dy")
    if y.shape != dy.shape:
        raise errors.InvalidArgumentError("y and dy must have equal shape")
    out = torch.empty_like(y)
    with _on_device(y):
        _check(_lib.b2_sigmoid_grad(_stream(y), _p(y), _p(dy), _p(out), y.numel()))
    return out


def _k_batch_norm_training(x, gamma, beta, epsilon=1e-3):
    x = _input(x, "x")
    g = _input(gamma, "gamma")
    b = _input(beta, "beta")
    _rank(x, 4, "x must be NHWC")
    C = x.shape[3]
    y = torch.empty_like(x)
    mean = torch.empty(C, device=x.device, dtype=torch.float32)
    var = torch.empty(C, device=x.device, dtype=torch.float32)
    with _on_device(x):
        _check(_lib.b2_batch_norm_training(_stream(x), _p(x), _I64x4(*x.shape), _p(g), g.numel(), _p(b), b.numel(),
                                           float(epsilon), _p(y), _p(mean), _p(var)))
    return y, mean, var


def batch_norm_update_moving(moving_mean, moving_var, batch_mean, batch_var, momentum):
    """moving = momentum * moving + (1 - momentum) * batch, in place, for the
    mean and variance buffers in one launch (opencl_tf/layers.py:189-194)."""
    bufs = (moving_mean, moving_var, batch_mean, batch_var)
    C = moving_mean.numel()
    if any(not (t.is_cuda and t.dtype == torch.float32 and t.is_contiguous() and t.numel() == C) for t in bufs):
        raise errors.InvalidArgumentError("moving/batch statistics must be contiguous fp32 CUDA vectors of one length")
    with _on_device(moving_mean):
        _check(_lib.b2_batch_norm_update_moving(_stream(moving_mean), _p(moving_mean), _p(moving_var),
                                                _p(batch_mean), _p(batch_var), C, float(momentum),
                                                float(1.0 - momentum)))


def _k_batch_norm_relu_training(x, gamma, beta, epsilon=1e-3, moving=None):
    """moving: optional (moving_mean, moving_var, momentum), updated in place."""
    x = _input(x, "x")
    g = _input(gamma, "gamma")
    b = _input(beta, "beta")
    _rank(x, 4, "x must be NHWC")
    C = x.shape[3]
    z = torch.empty_like(x)
    mean = torch.empty(C, device=x.device, dtype=torch.float32)
    var = torch.empty(C, device=x.device, dtype=torch.float32)
    mm = mv = None
    mom = 0.0
    if moving is not None:
        mm, mv, mom = moving
        for t in (mm, mv):
            if not (t.is_cuda and t.dtype == torch.float32 and t.is_contiguous() and t.numel() == C):
                raise errors.InvalidArgumentError("moving statistics must be contiguous fp32 CUDA vectors of C")
    with _on_device(x):
        _check(_lib.b2_batch_norm_relu_training(_stream(x), _p(x), _I64x4(*x.shape), _p(g), g.numel(), _p(b),
                                                b.numel(), float(epsilon), _p(z), _p(mean), _p(var),
                                                _p(mm) if mm is not None else None,
                                                _p(mv) if mv is not None else None, float(mom),
                                                float(1.0 - mom)))
    return z, mean, var


def _k_batch_norm_relu_grad(grad_z, x, gamma, beta, saved_mean, saved_var, epsilon=1e-3):
    dz = _input(grad_z, "grad_z")
    x = _input(x, "x")
    g, b = _input(gamma, "gamma"), _input(beta, "beta")
    m, v = _input(saved_mean, "saved_mean"), _input(saved_var, "saved_var")
    if x.dim() != 4 or dz.shape != x.shape:
        raise errors.InvalidArgumentError("grad_z and x must have matching NHWC shapes")
    C = x.shape[3]
    if g.numel() < C or b.numel() < C or m.numel() < C or v.numel() < C:
        raise errors.InvalidArgumentError("gamma/beta/saved_mean/saved_var must have C elements")
    dx = torch.empty_like(x)
    dg = torch.empty(C, device=x.device, dtype=torch.float32)
    db = torch.empty(C, device=x.device, dtype=torch.float32)
    with _on_device(x):
        _check(_lib.b2_batch_norm_relu_grad(_stream(x), _p(dz), _I64x4(*dz.shape), _p(x), _I64x4(*x.shape), _p(g),
                                            _p(b), _p(m), _p(v), float(epsilon), _p(dx), _p(dg), _p(db)))
    return dx, dg, db


def _k_batch_norm_inference(x, gamma, beta, mean, var, epsilon=1e-3):
    x = _input(x, "x")
    g, b = _input(gamma, "gamma"), _input(beta, "beta")
    m, v = _input(mean, "mean"), _input(var, "var")
    _rank(x, 4, "x must be NHWC")
    y = torch.empty_like(x)
    with _on_device(x):
        _check(_lib.b2_batch_norm_inference(_stream(x), _p(x), _I64x4(*x.shape), _p(g), g.numel(), _p(b),
                                            b.numel(), _p(m), m.numel(), _p(v), v.numel(), float(epsilon), _p(y)))
    return y


def _k_batch_norm_grad(grad_y, x, gamma, saved_mean, saved_var, epsilon=1e-3):
    dy = _input(grad_y, "grad_y")
    x = _input(x, "x")
    g = _input(gamma, "gamma")
    m, v = _input(saved_mean, "saved_mean"), _input(saved_var, "saved_var")
    if x.dim() != 4 or dy.shape != x.shape:
        raise errors.InvalidArgumentError("grad_y and x must have matching NHWC shapes")
    C = x.shape[3]
    if g.numel() < C or m.numel() < C or v.numel() < C:
        raise errors.InvalidArgumentError("gamma/saved_mean/saved_var must have C elements")
    dx = torch.empty_like(x)
    dg = torch.empty(C, device=x.device, dtype=torch.float32)
    db = torch.empty(C, device=x.device, dtype=torch.float32)
    with _on_device(x):
        _check(_lib.b2_batch_norm_grad(_stream(x), _p(dy), _I64x4(*dy.shape), _p(x), _I64x4(*x.shape), _p(g),
                                       _p(m), _p(v), float(epsilon), _p(dx), _p(dg), _p(db)))
    return dx, dg, db


def _dense_call(x, w, b, relu):
    x = _input(x, "x")
    w = _input(w, "W")
    b = _input(b, "b")
    _rank(x, 2, "x must be rank 2")
    _rank(w, 2, "W must be rank 2")
    _rank(b, 1, "b must be rank 1")
    y = torch.empty((x.shape[0], w.shape[1]), device=x.device, dtype=torch.float32)
    entry = _lib.b2_dense_relu if relu else _lib.b2_dense
    with _on_device(x):
        _check(entry(_stream(x), _p(x), _I64x2(*x.shape), _p(w), _I64x2(*w.shape), _p(b), b.shape[0], _p(y)))
    return y


def _k_dense(x, w, b):
    return _dense_call(x, w, b, False)


def _k_dense_relu(x, w, b):
    return _dense_call(x, w, b, True)


def _k_dense_backprop_input(grad_y, w):
    dy = _input(grad_y, "grad_y")
    w = _input(w, "W")
    _rank(dy, 2, "grad_y must be rank 2")
    _rank(w, 2, "W must be rank 2")
    dx = torch.empty((dy.shape[0], w.shape[0]), device=dy.device, dtype=torch.float32)
    with _on_device(dy):
        _check(_lib.b2_dense_backprop_input(_stream(dy), _p(dy), _I64x2(*dy.shape), _p(w), _I64x2(*w.shape),
                                            _p(dx)))
    return dx


def _k_dense_backprop_weight(x, grad_y):
    x = _input(x, "x")
    dy = _input(grad_y, "grad_y")
    _rank(x, 2, "x must be rank 2")
    _rank(dy, 2, "grad_y must be rank 2")
    dw = torch.empty((x.shape[1], dy.shape[1]), device=x.device, dtype=torch.float32)
    with _on_device(x):
        _check(_lib.b2_dense_backprop_weight(_stream(x), _p(x), _I64x2(*x.shape), _p(dy), _I64x2(*dy.shape),
                                             _p(dw)))
    return dw


def _k_dense_backprop_bias(grad_y):
    dy = _input(grad_y, "grad_y")
    _rank(dy, 2, "grad_y must be rank 2")
    db = torch.empty((dy.shape[1],), device=dy.device, dtype=torch.float32)
    with _on_device(dy):
        _check(_lib.b2_dense_backprop_bias(_stream(dy), _p(dy), _I64x2(*dy.shape), _p(db)))
    return db


def _pred_target(pred, target):
    p = _input(pred, "y_pred")
    t = _input(target, "y_true")
    if p.shape != t.shape:
        raise errors.InvalidArgumentError(
            f"y_pred and y_true must have the same shape, got {tuple(p.shape)} and {tuple(t.shape)}")
    if p.device != t.device:
        raise errors.InvalidArgumentError("y_pred and y_true must live on the same device")
    if p.numel() == 0:
        raise errors.InvalidArgumentError("mean squared error of an empty batch is undefined")
    return p, t


def _k_mse_loss(pred, target):
    p, t = _pred_target(pred, target)
    loss = torch.empty((), device=p.device, dtype=torch.float32)
    with _on_device(p):
        _check(_lib.b2_mse_loss(_stream(p), _p(p), _p(t), p.numel(), _p(loss)))
    return loss


def _k_mse_loss_grad(pred, target, grad_loss):
    p, t = _pred_target(pred, target)
    g = _input(grad_loss, "grad_loss")
    if g.numel() != 1 or g.device != p.device:
        raise errors.InvalidArgumentError("grad_loss must be a scalar on the prediction's device")
    out = torch.empty_like(p)
    with _on_device(p):
        _check(_lib.b2_mse_loss_grad(_stream(p), _p(p), _p(t), p.numel(), _p(g), _p(out)))
    return out


def adam_update(params, grads, ms, vs, learning_rate, beta_1, beta_2, epsilon, iterations, ticket):
    """One Keras Adam update of every (param, grad, m, v) quadruple in one
    multi-tensor launch (all fp32, contiguous, on one device); ``iterations``
    (int64 scalar) and ``ticket`` (32-bit scalar, zero) are the optimizer's
    device state.  ``1 - beta`` is rounded as Keras rounds it: in double, then
    to fp32."""
    n = len(params)
    if not (len(grads) == len(ms) == len(vs) == n):
        raise errors.InvalidArgumentError("params, grads, m and v must have the same length")
    if n == 0:
        return
    dev = params[0].device
    for group in (params, grads, ms, vs):
        for t in group:
            if not (isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()
                    and t.device == dev):
                raise errors.InvalidArgumentError(
                    "Adam operands must be contiguous fp32 tensors on the parameters' CUDA device")
    for a, b, c, d in zip(params, grads, ms, vs):
        if not (a.numel() == b.numel() == c.numel() == d.numel()):
            raise errors.InvalidArgumentError("a parameter, its gradient and its slots must have the same size")
    if not (iterations.is_cuda and iterations.dtype == torch.int64 and iterations.device == dev and
            ticket.is_cuda and ticket.element_size() == 4 and ticket.device == dev):
        raise errors.InvalidArgumentError("iterations (int64) and ticket (32-bit) must live on the parameters' device")
    arr = ctypes.c_void_p * n
    with _on_device(params[0]):
        _check(_lib.b2_adam_update(_stream(params[0]), n, arr(*(_p(t) for t in params)),
                                   arr(*(_p(t) for t in grads)), arr(*(_p(t) for t in ms)),
                                   arr(*(_p(t) for t in vs)), (_I64 * n)(*(t.numel() for t in params)),
                                   float(learning_rate), float(beta_1), float(beta_2), float(1.0 - beta_1),
                                   float(1.0 - beta_2), float(epsilon), _p(iterations), _p(ticket)))


def _size_arr(size):
    s = [int(a) for a in size]
    return (ctypes.c_int32 * len(s))(*s), len(s)


def _k_upsampling_bilinear2d(input, size):
    x = _input(input, "input")
    _rank(x, 4, "input must be NHWC")
    sz, n = _size_arr(size)
    if n != 2:
        raise errors.InvalidArgumentError("size must have exactly 2 elements")
    if sz[0] < 1 or sz[1] < 1:
        raise errors.InvalidArgumentError("size elements must be >= 1")
    N, H, W, C = x.shape
    y = torch.empty((N, H * sz[0], W * sz[1], C), device=x.device, dtype=torch.float32)
    with _on_device(x):
        _check(_lib.b2_upsampling_bilinear2d(_stream(x), _p(x), _I64x4(*x.shape), sz, n, _p(y)))
    return y


def _k_upsampling_bilinear2d_grad(grad_out, input_sizes, size):
    dy = _input(grad_out, "grad_out")
    sizes = _host_ints(input_sizes, 4, "input_sizes [N,H,W,C]")
    _rank(dy, 4, "grad_out must be NHWC")
    sz, n = _size_arr(size)
    dx = torch.empty(tuple(sizes), device=dy.device, dtype=torch.float32)
    with _on_device(dy):
        _check(_lib.b2_upsampling_bilinear2d_grad(_stream(dy), _p(dy), _I64x4(*dy.shape), _I32x4(*sizes), sz, n,
                                                  _p(dx)))
    return dx


# ------------------------------------------------------- gradient registry

_GRADIENTS: dict = {}


def RegisterGradient(op_type: str):
    """Decorator attaching ``fn(op, *output_grads) -> list of input grads`` to
    ``op_type`` -- the role of ``tf.RegisterGradient`` in the reference."""

    def deco(fn):
        _GRADIENTS[op_type] = fn
        return fn

    return deco


class Operation:
    """What a gradient function sees: the op's type, inputs, outputs, attrs
    (``op.inputs[i]``, ``op.outputs[i]``, ``op.get_attr(name)`` as in TF) and
    which inputs need a gradient."""

    __slots__ = ("type", "inputs", "outputs", "_attrs", "needs_input_grad")

    def __init__(self, type_, inputs, outputs, attrs, needs):
        self.type = type_
        self.inputs = inputs
        self.outputs = outputs
        self._attrs = attrs
        self.needs_input_grad = needs

    def get_attr(self, name):
        return self._attrs[name]


class _OpNode(torch.autograd.Function):
    @staticmethod
    def forward(ctx, op_type, attrs, kernel, nondiff, *inputs):
        outs = kernel(*inputs, **attrs)
        tup = outs if isinstance(outs, tuple) else (outs,)
        ctx.op_type = op_type
        ctx.attrs = attrs
        ctx.n_in = len(inputs)
        ctx.save_for_backward(*inputs, *tup)
        ctx.set_materialize_grads(False)
        if nondiff:
            ctx.mark_non_differentiable(*(tup[i] for i in nondiff))
        return outs

    @staticmethod
    def backward(ctx, *grads):
        saved = ctx.saved_tensors
        op = Operation(ctx.op_type, saved[:ctx.n_in], saved[ctx.n_in:], ctx.attrs, ctx.needs_input_grad[4:])
        fn = _GRADIENTS.get(ctx.op_type)
        if fn is None:
            raise LookupError(f"No gradient defined for operation '{ctx.op_type}' (op type: {ctx.op_type})")
        if grads[0] is None:
            return (None,) * (4 + ctx.n_in)
        res = list(fn(op, *grads))
        res = [r if need else None for r, need in zip(res, op.needs_input_grad)]
        return (None, None, None, None, *res)


def _apply(op_type: str, kernel, inputs, attrs, nondiff=()):
    if torch.is_grad_enabled() and any(isinstance(t, torch.Tensor) and t.requires_grad for t in inputs):
        return _OpNode.apply(op_type, attrs, kernel, tuple(nondiff), *inputs)
    return kernel(*inputs, **attrs)


# --------------------------------------------------------------- raw_ops

# B2_NVTX=1: every op call is an NVTX range named after the op (for nsys /
# ncu --nvtx filtering), the tracing hook the reference's roadmap plans.
_NVTX = os.environ.get("B2_NVTX", "0") not in ("", "0")


def _traced(name: str, fn):
    if not _NVTX:
        return fn

    def wrapper(*args, **kwargs):
        torch.cuda.nvtx.range_push(name)
        try:
            return fn(*args, **kwargs)
        finally:
            torch.cuda.nvtx.range_pop()

    wrapper.__name__ = fn.__name__
    wrapper.__doc__ = fn.__doc__
    return wrapper


def _mk_raw_ops():
    ns = types.SimpleNamespace()

    def opencl_conv2d(input, filter, strides, padding):
        return _apply("OpenclConv2d", _k_conv2d, (input, filter),
                      {"strides": list(strides), "padding": padding})

    def opencl_conv2d_backprop_input(input_sizes, filter, out_backprop, strides, padding):
        return _k_conv2d_backprop_input(input_sizes, filter, out_backprop, list(strides), padding)

    def opencl_conv2d_backprop_filter(input, filter_sizes, out_backprop, strides, padding):
        return _k_conv2d_backprop_filter(input, filter_sizes, out_backprop, list(strides), padding)

    def opencl_depthwise_conv2d(input, filter, strides, padding):
        return _apply("OpenclDepthwiseConv2d", _k_depthwise_conv2d, (input, filter),
                      {"strides": list(strides), "padding": padding})

    def opencl_depthwise_conv2d_backprop_input(input_sizes, filter, out_backprop, strides, padding):
        return _k_depthwise_conv2d_backprop_input(input_sizes, filter, out_backprop, list(strides), padding)

    def opencl_depthwise_conv2d_backprop_filter(input, filter_sizes, out_backprop, strides, padding):
        return _k_depthwise_conv2d_backprop_filter(input, filter_sizes, out_backprop, list(strides), padding)

    def opencl_relu(input):
        return _apply("OpenclRelu", _k_relu, (input,), {})

    def opencl_relu_grad(gradients, features):
        return _k_relu_grad(gradients, features)

    def opencl_sigmoid(input):
        return _apply("OpenclSigmoid", _k_sigmoid, (input,), {})

    def opencl_sigmoid_grad(y, dy):
        return _k_sigmoid_grad(y, dy)

    def opencl_batch_norm_training(x, gamma, beta, epsilon=1e-3):
        return _apply("OpenclBatchNormTraining", _k_batch_norm_training, (x, gamma, beta),
                      {"epsilon": float(epsilon)}, nondiff=(1, 2))

    def opencl_batch_norm_inference(x, gamma, beta, mean, var, epsilon=1e-3):
        return _apply("OpenclBatchNormInference", _k_batch_norm_inference, (x, gamma, beta, mean, var),
                      {"epsilon": float(epsilon)})

    def opencl_batch_norm_grad(grad_y, x, gamma, saved_mean, saved_var, epsilon=1e-3):
        return _k_batch_norm_grad(grad_y, x, gamma, saved_mean, saved_var, float(epsilon))


    def opencl_dense(x, w, b):
        return _apply("OpenclDense", _k_dense, (x, w, b), {})

    def opencl_dense_backprop_input(grad_y, w):
        return _k_dense_backprop_input(grad_y, w)

    def opencl_dense_backprop_weight(x, grad_y):
        return _k_dense_backprop_weight(x, grad_y)

    def opencl_dense_backprop_bias(grad_y):
        return _k_dense_backprop_bias(grad_y)

    def opencl_upsampling_bilinear2d(input, size):
        return _apply("OpenclUpsamplingBilinear2d", _k_upsampling_bilinear2d, (input,), {"size": list(size)})

    def opencl_upsampling_bilinear2d_grad(grad_out, input_sizes, size):
        return _k_upsampling_bilinear2d_grad(grad_out, input_sizes, list(size))

    for k, v in list(locals().items()):
        if k.startswith("opencl_"):
            setattr(ns, k, _traced(k, v))
    return ns


raw_ops = _mk_raw_ops()
"""One function per reference op, named as TF names the op library's ops."""


def _mk_fused_ops():
    ns = types.SimpleNamespace()

    def opencl_batch_norm_relu_training(x, gamma, beta, epsilon=1e-3, moving=None):
        """moving: optional (moving_mean, moving_var, momentum) updated in the
        statistics pass with the layer's EMA (same rounding as the layer)."""
        attrs = {"epsilon": float(epsilon)}
        if moving is not None:
            attrs["moving"] = moving
        return _apply("OpenclBatchNormReluTraining", _k_batch_norm_relu_training, (x, gamma, beta), attrs,
                      nondiff=(1, 2))

    def opencl_batch_norm_relu_grad(grad_z, x, gamma, beta, saved_mean, saved_var, epsilon=1e-3):
        return _k_batch_norm_relu_grad(grad_z, x, gamma, beta, saved_mean, saved_var, float(epsilon))

    def opencl_dense_relu(x, w, b):
        """relu(x @ W + b) with the ReLU in the GEMM's epilogue."""
        return _apply("OpenclDenseRelu", _k_dense_relu, (x, w, b), {})

    for k in ("opencl_batch_norm_relu_training", "opencl_batch_norm_relu_grad", "opencl_dense_relu"):
        setattr(ns, k, _traced(k, locals()[k]))
    return ns


fused_ops = _mk_fused_ops()
"""Ops with no counterpart in the reference: pairs its layers run back to back
(BatchNormTraining -> Relu, Dense -> Relu), fused, with bit-identical results."""


def _mk_step_ops():
    ns = types.SimpleNamespace()

    def opencl_mse_loss(y_pred, y_true):
        """Keras "mse" of one batch as a device scalar (differentiable in
        y_pred and y_true)."""
        return _apply("OpenclMseLoss", _k_mse_loss, (y_pred, y_true), {})

    def opencl_mse_loss_grad(y_pred, y_true, grad_loss):
        return _k_mse_loss_grad(y_pred, y_true, grad_loss)

    ns.opencl_mse_loss = _traced("opencl_mse_loss", opencl_mse_loss)
    ns.opencl_mse_loss_grad = _traced("opencl_mse_loss_grad", opencl_mse_loss_grad)
    return ns


step_ops = _mk_step_ops()
"""The training step's loss on the device: stock Keras in the reference
(``model.compile(loss="mse")``, README.md:188-196), not an op of its library."""


# ------------------------------------------------------- runtime utilities

def init(device: int = 0) -> None:
    """Select and check a device (``b2_init``); optional, ops init lazily."""
    _check(_lib.b2_init(int(device)))


def pool_stats() -> dict:
    s = PoolStats()
    _check(_lib.b2_pool_stats(ctypes.byref(s)))
    return {f: int(getattr(s, f)) for f, _ in PoolStats._fields_}


def pool_trim() -> None:
    _check(_lib.b2_pool_trim())


def kernel_launch_count() -> int:
    """Kernels the library has enqueued so far (graph replays not included)."""
    c = ctypes.c_uint64(0)
    _check(_lib.b2_kernel_launch_count(ctypes.byref(c)))
    return int(c.value)


def device_timeouts() -> int:
    c = ctypes.c_uint(0)
    _check(_lib.b2_device_timeouts(ctypes.byref(c)))
    return int(c.value)


def stream_status(device=None) -> None:
    """Synchronises torch's current stream of ``device`` and raises
    :class:`opencl_tf.errors.DeadlineExceededError` if a bounded device-side
    wait of one of this library's kernels expired since the last check (the
    state is then cleared).  Until then every op call raises that error too."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        _check(_lib.b2_stream_status(torch.cuda.current_stream(dev).cuda_stream))


def set_reserved_sms(count: int) -> None:
    """Keep ``count`` SMs free of the library's persistent tensor-core kernels
    (for NCCL's kernels during data-parallel training); 0 uses every SM."""
    _check(_lib.b2_set_reserved_sms(int(count)))


def set_wait_limit_ns(limit_ns: int) -> None:
    """Limit of each bounded device-side wait for kernels launched from now on
    (0 restores the 10 s default); a test hook."""
    _check(_lib.b2_set_wait_limit_ns(int(limit_ns)))


def upsampling_coords(in_size: int, out_size: int, device=None):
    """(lo, hi, frac) device arrays of the upsampling source coordinates."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    lo = torch.empty(out_size, dtype=torch.int32, device=dev)
    hi = torch.empty(out_size, dtype=torch.int32, device=dev)
    frac = torch.empty(out_size, dtype=torch.float32, device=dev)
    with _on_device(lo):
        _check(_lib.b2_upsampling_coords(_stream(lo), int(in_size), int(out_size), _p(lo), _p(hi), _p(frac)))
    return lo, hi, frac
