"""The C ABI: the library loads without a GPU, exports every entry point
include/b2_opencl_tf.h declares, and its host-only helpers (padding and
output-shape resolution, argument validation) behave like the reference's
ResolvePadding and shape functions.  No device work is done here."""
from __future__ import annotations

import ctypes
import re
import threading
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "b2_opencl_tf.h"


def _declared():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b2_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    path = ROOT / "opencl-tensorflow_b200" / "opencl_tf" / "libb2ocl.so"
    if not path.exists():
        import subprocess
        import sys
        subprocess.run([sys.executable, str(ROOT / "opencl-tensorflow_b200" / "build.py")], check=True)
    return ctypes.CDLL(str(path))


def test_every_declared_symbol_is_exported(lib):
    names = _declared()
    assert len(names) >= 30, names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    ops = {"b2_conv2d", "b2_conv2d_backprop_input", "b2_conv2d_backprop_filter", "b2_depthwise_conv2d",
           "b2_depthwise_conv2d_backprop_input", "b2_depthwise_conv2d_backprop_filter", "b2_relu", "b2_relu_grad",
           "b2_sigmoid", "b2_sigmoid_grad", "b2_batch_norm_training", "b2_batch_norm_inference",
           "b2_batch_norm_grad", "b2_dense", "b2_dense_backprop_input", "b2_dense_backprop_weight",
           "b2_dense_backprop_bias", "b2_upsampling_bilinear2d", "b2_upsampling_bilinear2d_grad"}
    assert ops <= set(names), ops - set(names)  # one entry per REGISTER_OP


def test_abi_version(lib):
    lib.b2_abi_version.restype = ctypes.c_int
    assert lib.b2_abi_version() == 1


def test_resolve_padding_matches_reference_rule(lib):
    from oracle.oracle import resolve_padding
    f = lib.b2_resolve_padding
    f.argtypes = [ctypes.c_int64] * 3 + [ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64),
                                         ctypes.POINTER(ctypes.c_int64)]
    out, pad = ctypes.c_int64(), ctypes.c_int64()
    for n in (1, 2, 5, 9, 64, 65):
        for k in (1, 2, 3, 7):
            for s in (1, 2, 3):
                for mode in ("SAME", "VALID"):
                    assert f(n, k, s, mode.encode(), ctypes.byref(out), ctypes.byref(pad)) == 0
                    assert (out.value, pad.value) == resolve_padding(n, k, s, mode)
    assert f(5, 3, 1, b"FULL", ctypes.byref(out), ctypes.byref(pad)) == 1
    assert f(5, 3, 0, b"SAME", ctypes.byref(out), ctypes.byref(pad)) == 1


def _shape_fn(lib, name):
    f = getattr(lib, name)
    f.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int, ctypes.c_char_p, ctypes.c_void_p]
    f.restype = ctypes.c_int
    lib.b2_last_error.restype = ctypes.c_char_p

    def call(xs, ws, strides, padding):
        out = (ctypes.c_int64 * 4)()
        st = (ctypes.c_int32 * len(strides))(*strides)
        rc = f((ctypes.c_int64 * 4)(*xs), (ctypes.c_int64 * 4)(*ws), st, len(strides), padding.encode(), out)
        return rc, tuple(out), lib.b2_last_error().decode()

    return call


def test_conv2d_output_shape_and_errors(lib):
    call = _shape_fn(lib, "b2_conv2d_output_shape")
    assert call((256, 64, 64, 3), (3, 7, 3, 48), (1, 1, 2, 1), "SAME")[:2] == (0, (256, 64, 32, 48))
    assert call((2, 9, 9, 3), (3, 3, 3, 5), (1, 2, 2, 1), "VALID")[:2] == (0, (2, 4, 4, 5))
    rc, _, msg = call((2, 9, 9, 3), (3, 3, 3, 5), (1, 1, 1), "SAME")
    assert rc == 1 and "at least 4" in msg
    rc, _, msg = call((2, 9, 9, 3), (3, 3, 3, 5), (2, 1, 1, 1), "SAME")
    assert rc == 1 and "strides on N and C must be 1" in msg
    rc, _, msg = call((2, 9, 9, 3), (3, 3, 4, 5), (1, 1, 1, 1), "SAME")
    assert rc == 1 and "filter[2] must equal input channels" in msg
    rc, _, msg = call((2, 9, 9, 3), (3, 3, 3, 5), (1, 1, 1, 1), "same")
    assert rc == 1 and "padding" in msg


def test_depthwise_output_shape(lib):
    call = _shape_fn(lib, "b2_depthwise_conv2d_output_shape")
    assert call((256, 64, 32, 48), (3, 3, 48, 1), (1, 2, 2, 1), "SAME")[:2] == (0, (256, 32, 16, 48))
    assert call((2, 9, 9, 4), (3, 3, 4, 2), (1, 1, 1, 1), "VALID")[:2] == (0, (2, 7, 7, 8))


def test_last_error_is_per_thread(lib):
    call = _shape_fn(lib, "b2_conv2d_output_shape")
    rc, _, msg = call((2, 9, 9, 3), (3, 3, 3, 5), (2, 1, 1, 1), "SAME")
    assert rc == 1 and msg
    seen = []
    th = threading.Thread(target=lambda: seen.append(lib.b2_last_error()))
    th.start()
    th.join()
    assert seen == [b""]
