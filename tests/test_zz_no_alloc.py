"""b2_batch_norm_training_no_alloc -- the BatchNorm training forward for
callers that must not have device memory allocated during a call (a runtime
whose memory manager owns all of HBM, or a warm serving loop that cannot take
an allocation's synchronisation and latency).  It keeps its reduction scratch
in a fixed 256 KiB array of the library instead of the scratch pool.

Checked through the C ABI against b2_batch_norm_training (same outputs within
the fp32 tolerance of the other tests) on two calls in a row, which also
shows the shared array carries nothing wrong from one call into the next;
the pool's allocation counter must not move during these calls.  This file
is collected last and needs nothing from the other tests."""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from helpers import assert_close

pytestmark = pytest.mark.gpu

LIB = Path(__file__).resolve().parent.parent / "opencl-tensorflow_b200" / "opencl_tf" / "libb2ocl.so"
P, I64, F32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float


class _PoolStats(ctypes.Structure):
    _fields_ = [("bytes_in_use", ctypes.c_uint64), ("bytes_reserved", ctypes.c_uint64),
                ("peak_in_use", ctypes.c_uint64), ("num_allocs", ctypes.c_uint64)]


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = ctypes.CDLL(str(LIB))
    sig = [P, P, P, P, I64, P, I64, F32, P, P, P]
    for name in ("b2_batch_norm_training", "b2_batch_norm_training_no_alloc"):
        getattr(lib, name).argtypes = sig
        getattr(lib, name).restype = ctypes.c_int
    lib.b2_last_error.restype = ctypes.c_char_p
    lib.b2_pool_stats.argtypes = [ctypes.POINTER(_PoolStats)]
    return lib


def _run(lib, name, x, g, b, eps=1e-3):
    C = x.shape[3]
    y = torch.empty_like(x)
    mean = torch.empty(C, device=x.device)
    var = torch.empty(C, device=x.device)
    rc = getattr(lib, name)(torch.cuda.current_stream().cuda_stream, x.data_ptr(), (I64 * 4)(*x.shape),
                            g.data_ptr(), C, b.data_ptr(), C, eps, y.data_ptr(), mean.data_ptr(), var.data_ptr())
    assert rc == 0, lib.b2_last_error().decode()
    return y, mean, var


def _allocs(lib):
    s = _PoolStats()
    assert lib.b2_pool_stats(ctypes.byref(s)) == 0
    return s.num_allocs


# (256, 64, 32, 48) and (7, 5, 9, 6) keep the pooled entry point's row blocks;
# the others have so many channels that the row blocks are capped to fit the
# fixed array (C = 256: at most 127 blocks, 4096: 7, 16384: 1).
@pytest.mark.parametrize("shape", [(256, 64, 32, 48), (7, 5, 9, 6), (64, 32, 32, 256), (2, 8, 8, 4096),
                                   (1, 4, 4, 16384)])
def test_no_alloc_matches_pooled_entry_point_two_calls(lib, shape):
    torch.manual_seed(1)
    C = shape[3]
    inputs = [(torch.randn(*shape, device="cuda") * 2 + 0.5, torch.randn(C, device="cuda") + 1,
               torch.randn(C, device="cuda") * 0.1) for _ in range(2)]
    for x, g, b in inputs:  # the pooled entry point first (it may grow the pool)
        _run(lib, "b2_batch_norm_training", x, g, b)
    torch.cuda.synchronize()
    before = _allocs(lib)
    got = [_run(lib, "b2_batch_norm_training_no_alloc", x, g, b) for x, g, b in inputs]
    torch.cuda.synchronize()
    assert _allocs(lib) == before  # no scratch was taken from the pool
    for (x, g, b), outs in zip(inputs, got):
        want = _run(lib, "b2_batch_norm_training", x, g, b)
        for name, a, w in zip(("y", "mean", "var"), outs, want):
            assert_close(a.cpu().numpy(), w.cpu().numpy(), what=name)
        # and the statistics against float64: biased variance E[x^2] - mean^2
        xd = x.double().reshape(-1, C).cpu().numpy()
        m64 = xd.mean(axis=0)
        v64 = (xd * xd).mean(axis=0) - m64 * m64
        assert_close(outs[1].cpu().numpy(), m64, what="mean vs float64")
        assert_close(outs[2].cpu().numpy(), v64, what="var vs float64")


@pytest.mark.parametrize("shape", [(16, 32, 16, 48), (7, 5, 9, 6), (64, 32, 32, 256), (2, 8, 8, 4096),
                                   (1, 4, 4, 16384)])
def test_no_alloc_against_the_oracle(lib, port, shape):
    """y, saved_mean and saved_var against the reference's BatchNorm kernels
    (batchnorm_kernels.cl:35-80, in the oracle's bit-exact C restatement), at
    the contract tolerance: the sums run in another order than the
    reference's serial loop; y is then exact given the statistics."""
    rng = np.random.default_rng(5)
    C = shape[3]
    x = (rng.standard_normal(shape) * 2 + 0.5).astype(np.float32)
    g = (rng.standard_normal(C) + 1).astype(np.float32)
    b = (rng.standard_normal(C) * 0.1).astype(np.float32)
    y, mean, var = _run(lib, "b2_batch_norm_training_no_alloc", torch.from_numpy(x).cuda(),
                        torch.from_numpy(g).cuda(), torch.from_numpy(b).cuda())
    torch.cuda.synchronize()
    ry, rm, rv = port.batch_norm_training(x, g, b, 1e-3)
    assert_close(mean.cpu().numpy(), rm, what="mean vs oracle")
    assert_close(var.cpu().numpy(), rv, what="var vs oracle")
    assert_close(y.cpu().numpy(), ry, what="y vs oracle")


def test_no_alloc_rejects_too_many_channels(lib):
    x = torch.zeros(1, 1, 1, 16385, device="cuda")
    c = torch.zeros(16385, device="cuda")
    y = torch.empty_like(x)
    rc = lib.b2_batch_norm_training_no_alloc(torch.cuda.current_stream().cuda_stream, x.data_ptr(),
                                             (I64 * 4)(*x.shape), c.data_ptr(), 16385, c.data_ptr(), 16385, 1e-3,
                                             y.data_ptr(), c.data_ptr(), c.data_ptr())
    assert rc == 1
    assert b"at most 16384 channels" in lib.b2_last_error()
