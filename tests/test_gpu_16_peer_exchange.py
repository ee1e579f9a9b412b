"""The NVLink peer-memory gradient exchange (b2_peer_allreduce_avg) on one GPU.

Between GPUs it is covered by tests/test_gpu_9_dp.py (the data-parallel step
averages its last gradient bucket with it).  Here, without peers:

* world = 1: the whole protocol (store into the block, flag, wait, add)
  against itself; the data must come back unchanged, call after call (the
  epoch advances, the halves alternate);
* a rank that never arrives: a two-rank call whose second block is a local
  buffer nobody writes.  The bounded wait runs out (limit set to 2 ms): the
  call's data is left as it was, the expiry is reported as
  DeadlineExceededError by stream_status, and the next call of another op
  works.  No GPU fault is involved: the wait simply gives up.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _block(lib, n, world):
    size = lib.b2_peer_exchange_bytes(n, world)
    assert size > 0
    ptr, handle = ctypes.c_void_p(), (ctypes.c_ubyte * 64)()
    assert lib.b2_peer_buffer_create(size, ctypes.byref(ptr), handle) == 0
    return ptr.value


def test_single_rank_round_trips(otf):
    from opencl_tf import _library as L
    n = 3024
    blk = _block(L._lib, n, 1)
    try:
        bases = (ctypes.c_void_p * 1)(blk)
        counters = torch.zeros(2, dtype=torch.int32, device="cuda")
        x = torch.randn(n, device="cuda")
        want = x.clone()
        for i in range(5):
            L._check(L._lib.b2_peer_allreduce_avg(L._stream(x), L._p(x), n, 0, 1, bases, L._p(counters)))
        otf.stream_status()
        assert torch.equal(x, want)
        assert int(counters[0]) == 5 and int(counters[1]) == 0
    finally:
        torch.cuda.synchronize()
        L._lib.b2_peer_buffer_free(blk)


def test_missing_rank_is_a_deadline_error(otf):
    from opencl_tf import _library as L
    from opencl_tf import errors
    n = 5000  # two CTAs
    mine, other = _block(L._lib, n, 2), _block(L._lib, n, 2)
    try:
        bases = (ctypes.c_void_p * 2)(mine, other)  # "rank 1" never runs
        counters = torch.zeros(2, dtype=torch.int32, device="cuda")
        x = torch.randn(n, device="cuda")
        want = x.clone()
        before = otf.device_timeouts()
        try:
            otf.set_wait_limit_ns(2_000_000)
            try:
                L._check(L._lib.b2_peer_allreduce_avg(L._stream(x), L._p(x), n, 0, 2, bases, L._p(counters)))
            except errors.DeadlineExceededError:
                pass  # an expiry pending from before
            with pytest.raises(errors.DeadlineExceededError):
                otf.stream_status()
        finally:
            otf.set_wait_limit_ns(0)
        assert otf.device_timeouts() > before
        assert torch.equal(x, want)
        y = torch.randn(1024, device="cuda")
        from opencl_tf import raw_ops
        assert torch.equal(raw_ops.opencl_relu(y), torch.where(y > 0, y, torch.zeros_like(y)))
        otf.stream_status()
    finally:
        torch.cuda.synchronize()
        L._lib.b2_peer_buffer_free(mine)
        L._lib.b2_peer_buffer_free(other)
