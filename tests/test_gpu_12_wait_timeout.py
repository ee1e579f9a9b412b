"""A device-side wait that runs out is an op error, and the context survives it.

The reference maps every device failure to a TF status (OP_REQUIRES_CL ->
errors::Internal, src/ops/conv2d_ops.cc:43-45).  Here every spin-wait of the
tensor-core pipelines is bounded; the limit is a launch parameter that
``set_wait_limit_ns`` shortens.  With a 1 ns limit a real TMA-engine GEMM
(the Dense forward, K = 4096: 128 k-blocks per tile through the raw and
operand rings) cannot keep its waits short enough, so they expire: the CTAs
raise their abort flags, let their copies land, wait for their MMAs, free
TMEM and exit.  The expiry must come back as DeadlineExceededError
(B2_ERR_TIMEOUT) from ``stream_status`` and from the op calls made while it
is pending, and the very next call with the default limit must give the
same bits as before.  No GPU fault is involved: the wait simply gives up.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_expired_wait_is_reported_and_next_call_is_exact(otf):
    from opencl_tf import errors, raw_ops
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(1024, 4096, device="cuda", generator=g)
    w = torch.randn(4096, 128, device="cuda", generator=g)
    b = torch.randn(128, device="cuda", generator=g)
    good = raw_ops.opencl_dense(x, w, b)
    otf.stream_status()  # nothing pending
    before = otf.device_timeouts()

    expired = False
    try:
        otf.set_wait_limit_ns(1)
        for _ in range(5):  # each attempt is a full GEMM whose waits get 1 ns
            try:
                raw_ops.opencl_dense(x, w, b)
            except errors.DeadlineExceededError:
                pass  # an earlier attempt's expiry was already visible
            try:
                otf.stream_status()
            except errors.DeadlineExceededError:
                expired = True
                break
    finally:
        otf.set_wait_limit_ns(0)
    assert expired, "no wait expired with a 1 ns limit"
    assert otf.device_timeouts() > before

    otf.stream_status()  # the state was cleared by the report
    again = raw_ops.opencl_dense(x, w, b)
    otf.stream_status()
    assert torch.equal(again, good)


def test_pending_expiry_fails_the_next_op_call(otf):
    """While an expiry is pending (reported by no stream_status yet), op calls
    raise DeadlineExceededError after enqueueing their work."""
    from opencl_tf import errors, raw_ops
    x = torch.randn(512, 4096, device="cuda")
    w = torch.randn(4096, 96, device="cuda")
    b = torch.zeros(96, device="cuda")
    before = otf.device_timeouts()
    try:
        otf.set_wait_limit_ns(1)
        for _ in range(5):
            try:
                raw_ops.opencl_dense(x, w, b)
            except errors.DeadlineExceededError:
                pass
            torch.cuda.synchronize()
            if otf.device_timeouts() > before:
                break
    finally:
        otf.set_wait_limit_ns(0)
    torch.cuda.synchronize()
    with pytest.raises(errors.DeadlineExceededError):
        raw_ops.opencl_relu(x)
    with pytest.raises(errors.DeadlineExceededError):
        otf.stream_status()
    y = raw_ops.opencl_relu(x)  # cleared
    assert torch.equal(y, torch.where(x > 0, x, torch.zeros_like(x)))
