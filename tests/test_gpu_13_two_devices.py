"""One process driving two GPUs (as TF's MirroredStrategy does): each kernel
that opts into more than 48 KB of shared memory must be set up on each device
it runs on.  A TMA-engine GEMM, the stem Conv2D (staged-row im2col) and the
staged depthwise filter gradient run on cuda:0, then on cuda:1, from one
thread and then from two threads at once; every result must equal cuda:0's
bit for bit (all three are deterministic).  Skipped with fewer than 2 GPUs."""
from __future__ import annotations

import threading

import pytest
import torch

pytestmark = pytest.mark.gpu


def _work(dev):
    g = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn(512, 2048, device=dev, generator=g)
    w = torch.randn(2048, 96, device=dev, generator=g)
    b = torch.zeros(96, device=dev)
    img = torch.rand(8, 64, 64, 3, device=dev, generator=g)
    k = torch.randn(3, 7, 3, 48, device=dev, generator=g) * 0.1
    a = torch.rand(8, 64, 32, 48, device=dev, generator=g)
    dy = torch.randn(8, 32, 16, 48, device=dev, generator=g)
    return x, w, b, img, k, a, dy


def _run(otf, dev):
    from opencl_tf import raw_ops
    with torch.cuda.device(dev):
        x, w, b, img, k, a, dy = _work(dev)
        outs = [raw_ops.opencl_dense(x, w, b),
                otf.conv2d(img, k, strides=(1, 1, 2, 1), padding="SAME"),
                otf.depthwise_conv2d_backprop_filter(a, [3, 3, 48, 1], dy, strides=(1, 2, 2, 1), padding="SAME")]
        otf.stream_status(dev)
        return [o.cpu() for o in outs]


def test_ops_on_two_devices_from_one_process(otf):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    d0, d1 = torch.device("cuda", 0), torch.device("cuda", 1)
    first = _run(otf, d0)
    second = _run(otf, d1)
    for a, b in zip(first, second):
        assert torch.equal(a, b)
    # and concurrently, one host thread per device
    res, errs = {}, []

    def go(dev):
        try:
            res[dev.index] = _run(otf, dev)
        except Exception as e:  # noqa: BLE001
            errs.append(repr(e))

    ts = [threading.Thread(target=go, args=(d,)) for d in (d0, d1)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(300)
    assert not errs, errs
    for a, b in zip(res[0], res[1]):
        assert torch.equal(a, b)
