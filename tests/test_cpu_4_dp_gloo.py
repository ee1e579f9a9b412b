"""Data-parallel gradient averaging (opencl_tf.train.GradientAverager) across
two gloo ranks on CPU: every rank ends with the mean of all ranks'
gradients, and a rank that never joins makes the others fail on the host
with a timeout instead of hanging."""
from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    sys.path.insert(0, str(ROOT / "opencl-tensorflow_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    from opencl_tf.train import GradientAverager
    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Linear(5, 7), torch.nn.Linear(7, 3))
    torch.manual_seed(100 + rank)
    x = torch.randn(4, 5)
    model(x).pow(2).sum().backward()
    mine = [p.grad.clone() for p in model.parameters()]
    GradientAverager(model.parameters())()
    q.put((rank, [m.numpy() for m in mine], [p.grad.numpy() for p in model.parameters()]))
    dist.destroy_process_group()


def test_gradients_are_averaged_across_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (m, a)) for r, m, a in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    for i in range(4):
        want = (res[0][0][i] + res[1][0][i]) / 2
        assert abs(res[0][1][i] - want).max() < 1e-6
        assert abs(res[1][1][i] - want).max() < 1e-6


def _lonely(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
        t = torch.ones(3)
        dist.all_reduce(t)
        q.put("completed")
    except Exception as e:  # noqa: BLE001
        q.put(type(e).__name__)


def test_missing_rank_times_out_on_the_host():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(0, 2, _port(), q))
    p.start()
    out = q.get(timeout=120)
    p.join(30)
    assert out != "completed"


def test_bucket_plan_matches_backward_order():
    """The data-parallel step's buckets (opencl_tf/train.py: plan_buckets):
    reverse parameter order, closed at the size threshold, the first
    parameter alone in the last bucket.  The README model's parameter sizes
    give three buckets: the Dense weight (9.4 MB) with its bias before it,
    the other small parameters, and the stem filter."""
    import importlib
    sys.path.insert(0, str(ROOT / "opencl-tensorflow_b200"))
    train = importlib.import_module("opencl_tf.train")
    plan = train.plan_buckets
    assert plan([]) == []
    assert plan([100]) == [[0]]
    assert plan([100, 200]) == [[1], [0]]
    assert plan([8, 8, 8, 8], bucket_bytes=16) == [[3, 2], [1], [0]]
    assert plan([8, 8, 8, 8], bucket_bytes=8) == [[3], [2], [1], [0]]
    # the README network: stem kernel, BN gamma/beta, two blocks of
    # (dw kernel, BN, pw kernel, BN), Dense W and b -- float32 bytes
    sizes = [3 * 7 * 3 * 48, 48, 48,
             9 * 48, 48, 48, 48 * 96, 96, 96,
             9 * 96, 96, 96, 96 * 144, 144, 144,
             18432 * 128, 128]
    nbytes = [4 * n for n in sizes]
    b = plan(nbytes)
    assert b[0] == [16, 15]
    assert b[-1] == [0]
    assert b[1] == list(range(14, 0, -1))
    assert sorted(i for bucket in b for i in bucket) == list(range(len(sizes)))
