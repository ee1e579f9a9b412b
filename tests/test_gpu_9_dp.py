"""Data parallelism on 2 GPUs (skipped with fewer): one process per GPU over
NCCL, each rank trains the README network on its own batch shard; the
gradient all-reduce must leave every rank with the mean of the ranks'
gradients and identical weights after CUDA-graph-captured steps."""
from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    try:
        sys.path[:0] = [str(ROOT / "opencl-tensorflow_b200"), str(ROOT)]
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import torch.distributed as dist
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        from opencl_tf.model import build_model
        from opencl_tf.train import GradientAverager, TrainStep, mse
        dev = torch.device("cuda", rank)
        torch.manual_seed(0)
        model = build_model(device=dev)
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        x = torch.rand(16, 64, 64, 3, device=dev, generator=g)
        t = torch.rand(16, 8, 8, 8, device=dev, generator=g)
        # 1) the averaged gradient is the mean of the per-rank gradients
        mse(model(x, training=True), t).backward()
        mine = [p.grad.clone() for p in model.parameters()]
        GradientAverager(model.parameters())()
        gathered = [[torch.empty_like(m) for _ in range(world)] for m in mine]
        for m, slot in zip(mine, gathered):
            dist.all_gather(slot, m)
        err = max(float((p.grad - torch.stack(s).mean(0)).abs().max()) for p, s in zip(model.parameters(), gathered))
        model.zero_grad(set_to_none=True)
        # 1b) the overlapped path (bucket all-reduces launched from gradient
        # hooks during backward) gives the same averages
        avg = GradientAverager(model.parameters())
        assert avg.overlap and len(avg.buckets) >= 2
        avg.begin()
        mse(model(x, training=True), t).backward()
        avg()
        torch.cuda.synchronize()
        err = max(err, max(float((p.grad - torch.stack(s).mean(0)).abs().max())
                           for p, s in zip(model.parameters(), gathered)))
        model.zero_grad(set_to_none=True)
        # 2) graphed steps keep the replicas identical
        step = TrainStep(model, graphed=True, warmup=3)
        for _ in range(3):
            loss = step(x, t)
        torch.cuda.synchronize()
        flat = torch.cat([p.detach().reshape(-1) for p in model.parameters()])
        other = [torch.empty_like(flat) for _ in range(world)]
        dist.all_gather(other, flat)
        same = all(torch.equal(other[0], o) for o in other)
        step.release()
        # 3) the step's optimizer is split in two (Adam over the parameters
        # whose all-reduce is done runs beside the last bucket's all-reduce):
        # the parameters equal one Adam over all of them, bit for bit
        from opencl_tf.optimizers import Adam
        torch.manual_seed(0)
        m1 = build_model(device=dev)
        torch.manual_seed(0)
        m2 = build_model(device=dev)
        s1 = TrainStep(m1, graphed=False)
        assert len(s1.opts) == 2
        avg2 = GradientAverager(m2.parameters())
        opt2 = Adam(list(m2.parameters()))
        for _ in range(2):
            s1(x, t)
            opt2.zero_grad()
            l2 = mse(m2(x, training=True), t)
            avg2.begin()
            l2.backward()
            avg2()
            opt2.step()
        torch.cuda.synchronize()
        split_same = all(torch.equal(a, b) for a, b in zip(m1.parameters(), m2.parameters()))
        dist.destroy_process_group()
        q.put((rank, err, same and split_same, float(loss)))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e), False, 0.0))


def test_two_rank_gradient_averaging_and_replica_sync():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(120)
    for rank, err, same, loss in res:
        assert isinstance(err, float), (rank, err)
        assert err < 1e-6, (rank, err)
        assert same, rank
