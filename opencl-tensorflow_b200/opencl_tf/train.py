"""One training step of a model built from this package: forward, MSE loss,
backward through the registered gradients, data-parallel gradient averaging,
Adam -- what ``model.compile(Adam(1e-3), "mse"); model.fit(...)`` runs per
batch in the reference (README.md:188-196).

``TrainStep(model, graphed=True)`` captures the whole step in one CUDA graph
after a few eager warm-up steps, so a step costs one graph launch instead of
~50 Python-level op calls; inputs are copied into static device buffers.

Data parallelism: with an initialised ``torch.distributed`` process group
each rank runs the step on its own batch shard; the weight gradients are
flattened into one bucket and averaged with a single all-reduce (NCCL over
NVLink on GPUs) before the optimizer step.  BatchNorm statistics and moving
averages stay per replica, as on one device in the reference.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def mse(pred: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    return torch.mean((pred - target) ** 2)


class GradientAverager:
    """Averages the gradients of ``params`` across the default process group
    with one bucketed all-reduce (a no-op on a single process)."""

    def __init__(self, params, group=None):
        self.params = [p for p in params if p.requires_grad]
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.flat = None

    def __call__(self) -> None:
        if self.world == 1:
            return
        grads = [p.grad for p in self.params]
        if any(g is None for g in grads):
            raise RuntimeError("a parameter has no gradient; every rank must produce every gradient")
        total = sum(g.numel() for g in grads)
        if self.flat is None or self.flat.numel() != total or self.flat.device != grads[0].device:
            self.flat = torch.empty(total, dtype=grads[0].dtype, device=grads[0].device)
        off = 0
        for g in grads:
            n = g.numel()
            self.flat[off:off + n].copy_(g.reshape(-1))
            off += n
        if self.flat.is_cuda:
            dist.all_reduce(self.flat, op=dist.ReduceOp.AVG, group=self.group)
        else:  # gloo has no AVG
            dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=self.group)
            self.flat.div_(self.world)
        off = 0
        for g in grads:
            n = g.numel()
            g.copy_(self.flat[off:off + n].view_as(g))
            off += n


class TrainStep:
    """fwd + MSE + bwd + gradient averaging + Adam for ``model`` on (x, y)."""

    def __init__(self, model: torch.nn.Module, lr: float = 1e-3, graphed: bool = True, warmup: int = 3,
                 group=None):
        self.model = model
        self.params = [p for p in model.parameters() if p.requires_grad]
        dev = self.params[0].device
        fused = dev.type == "cuda"
        self.opt = torch.optim.Adam(self.params, lr=lr, fused=fused, capturable=fused)
        self.avg = GradientAverager(self.params, group)
        self.graphed = graphed and dev.type == "cuda"
        self.warmup = warmup
        self.graph = None
        self.static_x = self.static_y = self.static_loss = None

    def _eager(self, x, y):
        self.opt.zero_grad(set_to_none=True)
        loss = mse(self.model(x, training=True), y)
        loss.backward()
        self.avg()
        self.opt.step()
        return loss.detach()

    def _capture(self, x, y):
        self.static_x = torch.empty_like(x)
        self.static_y = torch.empty_like(y)
        self.static_x.copy_(x)
        self.static_y.copy_(y)
        side = torch.cuda.Stream(device=x.device)
        side.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(side):
            for _ in range(self.warmup):
                self._eager(self.static_x, self.static_y)
        torch.cuda.current_stream(x.device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        self.opt.zero_grad(set_to_none=True)
        with torch.cuda.graph(self.graph):
            self.static_loss = self._eager(self.static_x, self.static_y)

    def __call__(self, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        """Runs one step; returns the loss as a device scalar (no host sync)."""
        if not self.graphed:
            return self._eager(x, y)
        if self.graph is None:
            self._capture(x, y)
        else:
            if x.data_ptr() != self.static_x.data_ptr():
                self.static_x.copy_(x, non_blocking=True)
            if y.data_ptr() != self.static_y.data_ptr():
                self.static_y.copy_(y, non_blocking=True)
        self.graph.replay()
        return self.static_loss

    def release(self) -> None:
        """Drop the captured graph (before destroying a process group)."""
        self.graph = None
