"""One training step of a model built from this package: forward, MSE loss,
backward through the registered gradients, data-parallel gradient averaging,
Adam -- what ``model.compile(Adam(1e-3), "mse"); model.fit(...)`` runs per
batch in the reference (README.md:188-196).  Loss and optimizer are this
package's device kernels with Keras's formulas (``step_ops.opencl_mse_loss``,
``optimizers.Adam``).

``TrainStep(model, graphed=True)`` captures the whole step in one CUDA graph
after a few eager warm-up steps, so a step costs one graph launch instead of
~50 Python-level op calls; inputs are copied into static device buffers.

Data parallelism: with an initialised ``torch.distributed`` process group
each rank runs the step on its own batch shard; the weight gradients are
averaged in buckets while backward runs (in-place NCCL all-reduces over
NVLink, the last small bucket over NVLink peer memory), and the optimizer
step is split around the last bucket (``GradientAverager``, ``TrainStep``).
BatchNorm statistics and moving averages stay per replica, as on one device
in the reference.
"""
from __future__ import annotations

import ctypes
import os
import socket

import torch
import torch.distributed as dist
from torch.distributed import distributed_c10d as c10d

from . import _library as _L
from ._library import set_reserved_sms, step_ops
from .optimizers import Adam


def mse(pred: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """Keras "mse" of the batch as a device scalar: one kernel forward, one
    backward (``step_ops.opencl_mse_loss``)."""
    return step_ops.opencl_mse_loss(pred, target)


def plan_buckets(nbytes, bucket_bytes: int = 4 << 20):
    """Gradient buckets for parameters of ``nbytes`` (in the model's order):
    lists of parameter indices, in the order backward produces the gradients
    (reverse), each closed once it holds ``bucket_bytes``; the first parameter
    (the first layer's weight, whose gradient comes last) gets a bucket of its
    own, so it does not hold back the exchange of the others."""
    buckets, cur, size = [], [], 0
    for i in reversed(range(len(nbytes))):
        cur.append(i)
        size += int(nbytes[i])
        if size >= bucket_bytes:
            buckets.append(cur)
            cur, size = [], 0
    if cur:
        buckets.append(cur)
    if buckets and len(buckets[-1]) > 1:
        buckets[-1], first = buckets[-1][:-1], buckets[-1][-1:]
        buckets.append(first)
    return buckets


class PeerExchange:
    """Averages an fp32 tensor of ``n`` elements in place across the ranks of
    ``group`` -- GPUs of one node, one process each -- over NVLink peer memory
    (``b2_peer_allreduce_avg``: one kernel per rank stores its copy into every
    rank's exchange block and adds the copies in rank order after every
    rank's flag, so all ranks get the same bits).  Setup is collective: every
    rank allocates its block, the CUDA IPC handles go through the process
    group, each rank maps the others' blocks.  ``PeerExchange.create`` returns
    None on every rank unless every rank could set it up."""

    def __init__(self, n: int, group, device):
        self.n = int(n)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.own = None
        self.opened = []
        size = _L._lib.b2_peer_exchange_bytes(self.n, self.world)
        if size == 0:
            raise RuntimeError("peer exchange: unsupported size or world")
        own, handle = ctypes.c_void_p(), (ctypes.c_ubyte * 64)()
        with torch.cuda.device(device):
            _L._check(_L._lib.b2_peer_buffer_create(size, ctypes.byref(own), handle))
        self.own = own.value
        self._handle = bytes(handle)
        self.device = device
        self.counters = torch.zeros(2, dtype=torch.int32, device=device)

    def _open(self, handles) -> None:
        bases = []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    bases.append(self.own)
                    continue
                p = ctypes.c_void_p()
                _L._check(_L._lib.b2_peer_buffer_open((ctypes.c_ubyte * 64).from_buffer_copy(h), ctypes.byref(p)))
                self.opened.append(p.value)
                bases.append(p.value)
        self.bases = (ctypes.c_void_p * self.world)(*bases)

    @classmethod
    def create(cls, n: int, group, device):
        world = dist.get_world_size(group)
        ex, err = None, ""
        try:
            ex = cls(n, group, device)
        except Exception as e:  # noqa: BLE001 -- agreed on below
            err = repr(e)
        info = [None] * world
        mine = (socket.gethostname(), ex._handle if ex is not None else None, err)
        dist.all_gather_object(info, mine, group=group)
        ok = all(h is not None for _, h, _ in info) and len({host for host, _, _ in info}) == 1 and world <= 8
        if ok:
            try:
                ex._open([h for _, h, _ in info])
            except Exception:  # noqa: BLE001
                ok = False
        flags = [None] * world
        dist.all_gather_object(flags, ok, group=group)
        if all(flags):
            return ex
        if ex is not None:
            ex.close()
        return None

    def __call__(self, t: torch.Tensor) -> None:
        """Average ``t`` (contiguous fp32, n elements) on the current stream."""
        _L._check(_L._lib.b2_peer_allreduce_avg(_L._stream(t), _L._p(t), self.n, self.rank, self.world, self.bases,
                                                _L._p(self.counters)))

    def close(self) -> None:
        with torch.cuda.device(self.device):
            for p in self.opened:
                _L._lib.b2_peer_buffer_close(p)
            if self.own is not None:
                _L._lib.b2_peer_buffer_free(self.own)
        self.opened, self.own = [], None


class GradientAverager:
    """Averages the gradients of ``params`` across the default process group
    (a no-op on a single process).

    On CUDA (NCCL) the gradients are averaged in place by coalesced all-reduces
    -- one NCCL group per bucket, no copies through a flat buffer.  With
    ``overlap`` (the default) the parameters are grouped into buckets of about
    ``bucket_bytes`` in reverse order (the order backward produces them) and a
    bucket's all-reduce is launched on a communication stream as soon as its
    last gradient is accumulated, so the exchange of the Dense layer's large
    weight gradient runs under the rest of the backward pass; ``begin()``
    before ``backward()`` arms it and calling the averager afterwards joins the
    communication stream back.  On CPU (gloo, which has no AVG) the gradients
    go through one flat buffer, summed and divided.
    """

    def __init__(self, params, group=None, overlap: bool = True, bucket_bytes: int = 4 << 20):
        self.params = [p for p in params if p.requires_grad]
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.flat = None
        self.armed = False
        self.overlap = bool(overlap) and self.world > 1 and bool(self.params) and self.params[0].is_cuda
        if self.overlap:
            plan = plan_buckets([p.numel() * p.element_size() for p in self.params], bucket_bytes)
            self.buckets = [[self.params[i] for i in b] for b in plan]
            self.bucket_of = {p: b for b, ps in enumerate(self.buckets) for p in ps}
            self.comm = torch.cuda.Stream(device=self.params[0].device)
            self.done = [torch.cuda.Event() for _ in self.buckets]
            # The last bucket (one small tensor, always exposed) goes over
            # NVLink peer memory instead of a latency-bound NCCL ring when all
            # ranks share a node (B2_PEER_EXCHANGE=0 turns this off).
            self.peer = None
            last = self.buckets[-1]
            if (len(last) == 1 and last[0].dtype == torch.float32 and last[0].numel() <= (1 << 22)
                    and os.environ.get("B2_PEER_EXCHANGE", "1") != "0"):
                self.peer = PeerExchange.create(last[0].numel(), group, last[0].device)
            for p in self.params:
                p.register_post_accumulate_grad_hook(self._grad_ready)
        # Called on the communication stream once every bucket but the last
        # has been launched (before the last one), e.g. the optimizer step of
        # the parameters whose gradients are then final; early_ran tells
        # whether it ran in the current backward pass.
        self.early_hook = None
        self.early_ran = False

    def begin(self) -> None:
        """Arm the overlapped reduction for the next backward pass."""
        if self.overlap:
            self.ready = [0] * len(self.buckets)
            self.launched = 0
            self.early_ran = False
            self.armed = True

    def _grad_ready(self, p) -> None:
        if not self.armed:
            return
        b = self.bucket_of[p]
        self.ready[b] += 1
        if self.ready[b] == len(self.buckets[b]):
            self._reduce_bucket(b)

    def _reduce_bucket(self, b) -> None:
        grads = [q.grad for q in self.buckets[b]]
        dev = grads[0].device
        self.comm.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(self.comm):
            if self.peer is not None and b == len(self.buckets) - 1:
                if not grads[0].is_contiguous():
                    raise RuntimeError("peer exchange needs a contiguous gradient")
                self.peer(grads[0])
            else:
                with c10d._coalescing_manager(self.group, dev):
                    for g in grads:
                        dist.all_reduce(g, op=dist.ReduceOp.AVG, group=self.group)
            self.done[b].record(self.comm)
            self.launched += 1
            last = len(self.buckets) - 1
            if (self.early_hook is not None and self.launched == last and b != last
                    and self.ready[last] < len(self.buckets[last])):
                self.early_hook()
                self.early_ran = True

    def close(self) -> None:
        """Unmap and free the peer-exchange blocks (after the last step, before
        the process group goes)."""
        if getattr(self, "peer", None) is not None:
            torch.cuda.synchronize(self.peer.device)
            self.peer.close()
            self.peer = None

    def wait_buckets(self, buckets) -> None:
        """Make the current stream wait for the all-reduces of ``buckets``
        (indices into ``self.buckets``) of the armed backward pass only, so
        work on their parameters can start while later buckets are still in
        flight.  Calling the averager afterwards still joins every bucket."""
        if not self.armed:
            return
        if self.launched != len(self.buckets):
            raise RuntimeError("a parameter has no gradient; every rank must produce every gradient")
        cur = torch.cuda.current_stream(self.params[0].device)
        for b in buckets:
            cur.wait_event(self.done[b])

    def __call__(self) -> None:
        if self.world == 1:
            return
        if self.armed:
            self.armed = False
            if self.launched != len(self.buckets):
                raise RuntimeError("a parameter has no gradient; every rank must produce every gradient")
            torch.cuda.current_stream(self.params[0].device).wait_stream(self.comm)
            return
        grads = [p.grad for p in self.params]
        if any(g is None for g in grads):
            raise RuntimeError("a parameter has no gradient; every rank must produce every gradient")
        if grads[0].is_cuda:
            with c10d._coalescing_manager(self.group, grads[0].device):
                for g in grads:
                    dist.all_reduce(g, op=dist.ReduceOp.AVG, group=self.group)
            return
        total = sum(g.numel() for g in grads)
        if self.flat is None or self.flat.numel() != total or self.flat.device != grads[0].device:
            self.flat = torch.empty(total, dtype=grads[0].dtype, device=grads[0].device)
        off = 0
        for g in grads:
            n = g.numel()
            self.flat[off:off + n].copy_(g.reshape(-1))
            off += n
        dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=self.group)
        self.flat.div_(self.world)
        off = 0
        for g in grads:
            n = g.numel()
            g.copy_(self.flat[off:off + n].view_as(g))
            off += n


class TrainStep:
    """fwd + MSE + bwd + gradient averaging + Adam for ``model`` on (x, y).

    ``reserved_sms``: with more than one rank, SMs kept free of the library's
    persistent tensor-core kernels so that NCCL's all-reduce kernels (and the
    early optimizer step) run beside the backward pass's last kernel, the
    stem filter gradient, instead of waiting for it (default: the
    ``B2_RESERVED_SMS`` environment variable, else 4).  The gradient buckets
    are about ``B2_BUCKET_BYTES`` (default 4 MiB) each."""

    def __init__(self, model: torch.nn.Module, lr: float = 1e-3, graphed: bool = True, warmup: int = 3,
                 group=None, reserved_sms: int | None = None):
        self.model = model
        self.params = [p for p in model.parameters() if p.requires_grad]
        dev = self.params[0].device
        bucket = int(os.environ.get("B2_BUCKET_BYTES", str(4 << 20)))
        self.avg = GradientAverager(self.params, group, bucket_bytes=bucket)
        # With overlapped buckets the last bucket's all-reduce can only start
        # after the last gradient of backward (the first layer's weight); Adam
        # over every other parameter runs on the communication stream as soon
        # as their buckets are exchanged (beside the backward pass's last
        # kernels), Adam over the last bucket after it.  Two optimizers, each
        # with its own step counter (always equal), apply exactly Keras's
        # update to each parameter.
        if self.avg.overlap and len(self.avg.buckets) > 1:
            late = {id(p) for p in self.avg.buckets[-1]}
            self.opts = [Adam([p for p in self.params if id(p) not in late], learning_rate=lr),
                         Adam([p for p in self.params if id(p) in late], learning_rate=lr)]
            # on a stream of its own, right after the other buckets' exchange
            # (so the last bucket's all-reduce does not queue behind it)
            self.opt_stream = torch.cuda.Stream(device=dev)
            self.avg.early_hook = self._early_step
        else:
            self.opts = [Adam(self.params, learning_rate=lr)]
        if self.avg.world > 1 and dev.type == "cuda":
            if reserved_sms is None:
                reserved_sms = int(os.environ.get("B2_RESERVED_SMS", "4"))
            set_reserved_sms(reserved_sms)
        self.graphed = graphed and dev.type == "cuda"
        self.warmup = warmup
        self.graph = None
        self.static_x = self.static_y = self.static_loss = None
        self.graph1 = None
        self.static_x1 = self.static_y1 = self.static_loss1 = None

    def _early_step(self) -> None:
        # called with the communication stream current
        self.opt_stream.wait_stream(self.avg.comm)
        with torch.cuda.stream(self.opt_stream):
            self.opts[0].step()

    def zero_grad(self) -> None:
        for o in self.opts:
            o.zero_grad(set_to_none=True)

    def _eager(self, x, y):
        self.zero_grad()
        loss = mse(self.model(x, training=True), y)
        self.avg.begin()
        loss.backward()
        if len(self.opts) == 2:
            if not self.avg.early_ran:  # the last bucket was not the last to complete
                self.avg.wait_buckets(range(len(self.avg.buckets) - 1))
                self.opts[0].step()
            self.avg()
            if self.avg.early_ran:
                torch.cuda.current_stream(x.device).wait_stream(self.opt_stream)
            self.opts[1].step()
        else:
            self.avg()
            self.opts[0].step()
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
        self.zero_grad()
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

    def graph_inputs(self, slot: int):
        """The static input buffers (x, y) of captured graph ``slot`` (0 or 1).
        Graph 1 is the same step captured on a second pair of buffers, so an
        input pipeline can copy the next batch straight into the buffers of
        the graph that will run it while the other graph runs (no staging
        copy inside the step).  Graph 0 must have been captured (one call)."""
        if self.graph is None:
            raise RuntimeError("run the step once before asking for its graph inputs")
        if slot == 0:
            return self.static_x, self.static_y
        if self.graph1 is None:
            self.static_x1 = torch.empty_like(self.static_x)
            self.static_y1 = torch.empty_like(self.static_y)
            self.static_x1.copy_(self.static_x)
            self.static_y1.copy_(self.static_y)
            torch.cuda.current_stream(self.static_x.device).synchronize()
            self.graph1 = torch.cuda.CUDAGraph()
            self.zero_grad()
            with torch.cuda.graph(self.graph1):
                self.static_loss1 = self._eager(self.static_x1, self.static_y1)
        return self.static_x1, self.static_y1

    def replay(self, slot: int) -> torch.Tensor:
        """One step on graph ``slot``'s input buffers; returns its loss (a
        device scalar)."""
        if slot == 0:
            self.graph.replay()
            return self.static_loss
        self.graph1.replay()
        return self.static_loss1

    def release(self) -> None:
        """Drop the captured graphs and the peer-exchange mappings (before
        destroying a process group)."""
        self.graph = None
        self.graph1 = None
        self.avg.close()
