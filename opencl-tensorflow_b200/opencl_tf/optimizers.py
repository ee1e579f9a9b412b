"""Keras Adam on the device: ``Adam(learning_rate=0.001, beta_1=0.9,
beta_2=0.999, epsilon=1e-7)``, the optimizer of the reference's training
recipe (``model.compile(optimizer=tf.keras.optimizers.Adam(1e-3), ...)``,
README.md:188-196), which runs as stock TensorFlow there.

One step is one multi-tensor kernel (``b2_adam_update``) over every parameter
with a gradient, with Keras's update rule and rounding of ``1 - beta``; the
step counter ``iterations`` lives on the device, so a step captured in a CUDA
graph replays correctly.  The moment slots ``m`` / ``v`` are kept per
parameter, zero-initialised like Keras's.
"""
from __future__ import annotations

from typing import Iterable

import torch

from . import _library, errors


class Adam:
    def __init__(self, params: Iterable[torch.Tensor], learning_rate: float = 0.001, beta_1: float = 0.9,
                 beta_2: float = 0.999, epsilon: float = 1e-7):
        self.params = [p for p in params if p.requires_grad]
        if not self.params:
            raise errors.InvalidArgumentError("Adam needs at least one trainable parameter")
        dev = self.params[0].device
        if dev.type != "cuda" or any(p.device != dev or p.dtype != torch.float32 or not p.is_contiguous()
                                     for p in self.params):
            raise errors.InvalidArgumentError("Adam parameters must be contiguous fp32 tensors on one CUDA device")
        self.learning_rate = float(learning_rate)
        self.beta_1 = float(beta_1)
        self.beta_2 = float(beta_2)
        self.epsilon = float(epsilon)
        self.m = [torch.zeros_like(p) for p in self.params]
        self.v = [torch.zeros_like(p) for p in self.params]
        self.iterations = torch.zeros((), dtype=torch.int64, device=dev)
        self._ticket = torch.zeros((), dtype=torch.int32, device=dev)

    @torch.no_grad()
    def step(self) -> None:
        """Applies every parameter's ``.grad`` (parameters without one are
        skipped, as Keras skips variables without a gradient)."""
        live = [i for i, p in enumerate(self.params) if p.grad is not None]
        for i in live:
            g = self.params[i].grad
            if not g.is_contiguous():
                self.params[i].grad = g.contiguous()
        _library.adam_update([self.params[i] for i in live], [self.params[i].grad for i in live],
                             [self.m[i] for i in live], [self.v[i] for i in live], self.learning_rate, self.beta_1,
                             self.beta_2, self.epsilon, self.iterations, self._ticket)

    def zero_grad(self, set_to_none: bool = True) -> None:
        for p in self.params:
            if p.grad is None:
                continue
            if set_to_none:
                p.grad = None
            else:
                p.grad.zero_()

    def get_config(self) -> dict:
        return {"name": "Adam", "learning_rate": self.learning_rate, "beta_1": self.beta_1, "beta_2": self.beta_2,
                "epsilon": self.epsilon}
