"""Weight initializers named like Keras's (``initializers.get("glorot_uniform")``).

Fan-in / fan-out follow the Keras convention for a kernel of shape
[..., in, out]: receptive field = product of the leading dims,
fan_in = in * rf, fan_out = out * rf.
"""
from __future__ import annotations

import math

import torch


def _fans(shape):
    if len(shape) == 1:
        return shape[0], shape[0]
    if len(shape) == 2:
        return shape[0], shape[1]
    rf = 1
    for d in shape[:-2]:
        rf *= d
    return shape[-2] * rf, shape[-1] * rf


def glorot_uniform(shape, generator=None):
    fi, fo = _fans(shape)
    lim = math.sqrt(6.0 / max(1, fi + fo))
    return torch.empty(shape, dtype=torch.float32).uniform_(-lim, lim, generator=generator)


def he_normal(shape, generator=None):
    fi, _ = _fans(shape)
    std = math.sqrt(2.0 / max(1, fi)) / 0.87962566103423978  # truncated at 2 sigma, as Keras does
    t = torch.empty(shape, dtype=torch.float32)
    torch.nn.init.trunc_normal_(t, 0.0, std, -2 * std, 2 * std, generator=generator)
    return t


def zeros(shape, generator=None):
    return torch.zeros(shape, dtype=torch.float32)


def ones(shape, generator=None):
    return torch.ones(shape, dtype=torch.float32)


_BY_NAME = {"glorot_uniform": glorot_uniform, "he_normal": he_normal, "zeros": zeros, "ones": ones}


def get(init):
    if callable(init):
        return init
    try:
        return _BY_NAME[str(init)]
    except KeyError:
        raise ValueError(f"unknown initializer {init!r}") from None


def serialize(init) -> str:
    for k, v in _BY_NAME.items():
        if v is init:
            return k
    return getattr(init, "__name__", repr(init))
