"""Error types raised by the ops, mirroring the TF statuses the reference ops
return (``errors::InvalidArgument`` for shape/attr problems,
``errors::Internal`` for device failures; src/ops/conv2d_ops.cc:43-45)."""
from __future__ import annotations


class OpError(Exception):
    """Base class; ``.code`` is the C-ABI ``b2_status_t`` value."""

    code = 2


class InvalidArgumentError(OpError, ValueError):
    code = 1


class InternalError(OpError, RuntimeError):
    code = 2


class ResourceExhaustedError(OpError, MemoryError):
    code = 3


class UnavailableError(OpError, RuntimeError):
    code = 4


class DeadlineExceededError(OpError, RuntimeError):
    code = 5


_BY_CODE = {1: InvalidArgumentError, 2: InternalError, 3: ResourceExhaustedError,
            4: UnavailableError, 5: DeadlineExceededError}


def from_status(code: int, message: str) -> OpError:
    return _BY_CODE.get(int(code), InternalError)(message)
