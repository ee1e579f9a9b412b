"""BatchNormalization ops (reference: opencl_tf/ops/batchnorm.py,
src/ops/batchnorm_ops.cc)."""
from __future__ import annotations

from .._library import raw_ops


def batch_norm_training(x, gamma, beta, epsilon: float = 1e-3):
    """Training-mode BN over NHWC channels.  Returns (y, saved_mean,
    saved_var); saved_var is the biased batch variance."""
    return raw_ops.opencl_batch_norm_training(x, gamma, beta, epsilon=epsilon)


def batch_norm_inference(x, gamma, beta, mean, var, epsilon: float = 1e-3):
    """Inference-mode BN with supplied statistics (no gradient)."""
    return raw_ops.opencl_batch_norm_inference(x, gamma, beta, mean, var, epsilon=epsilon)


def batch_norm_grad(grad_y, x, gamma, saved_mean, saved_var, epsilon: float = 1e-3):
    """Gradient of batch_norm_training: (grad_x, grad_gamma, grad_beta)."""
    return raw_ops.opencl_batch_norm_grad(grad_y, x, gamma, saved_mean, saved_var, epsilon=epsilon)
