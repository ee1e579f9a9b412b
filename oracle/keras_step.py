"""TEST INFRASTRUCTURE (oracle). The training step's loss and optimizer as
Keras defines them, restated in numpy -- the oracle for the device loss and
Adam kernels, never called by the product path.

The reference trains with ``model.compile(optimizer=tf.keras.optimizers.Adam(
1e-3), loss="mse")`` (README.md:188-196).  Both live in TensorFlow, a
dependency that is not part of the reference checkout (TF 2.10-2.15, the range
the reference's op library builds against).  Restated from TF's published
algorithm:

* ``mean_squared_error``: ``mean(square(y_pred - y_true), axis=-1)`` then the
  mean over the batch (the default ``SUM_OVER_BATCH_SIZE`` reduction); with
  every row the same length that is one mean over all elements.
* ``Adam.update_step`` (keras/optimizers/adam.py, TF 2.11+; the legacy
  ``ApplyAdam`` kernel of TF 2.10 computes the same expressions), in float32::

      local_step = iterations + 1
      alpha = lr * sqrt(1 - beta_2 ** local_step) / (1 - beta_1 ** local_step)
      m += (g - m) * (1 - beta_1)
      v += (g * g - v) * (1 - beta_2)
      var -= (m * alpha) / (sqrt(v) + epsilon)

  ``1 - beta`` is Python double arithmetic rounded to float32 when it meets
  the float32 tensor.  Parity is pinned by the algebra above (there is no TF
  in this image to generate fixtures from): m and v must match bit for bit,
  the parameter within the tolerance that ``beta ** t`` (a library ``powf``
  on each side) leaves.
"""
from __future__ import annotations

import numpy as np


def mse_loss_f64(pred, target) -> float:
    d = np.asarray(pred, np.float64) - np.asarray(target, np.float64)
    return float(np.mean(d * d))


def mse_loss_grad_f64(pred, target, grad_loss: float = 1.0) -> np.ndarray:
    d = np.asarray(pred, np.float64) - np.asarray(target, np.float64)
    return 2.0 * grad_loss * d / d.size


def adam_update_f32(p, g, m, v, iterations: int, lr=1e-3, beta_1=0.9, beta_2=0.999, epsilon=1e-7):
    """One Keras Adam step in float32; returns (p, m, v) as new arrays."""
    f = np.float32
    p, g, m, v = (np.asarray(a, np.float32) for a in (p, g, m, v))
    t = f(iterations + 1)
    b1p = np.power(f(beta_1), t, dtype=np.float32)
    b2p = np.power(f(beta_2), t, dtype=np.float32)
    alpha = f(f(lr) * np.sqrt(f(1.0) - b2p, dtype=np.float32)) / f(f(1.0) - b1p)
    m = m + (g - m) * f(1.0 - beta_1)
    v = v + (g * g - v) * f(1.0 - beta_2)
    p = p - (m * f(alpha)) / (np.sqrt(v) + f(epsilon))
    return p.astype(np.float32), m.astype(np.float32), v.astype(np.float32)
