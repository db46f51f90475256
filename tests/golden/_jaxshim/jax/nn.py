"""`jax.nn.softmax` / `silu` with JAX's definitions: exp(x - max) / sum, computed in the input dtype."""
from __future__ import annotations

import numpy as _np


def softmax(x, axis=-1):
    unnormalized = _np.exp(x - _np.max(x, axis=axis, keepdims=True))
    return unnormalized / _np.sum(unnormalized.astype(_np.float64), axis=axis, keepdims=True).astype(x.dtype)


def sigmoid(x):
    return 1.0 / (1.0 + _np.exp(-x))


def silu(x):
    return x / (1.0 + _np.exp(-x))
