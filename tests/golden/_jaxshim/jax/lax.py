"""`jax.lax` pieces used on the reference's XLA path."""
from __future__ import annotations

import numpy as _np


def rsqrt(x):
    return (1.0 / _np.sqrt(x.astype(_np.float64))).astype(x.dtype)
