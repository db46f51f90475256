"""A numpy-backed stand-in for the small slice of JAX that the reference's XLA attention path uses.

JAX is not installed in this image and cannot be installed offline, so the golden-vector generator
(`tests/golden/make_golden.py`) imports the reference package with this module on `sys.path` in place
of `jax`. It implements only what `sa3jax.dit`, `sa3jax.same_l`, `sa3jax.band_attention`,
`sa3jax.dense_attention` and `sa3jax.dtypes` touch at import time and on their XLA code paths, and it
runs them in float32 (the reference's `FP32_PARITY` preset). `jnp.bfloat16` is a sentinel that fails
if anything tries to compute in it. This is test infrastructure only; nothing in the product imports it.
"""
from __future__ import annotations

import numpy as _np

from . import lax, nn  # noqa: F401
from . import numpy  # noqa: F401

Array = _np.ndarray


def jit(fun=None, **_kwargs):
    """`jax.jit` as the identity (also usable as `partial(jax.jit, static_argnums=...)`)."""
    if fun is None:
        return lambda f: f
    return fun


def default_backend() -> str:
    return "cpu"
