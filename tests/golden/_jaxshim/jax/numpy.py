"""`jax.numpy` for the golden generator: plain numpy, with contractions done in float64 and rounded back."""
from __future__ import annotations

import numpy as _np
from numpy import (  # noqa: F401
    abs, arange, broadcast_to, concatenate, cos, exp, float16, float32, inf, int32, linspace, max, mean, ones,
    pad, ravel, reshape, sin, size, split, sqrt, stack, swapaxes, tanh, tile, where, zeros, zeros_like,
)


class _NoBF16:
    """Placeholder: the generator runs the reference in fp32 only; bf16 compute is not emulated."""


bfloat16 = _NoBF16
dtype = _np.dtype


def einsum(spec, *operands):
    """fp32 in, fp32 out; accumulated in float64 so the oracle check is not limited by sum order."""
    out_type = _np.result_type(*operands)
    return _np.einsum(spec, *[o.astype(_np.float64) for o in operands]).astype(out_type)


class _At:
    """`x.at[index].add(v)`: a functional update returning a new array."""

    def __init__(self, arr, index=None):
        self._arr, self._index = arr, index

    def __getitem__(self, index):
        return _At(self._arr, index)

    def add(self, value):
        out = _np.array(self._arr, copy=True).view(type(self._arr))
        out[self._index] += value
        return out


class ArrayAt(_np.ndarray):
    """An ndarray with JAX's `.at[...]` update syntax (results of arithmetic on it keep the type)."""

    @property
    def at(self):
        return _At(self)


def array_at(x):
    """Wrap an array so the reference's `.at[...].add(...)` calls on values derived from it work."""
    return _np.asarray(x).view(ArrayAt)
