"""bf16 helpers and the tolerance check shared by the oracle's users (test infrastructure only)."""
from __future__ import annotations

import numpy as np

# Attention tolerances against the fp32 XLA-path oracle: max-abs 2e-2 / mean-abs 2e-3 on bf16 outputs.
ATTN_MAX_ABS = 2e-2
ATTN_MEAN_ABS = 2e-3


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bf16 (round-to-nearest-even), returned as uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 value, kept as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def check_close(out: np.ndarray, ref: np.ndarray, max_abs: float = ATTN_MAX_ABS,
                mean_abs: float = ATTN_MEAN_ABS) -> tuple[float, float]:
    """Assert |out - ref| max <= max_abs and mean <= mean_abs; return (max, mean)."""
    diff = np.abs(np.asarray(out, np.float64) - np.asarray(ref, np.float64))
    if not np.all(np.isfinite(diff)):
        raise AssertionError("non-finite values in the compared outputs")
    mx, mn = float(diff.max(initial=0.0)), float(diff.mean()) if diff.size else 0.0
    if mx > max_abs or mn > mean_abs:
        raise AssertionError(f"max-abs {mx:.3e} (tol {max_abs:.1e}), mean-abs {mn:.3e} (tol {mean_abs:.1e})")
    return mx, mn
