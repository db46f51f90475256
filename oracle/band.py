"""SAME-L differential band (sliding-window) attention, restated from the reference's XLA path — test infrastructure.

Follows `same_l._attention` (same_l.py:151-169) under `FP32_PARITY`, computed in float64:

* 5-way split, `b n (h d) -> b h n d` (same_l.py:162, 72-75)
* `_dyt`: `gamma * tanh(alpha * x) + beta` in fp32, one shared q norm and one shared k norm for both
  branches (same_l.py:58-69, 164-167)
* `_rope_tables` / `_rope`: fp32 angles `arange(L) * inv_freq`, half-half rotate (same_l.py:84-100)
* `_sdpa`: softmax over keys with `|k - q| <= window` and `0 <= k < L` (the grouped `_swa_mask` /
  `_windows` form, same_l.py:103-148, is the same function), weights times fp32 `v`
* `out = A - lambda * B` in fp32 (same_l.py:168; lambda = 1 is the reference).

and the front end of `same_l._attention` as `_block` calls it (`front_end`): the block's DyT pre-norm cast to
the compute dtype (same_l.py:191), then `_linear(x, to_qkv)` (same_l.py:52-55, 157) rounded to bf16.

Written as a direct band walked in query blocks, so any window and any L work (the grouped XLA form
needs `L % window == 0`).
"""
from __future__ import annotations

import numpy as np

from oracle.dense import HEAD_DIM, apply_rope, bf16, merge_heads, rope_cos_sin, split_heads


def dyt(x: np.ndarray, norm: dict) -> np.ndarray:
    """`DynamicTanh`: `gamma * tanh(alpha * x) + beta`, alpha a scalar (same_l.py:58-69)."""
    alpha = x.dtype.type(np.asarray(norm["alpha"], np.float32).reshape(-1)[0])
    return (np.asarray(norm["gamma"], x.dtype) * np.tanh(alpha * x) + np.asarray(norm["beta"], x.dtype))


def front_end(x: np.ndarray, to_qkv: np.ndarray, pre_norm: dict | None = None) -> np.ndarray:
    """`(B, L, d)` -> `(B, L, 5 H 64)` float64 holding bf16 values: `x' = bf16(dyt(x, pre_norm))` in fp32 when
    `pre_norm` is given (`_dyt(x, block["pre_norm"]).astype(dtype.compute)`, same_l.py:191), else x; then
    `bf16(x' @ to_qkv^T)` accumulated in float64 (`_linear`, same_l.py:52-55, 157, in the compute dtype)."""
    x = np.asarray(x, np.float32)
    if pre_norm is not None:
        x = bf16(dyt(x, pre_norm))
    y = np.matmul(x.astype(np.float64), np.asarray(to_qkv, np.float64).T)
    return bf16(y.astype(np.float32))


def band_attend(q: np.ndarray, k: np.ndarray, v: np.ndarray, window: int, block: int = 256,
                bf16_weights: bool = False) -> np.ndarray:
    """Band softmax attention `(B, H, L, 64)`: query i sees keys j with `|j - i| <= window`, `0 <= j < L`."""
    b, h, length, d = q.shape
    out = np.empty_like(q)
    scale = q.dtype.type(1.0 / np.sqrt(HEAD_DIM))
    for q0 in range(0, length, block):
        q1 = min(length, q0 + block)
        k0, k1 = max(0, q0 - window), min(length, q1 + window)
        logits = np.matmul(q[:, :, q0:q1], np.swapaxes(k[:, :, k0:k1], -1, -2)) * scale
        qi = np.arange(q0, q1)[:, None]
        kj = np.arange(k0, k1)[None, :]
        band = np.abs(kj - qi) <= window
        logits = np.where(band, logits, -np.inf)
        logits -= logits.max(-1, keepdims=True)
        w = np.exp(logits)
        if bf16_weights:  # the fused kernel's form (band_attention.py:96-101)
            out[:, :, q0:q1] = np.matmul(bf16(w), v[:, :, k0:k1]) / w.sum(-1, keepdims=True)
            continue
        w /= w.sum(-1, keepdims=True)
        out[:, :, q0:q1] = np.matmul(w, v[:, :, k0:k1])
    return out


def band_branches(qkv: np.ndarray, q_norm: dict, k_norm: dict, freqs: np.ndarray, num_heads: int,
                  window: int, offset: int = 0, fused_casts: bool = False,
                  dtype=np.float64) -> tuple[np.ndarray, np.ndarray]:
    """Branches A and B `(B, H, L, 64)`; `offset` is the sequence position of row 0 (for a slice).

    `fused_casts=True` adds the reference fused kernel's cast points (band_attention.py:82-85, 96-101):
    DyT + RoPE output -> bf16, bf16 softmax weights into `P @ V`, normalised after."""
    q, k, v, qd, kd = split_heads(qkv, num_heads, dtype=dtype)
    length = qkv.shape[1]
    cos, sin = rope_cos_sin(length, freqs, offset, dtype)
    cast = bf16 if fused_casts else (lambda t: t)
    q, qd = (cast(apply_rope(dyt(t, q_norm), cos, sin)) for t in (q, qd))
    k, kd = (cast(apply_rope(dyt(t, k_norm), cos, sin)) for t in (k, kd))
    return (band_attend(q, k, v, window, bf16_weights=fused_casts),
            band_attend(qd, kd, v, window, bf16_weights=fused_casts))


def band_diff_attention(qkv: np.ndarray, q_norm: dict, k_norm: dict, freqs: np.ndarray, num_heads: int,
                        window: int, lam: np.ndarray | None = None, offset: int = 0,
                        fused_casts: bool = False, dtype=np.float64) -> np.ndarray:
    """`(B, L, 5 * H * 64)` -> `(B, L, H * 64)` fp32: `A - lambda[pair] * B` per head (pair = head // 2)."""
    a, b = band_branches(qkv, q_norm, k_norm, freqs, num_heads, window, offset, fused_casts, dtype)
    lam_h = np.ones(num_heads, dtype) if lam is None else np.repeat(np.asarray(lam, dtype), 2)
    return merge_heads(a - lam_h[None, :, None, None] * b).astype(np.float32)
