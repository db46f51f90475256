"""Differential cross-attention of the DiT, restated from the reference's XLA path — test infrastructure.

Follows `sa3jax.dit._cross_attention` (dit.py:203-215) under `FP32_PARITY` (computed here in float64):

* `to_q` output split into q, q_diff and `b n (h d) -> b h n d` (dit.py:207-209, 101-104);
* the hoisted keys: `to_kv` output split into k, k_diff, v, k and k_diff RMS-normed with the k weight
  (`_cross_kv`, dit.py:274-284; `_k_norm`, dit.py:122-128), v never normed;
* `_attend` with no RoPE and no mask: q and q_diff RMS-normed with the q weight (dit.py:150-176);
* `_attend_out`: `SDPA(q, k, v) - SDPA(q_diff, k_diff, v)` at 1/sqrt(64) (dit.py:131-147), with the optional
  per-pair lambda the dense path takes (lambda = 1 reproduces the reference).

`fused_casts=True` adds the cast points of the fused kernels (normed q / k rounded to bf16, bf16 softmax
weights into P @ V, normalised after), as `oracle.dense` does for the self-attention.
"""
from __future__ import annotations

import numpy as np

from oracle.dense import HEAD_DIM, bf16, merge_heads, rms_norm, softmax_attend, split_heads


def cross_branches(q2: np.ndarray, kv: np.ndarray, q_weight: np.ndarray, k_weight: np.ndarray | None,
                   num_heads: int, eps: float, fused_casts: bool = False) -> tuple[np.ndarray, np.ndarray]:
    """Branches A (q, k) and B (q_diff, k_diff) with the shared v, each `(B, H, Lq, 64)`. `k_weight=None`:
    `kv` already holds the k-normed keys."""
    q, qd = split_heads(q2, num_heads, sections=2)
    k, kd, v = split_heads(kv, num_heads, sections=3)
    cast = bf16 if fused_casts else (lambda t: t)
    q, qd = cast(rms_norm(q, q_weight, eps)), cast(rms_norm(qd, q_weight, eps))
    if k_weight is not None:
        k, kd = cast(rms_norm(k, k_weight, eps)), cast(rms_norm(kd, k_weight, eps))
    return softmax_attend(q, k, v, fused_casts), softmax_attend(qd, kd, v, fused_casts)


def cross_diff_attention(q2: np.ndarray, kv: np.ndarray, q_weight: np.ndarray, k_weight: np.ndarray | None,
                         num_heads: int, eps: float = 1e-6, lam: np.ndarray | None = None,
                         fused_casts: bool = False) -> np.ndarray:
    """`(B, Lq, 2 * H * 64)` and `(B, Lkv, 3 * H * 64)` -> `(B, Lq, H * 64)` fp32: `A - lambda[h // 2] * B`."""
    assert q2.shape[-1] == 2 * num_heads * HEAD_DIM and kv.shape[-1] == 3 * num_heads * HEAD_DIM
    a, b = cross_branches(q2, kv, q_weight, k_weight, num_heads, eps, fused_casts)
    lam_h = np.ones(num_heads) if lam is None else np.repeat(np.asarray(lam, np.float64), 2)
    return merge_heads(a - lam_h[None, :, None, None] * b).astype(np.float32)
