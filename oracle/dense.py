"""Dense differential self-attention (DiT), restated from the reference's XLA path — test infrastructure.

Follows, cast point for cast point under `FP32_PARITY` (everything fp32; computed here in float64 and
rounded once at the end):

* split of `to_qkv` into `[q | k | v | q_diff | k_diff]` and `b n (h d) -> b h n d` (dit.py:196-198, 101-104)
* `_rms`: `x * rsqrt(mean(x^2) + eps) * w` over each head's 64 dims (dit.py:45-57), for q, k, q_diff, k_diff
* `_rope_tables`: angles `fp32(arange(L)) * fp32(inv_freq)` in fp32, `cat(freqs, freqs)` (dit.py:82-87)
* `_rope`: half-half rotate on the first `2 * half` dims (dit.py:90-98)
* `v * mask` (dit.py:174-175); no key mask: the softmax sees every key (dit.py:113-116)
* `_sdpa`: `softmax(q k^T / sqrt(64)) v` (dit.py:113-119); `out = A - lambda * B` (dit.py:144-146 with
  the per-pair lambda the benchmark configs add; lambda = 1 reproduces the reference).
"""
from __future__ import annotations

import numpy as np

HEAD_DIM = 64


def inv_freq(half: int, base: float = 10000.0) -> np.ndarray:
    """`RotaryEmbedding` frequencies for a `2 * half`-dim rotary: `base ** (-2i / (2 half))`, fp32."""
    rot_dim = 2 * half
    return (1.0 / (base ** (np.arange(0, rot_dim, 2, dtype=np.float64) / rot_dim))).astype(np.float32)


def rope_angles(length: int, freqs: np.ndarray, offset: int = 0) -> np.ndarray:
    """`fp32(arange) * fp32(inv_freq)` as the reference computes it (dit.py:85, same_l.py:87): `(L, half)` fp32."""
    pos = np.arange(offset, offset + length, dtype=np.float32)
    return pos[:, None] * np.asarray(freqs, np.float32)[None, :]


def rope_cos_sin(length: int, freqs: np.ndarray, offset: int = 0,
                 dtype=np.float64) -> tuple[np.ndarray, np.ndarray]:
    """`(L, 2 * half)` cos / sin of the fp32 angles (`cat(freqs, freqs)`), evaluated in float64."""
    ang = rope_angles(length, freqs, offset).astype(np.float64)
    ang = np.concatenate([ang, ang], axis=-1)
    return np.cos(ang).astype(dtype), np.sin(ang).astype(dtype)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Half-half `rotate_half` on the first `rot_dim` dims (dit.py:90-98). x `(..., L, 64)`, cos/sin `(L, rot_dim)`."""
    rot_dim = cos.shape[-1]
    rot, rest = x[..., :rot_dim], x[..., rot_dim:]
    rotated = np.concatenate([-rot[..., rot_dim // 2:], rot[..., :rot_dim // 2]], axis=-1)
    return np.concatenate([rot * cos + rotated * sin, rest], axis=-1)


def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float) -> np.ndarray:
    """`dit._rms` over the last (head) dim."""
    ms = np.mean(x * x, axis=-1, keepdims=True)
    return x / np.sqrt(ms + eps) * np.asarray(weight, np.float64)


def split_heads(qkv: np.ndarray, num_heads: int, sections: int = 5, dtype=np.float64) -> list[np.ndarray]:
    """`(B, L, sections * H * 64)` -> `sections` arrays `(B, H, L, 64)` (float64 unless `dtype` says otherwise:
    the timed CPU baseline runs in float32, the precision of the reference's FP32 XLA path)."""
    b, length, _ = qkv.shape
    parts = np.split(np.asarray(qkv, dtype), sections, axis=-1)
    return [p.reshape(b, length, num_heads, HEAD_DIM).transpose(0, 2, 1, 3) for p in parts]


def merge_heads(x: np.ndarray) -> np.ndarray:
    b, h, length, d = x.shape
    return x.transpose(0, 2, 1, 3).reshape(b, length, h * d)


def bf16(x: np.ndarray) -> np.ndarray:
    """Round to the nearest bf16 value (ties to even), kept in float64."""
    from oracle.common import bf16_round
    return bf16_round(np.asarray(x, np.float32)).astype(np.float64)


def softmax_attend(q: np.ndarray, k: np.ndarray, v: np.ndarray, bf16_weights: bool = False) -> np.ndarray:
    """`_sdpa`: unmasked softmax attention at 1/sqrt(64), per (b, h). With `bf16_weights`, the fused
    kernel's form: `bf16(exp(S - max)) @ v / sum(exp(S - max))` (dense_attention.py:79-83)."""
    logits = np.matmul(q, np.swapaxes(k, -1, -2)) * (1.0 / np.sqrt(HEAD_DIM))
    logits -= logits.max(-1, keepdims=True)
    w = np.exp(logits)
    if bf16_weights:
        return np.matmul(bf16(w), v) / w.sum(-1, keepdims=True)
    w /= w.sum(-1, keepdims=True)
    return np.matmul(w, v)


def dense_branches(qkv: np.ndarray, q_weight: np.ndarray, k_weight: np.ndarray, freqs: np.ndarray,
                   valid: np.ndarray, num_heads: int, eps: float,
                   fused_casts: bool = False, queries=None) -> tuple[np.ndarray, np.ndarray]:
    """The two softmax branches A (q, k) and B (q_diff, k_diff) with the shared masked v, `(B, H, L, 64)`
    (or `(B, H, len(queries), 64)` for the query rows `queries` only; every key is still attended).

    `fused_casts=False` is the XLA path in fp32 (the parity target). `fused_casts=True` adds the cast points
    of the reference's fused kernel (dense_attention.py:61-83): RMSNorm output -> bf16, RoPE output -> bf16,
    bf16 softmax weights into `P @ V`, normalised after; used where bf16 operand rounding dominates."""
    q, k, v, qd, kd = split_heads(qkv, num_heads)
    length = qkv.shape[1]
    cos, sin = rope_cos_sin(length, freqs)
    cast = bf16 if fused_casts else (lambda t: t)
    q, k, qd, kd = (cast(apply_rope(cast(rms_norm(t, w, eps)), cos, sin))
                    for t, w in ((q, q_weight), (k, k_weight), (qd, q_weight), (kd, k_weight)))
    v = cast(v * np.asarray(valid, np.float64)[:, None, :, None])
    if queries is not None:
        q, qd = q[:, :, queries], qd[:, :, queries]
    return softmax_attend(q, k, v, fused_casts), softmax_attend(qd, kd, v, fused_casts)


def dense_diff_attention(qkv: np.ndarray, q_weight: np.ndarray, k_weight: np.ndarray, freqs: np.ndarray,
                         valid: np.ndarray, num_heads: int, eps: float = 1e-6,
                         lam: np.ndarray | None = None, fused_casts: bool = False, queries=None) -> np.ndarray:
    """`(B, L, 5 * H * 64)` -> `(B, L, H * 64)` fp32: `A - lambda[pair] * B` per head (pair = head // 2);
    with `queries`, only those rows: `(B, len(queries), H * 64)`."""
    a, b = dense_branches(qkv, q_weight, k_weight, freqs, valid, num_heads, eps, fused_casts, queries)
    lam_h = np.ones(num_heads) if lam is None else np.repeat(np.asarray(lam, np.float64), 2)
    return merge_heads(a - lam_h[None, :, None, None] * b).astype(np.float32)
