"""One DiT transformer block, restated from the reference's XLA path — test infrastructure.

Follows `sa3jax.dit._block` (dit.py:224-250) under `FP32_PARITY`, computed in float64, in the reference's order:

* adaLN: `(to_scale_shift_gate + gcond)` split into scale / shift / gate for the self-attention and the MLP
  (dit.py:230-232);
* `x = RMSNorm(h, pre_norm) * (1 + scale_self) + shift_self` (dit.py:234-235; `_rms`, dit.py:45-57);
* self-attention `to_qkv -> differential attention -> to_out` (dit.py:185-200, via `oracle.dense`), then the
  gated residual `h + x * sigmoid(1 - gate_self)` — the `1 -` inside the sigmoid (dit.py:237);
* `h + cross_attention(RMSNorm(h, cross_attend_norm))` with the hoisted, k-normed keys (dit.py:239-240, 203-215,
  274-284; via `oracle.cross`);
* the `to_local_embed` constant added to the non-memory rows only (dit.py:242-244);
* `x = RMSNorm(h, ff_norm) * (1 + scale_ff) + shift_ff`, the GLU `value * silu(gate)` MLP (dit.py:218-221), then
  `h + x * sigmoid(1 - gate_ff)` (dit.py:246-250).

Nothing in the product imports this module.
"""
from __future__ import annotations

import numpy as np

from oracle.cross import cross_diff_attention
from oracle.dense import dense_diff_attention


def _rms(x: np.ndarray, weight: np.ndarray, eps: float) -> np.ndarray:
    """`dit._rms` over the model dim (a scale, not `1 + w`)."""
    x = np.asarray(x, np.float64)
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * np.asarray(weight, np.float64)


def _sigmoid(x: np.ndarray) -> np.ndarray:
    return 1.0 / (1.0 + np.exp(-x))


def dit_block(h: np.ndarray, p: dict, gcond: np.ndarray, kv: np.ndarray, freqs: np.ndarray, valid: np.ndarray, *,
              num_heads: int, memory: int, norm_eps: float = 1e-5, qk_eps: float = 1e-6) -> np.ndarray:
    """`(B, L, d)` -> `(B, L, d)` float64. `p` holds the block's weights (`[out, in]` as in the checkpoint):
    to_scale_shift_gate (6d), pre_norm / cross_attend_norm / ff_norm (d), sa_to_qkv (5d, d), sa_q_norm /
    sa_k_norm (64), sa_to_out (d, d), ca_to_q (2d, d), ca_q_norm (64), ca_to_out (d, d), local (d), glu_w (2F, d),
    glu_b (2F), proj_w (d, F), proj_b (d). `kv` is the hoisted cross K/V `(B, C, 3d)` = `[k | k_diff | v]` with
    k and k_diff already k-normed (`_cross_kv`). `valid` `(B, L)` is the value mask, `freqs` the RoPE
    frequencies."""
    f = lambda name: np.asarray(p[name], np.float64)  # noqa: E731
    h = np.asarray(h, np.float64)
    mods = (f("to_scale_shift_gate")[None, :] + np.asarray(gcond, np.float64))[:, None, :]
    ss, shs, gs, sf, shf, gf = np.split(mods, 6, axis=-1)
    x = _rms(h, p["pre_norm"], norm_eps) * (1 + ss) + shs
    qkv = x @ f("sa_to_qkv").T
    att = dense_diff_attention(qkv, p["sa_q_norm"], p["sa_k_norm"], freqs, valid, num_heads, qk_eps).astype(np.float64)
    h = h + (att @ f("sa_to_out").T) * _sigmoid(1 - gs)
    x = _rms(h, p["cross_attend_norm"], norm_eps)
    q2 = x @ f("ca_to_q").T
    cross = cross_diff_attention(q2, kv, p["ca_q_norm"], None, num_heads, qk_eps).astype(np.float64)
    h = h + cross @ f("ca_to_out").T
    h[:, memory:, :] += f("local")
    x = _rms(h, p["ff_norm"], norm_eps) * (1 + sf) + shf
    g = x @ f("glu_w").T + f("glu_b")
    value, gate = np.split(g, 2, axis=-1)
    y = (value * (gate * _sigmoid(gate))) @ f("proj_w").T + f("proj_b")
    return h + y * _sigmoid(1 - gf)
