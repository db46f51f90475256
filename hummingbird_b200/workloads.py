"""Seeded synthetic inputs for the benchmark configurations (no dataset or checkpoint is involved).

Draws use `numpy.random.default_rng(seed)` in a fixed order (x, then each weight section, then norm
parameters, then lambda); projections run on the device in fp32 and are rounded once to bf16, so the
kernel input `qkv = bf16(x @ W_qkv^T)` is shared bit for bit by the GPU path and the CPU oracle.

* dense (config 1): B=1, L=646, d=1024, 16 heads, full-head RoPE (half 32, base 1e4), RMSNorm scales
  1 + N(0, 0.02), eps 1e-6, the last 64 tokens' values masked, lambda ~ U(0.2, 0.8), seed 0.
* band (config 2): B=1, L=82,688, d=512, 8 heads, window 128, DyT alpha 0.5, gamma 1 + N(0, 0.02),
  beta N(0, 0.02), RoPE base 1e4 on the first 32 dims (half 16, the SAME-L reference's
  `RotaryEmbedding(dim_heads // 2)`, same_l.py:84-89), lambda ~ U(0.2, 0.8), seed 1.
* band layer (config 2 through the front end): the same shapes with x ~ N(0, 1) rounded to bf16 as the
  layer's input, to_qkv ~ N(0, 1/d) rounded to bf16, and the block's DyT pre-norm (alpha 0.5, gamma
  1 + N(0, 0.02), beta N(0, 0.02) over d), seed 11.
* w8a8 (config 3): M=2,584; x ~ N(0,1) bf16; W1 (4096, 1024) ~ N(0, 1/1024); W2 (1024, 4096) ~ N(0, 1/4096);
  biases N(0, 0.02); seed 3.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch


def inv_freq(half: int, base: float = 10000.0) -> np.ndarray:
    rot = 2 * half
    return (1.0 / (base ** (np.arange(0, rot, 2, dtype=np.float64) / rot))).astype(np.float32)


def _project(x: np.ndarray, w: np.ndarray, device) -> torch.Tensor:
    """bf16(x @ w^T) computed in fp32 on `device` (no TF32)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        xt = torch.from_numpy(np.asarray(x, np.float32)).to(device)
        wt = torch.from_numpy(np.asarray(w, np.float32)).to(device)
        return (xt @ wt.T).to(torch.bfloat16)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


@dataclass
class DenseInputs:
    qkv: torch.Tensor          # (B, L, 5 * H * 64) bf16
    q_weight: np.ndarray       # (64,)
    k_weight: np.ndarray
    inv_freq: np.ndarray       # (half,)
    valid: np.ndarray          # (B, L) float32 0/1
    lam: np.ndarray            # (H / 2,)
    heads: int
    half: int
    eps: float


def dense_inputs(device, *, seed=0, batch=1, length=646, d_model=1024, heads=16, half=32, masked_tail=64):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((batch * length, d_model), dtype=np.float32)
    w = np.concatenate([rng.standard_normal((heads * 64, d_model), dtype=np.float32) / np.sqrt(d_model)
                        for _ in range(5)])
    q_w = (1.0 + 0.02 * rng.standard_normal(64)).astype(np.float32)
    k_w = (1.0 + 0.02 * rng.standard_normal(64)).astype(np.float32)
    lam = rng.uniform(0.2, 0.8, heads // 2).astype(np.float32)
    qkv = _project(x, w, device).reshape(batch, length, 5 * heads * 64)
    valid = np.ones((batch, length), np.float32)
    if masked_tail:
        valid[:, length - masked_tail:] = 0.0
    return DenseInputs(qkv, q_w, k_w, inv_freq(half), valid, lam, heads, half, 1e-6)


@dataclass
class BandInputs:
    qkv: torch.Tensor          # (B, L, 5 * H * 64) bf16
    q_norm: dict
    k_norm: dict
    inv_freq: np.ndarray
    lam: np.ndarray
    heads: int
    window: int


def band_inputs(device, *, seed=1, batch=1, length=82_688, d_model=512, heads=8, half=16, window=128, x_seed=None):
    """`x_seed` (e.g. `(1, rank)`) draws other rows of the same sequence with the same weights."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((batch * length, d_model), dtype=np.float32)
    if x_seed is not None:
        x = np.random.default_rng(x_seed).standard_normal((batch * length, d_model), dtype=np.float32)
    w = np.concatenate([rng.standard_normal((heads * 64, d_model), dtype=np.float32) / np.sqrt(d_model)
                        for _ in range(5)])

    def norm():
        return {"alpha": np.float32(0.5), "gamma": (1.0 + 0.02 * rng.standard_normal(64)).astype(np.float32),
                "beta": (0.02 * rng.standard_normal(64)).astype(np.float32)}

    qn, kn = norm(), norm()
    lam = rng.uniform(0.2, 0.8, heads // 2).astype(np.float32)
    qkv = _project(x, w, device).reshape(batch, length, 5 * heads * 64)
    return BandInputs(qkv, qn, kn, inv_freq(half), lam, heads, window)


@dataclass
class BandLayerInputs:
    x: torch.Tensor            # (B, L, d) bf16: the block input before its DyT pre-norm
    to_qkv: torch.Tensor       # (5 H 64, d) bf16, the checkpoint's [out, in]
    to_out: torch.Tensor       # (H 64, H 64) bf16
    pre_norm: dict             # block DyT {"alpha", "gamma" (d,), "beta" (d,)}
    q_norm: dict
    k_norm: dict
    inv_freq: np.ndarray
    lam: np.ndarray
    heads: int
    window: int


def band_layer_inputs(device, *, seed=11, batch=1, length=82_688, d_model=512, heads=8, half=16, window=128,
                      x_seed=None):
    """The SAME-L attention layer's own inputs (x, the to_qkv / to_out weights) for the one-GEMM front end.
    `x_seed` (e.g. `(seed, rank)`) draws other rows of the same sequence with the same weights."""
    rng = np.random.default_rng(seed)
    bf = lambda a: torch.from_numpy(np.asarray(a, np.float32)).to(device).to(torch.bfloat16)  # noqa: E731
    x = rng.standard_normal((batch, length, d_model), dtype=np.float32)
    if x_seed is not None:
        x = np.random.default_rng(x_seed).standard_normal((batch, length, d_model), dtype=np.float32)
    x = bf(x)
    w = bf(np.concatenate([rng.standard_normal((heads * 64, d_model), dtype=np.float32) / np.sqrt(d_model)
                           for _ in range(5)]))
    pre = {"alpha": np.float32(0.5), "gamma": (1.0 + 0.02 * rng.standard_normal(d_model)).astype(np.float32),
           "beta": (0.02 * rng.standard_normal(d_model)).astype(np.float32)}

    def norm():
        return {"alpha": np.float32(0.5), "gamma": (1.0 + 0.02 * rng.standard_normal(64)).astype(np.float32),
                "beta": (0.02 * rng.standard_normal(64)).astype(np.float32)}

    qn, kn = norm(), norm()
    lam = rng.uniform(0.2, 0.8, heads // 2).astype(np.float32)
    to_out = bf(rng.standard_normal((heads * 64, heads * 64), dtype=np.float32) / np.sqrt(heads * 64))
    return BandLayerInputs(x, w, to_out, pre, qn, kn, inv_freq(half), lam, heads, window)


@dataclass
class W8A8Inputs:
    x: torch.Tensor    # (M, 1024) bf16
    w1: torch.Tensor   # (4096, 1024) bf16
    b1: torch.Tensor   # (4096,) bf16
    w2: torch.Tensor   # (1024, 4096) bf16
    b2: torch.Tensor   # (1024,) bf16


def w8a8_inputs(device, *, seed=3, m=2584, d_model=1024, inner=4096):
    rng = np.random.default_rng(seed)
    bf = lambda a: torch.from_numpy(np.asarray(a, np.float32)).to(device).to(torch.bfloat16)  # noqa: E731
    x = bf(rng.standard_normal((m, d_model), dtype=np.float32))
    w1 = bf(rng.standard_normal((inner, d_model), dtype=np.float32) / np.sqrt(d_model))
    w2 = bf(rng.standard_normal((d_model, inner), dtype=np.float32) / np.sqrt(inner))
    b1 = bf(0.02 * rng.standard_normal(inner))
    b2 = bf(0.02 * rng.standard_normal(d_model))
    return W8A8Inputs(x, w1, b1, w2, b2)
