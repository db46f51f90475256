"""The reference's drop-in switches, mirrored with a `"cuda"` value that selects this library's kernels.

`sa3jax.config.DiTConfig.attention` is `"xla" | "fused"` (config.py:57) and `SameConfig.attention` is
`"xla" | "pallas"` (config.py:115); both fall back to XLA off TPU. Here `"cuda"` selects the sm_100a kernels,
and a new `DiTConfig.ff_quant = "w8a8"` selects the W8A8 MLP (the reference has no int8 role,
dtypes.py:23-37). Only the fields the hot paths read are mirrored; the shapes follow the reference's
properties (`head_dim`, `rope_dim`, `sub_chunk_size`).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Literal


@dataclass(frozen=True)
class DiTConfig:
    """Fields of `sa3jax.config.DiTConfig` (config.py:36-78) used by the self-attention and MLP call sites."""

    embed_dim: int = 1024
    num_heads: int = 16
    num_memory_tokens: int = 64
    differential: bool = True
    qk_norm_eps: float = 1e-6
    norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    fourier_dim: int = 256
    ff_mult: float = 4.0
    attention: Literal["xla", "fused", "cuda"] = "cuda"
    fused_min_tokens: int = 0  # the reference gates its TPU kernel at 800 tokens; the B200 kernel has no floor
    ff_quant: Literal["none", "w8a8"] = "none"
    # "w8a8": the self-attention's `to_qkv` as a W8A8 GEMM fed by the pre-norm kernel's per-token int8 output
    # (glue="cuda", one rank per batch group)
    qkv_quant: Literal["none", "w8a8"] = "none"
    # "w8a8": the self-attention's `to_out` as a W8A8 GEMM; its input (the attention output, written per head by
    # the attention kernel) is quantised per token by a separate quantiser pass (glue="cuda")
    out_quant: Literal["none", "w8a8"] = "none"
    full_head_rope: bool = False  # True: rotate all 64 dims (the benchmark configs); False: the reference's 32

    @property
    def head_dim(self) -> int:
        return self.embed_dim // self.num_heads

    @property
    def rope_dim(self) -> int:
        """`RotaryEmbedding(max(dim_heads // 2, 32))` (config.py:67-70), or the full head."""
        return self.head_dim if self.full_head_rope else max(self.head_dim // 2, 32)

    @property
    def ff_inner(self) -> int:
        return int(self.embed_dim * self.ff_mult)


@dataclass(frozen=True)
class SameConfig:
    """Fields of `sa3jax.config.SameConfig` (config.py:81-141) used by the SAME-L attention call site."""

    channels: int = 256
    c_mults: tuple[int, ...] = (6,)
    dim_heads: int = 64
    stride: int = 16
    attention: Literal["xla", "pallas", "cuda"] = "cuda"
    rope_half: int = 16  # `RotaryEmbedding(dim_heads // 2)`: rot_dim 32 -> half 16 (same_l.py:84-89)

    @property
    def dim(self) -> int:
        return self.channels * self.c_mults[0]

    @property
    def num_heads(self) -> int:
        return self.dim // self.dim_heads

    @property
    def sub_chunk_size(self) -> int:
        """The band half-width the reference passes as `window` (same_l.py:159-160): stride + 1."""
        return self.stride + 1
