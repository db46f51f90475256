"""The reference's call sites of the hot paths, restated in torch around this library's kernels.

* `dit_self_attention`  — `dit._self_attention` (dit.py:185-200): `to_qkv` -> fused differential attention
                          -> `to_out`, taken when `DiTConfig.attention == "cuda"`.
* `same_l_attention`    — `same_l._attention` (same_l.py:151-161) for `SameConfig.attention == "cuda"`.
* `dit_feed_forward`    — `dit._feed_forward` (dit.py:218-221): GLU `value * silu(gate)`, with both `_linear`s
                          as W8A8 when `DiTConfig.ff_quant == "w8a8"`.

Projections that are plain library GEMMs (`to_qkv`, `to_out`, bf16 `_linear`) run as torch bf16 matmuls
(cuBLAS); weights are stored `[out, in]` as in the checkpoint (dit.py:33-36). There is no XLA / CPU path:
any other `attention` value raises.
"""
from __future__ import annotations

import torch

from hummingbird_b200 import band_attention as _band
from hummingbird_b200 import dense_attention as _dense
from hummingbird_b200.config import DiTConfig, SameConfig
from hummingbird_b200.w8a8 import W8A8Linear


def _linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """`nn.Linear` with the checkpoint's `[out, in]` weight (dit.py:33-36)."""
    y = x @ weight.T
    return y if bias is None else y + bias


def _require_cuda(attention: str) -> None:
    if attention != "cuda":
        raise ValueError(f"attention={attention!r}: hummingbird_b200 implements only the 'cuda' path")


def dit_self_attention(h: torch.Tensor, attn: dict, static: dict, cfg: DiTConfig,
                       lam: torch.Tensor | None = None) -> torch.Tensor:
    """`attn` holds `to_qkv.weight (5 H D, d)`, `q_norm.weight`, `k_norm.weight (D,)`, `to_out.weight (d, H D)`;
    `static` holds the lane tables from `dense_attention.tables` (`lane_cos`, `lane_sin`, `lane_mask`)."""
    _require_cuda(cfg.attention)
    qkv = _linear(h, attn["to_qkv"]["weight"])
    out = _dense.dense_attention(qkv, attn["q_norm"]["weight"], attn["k_norm"]["weight"], static["lane_cos"],
                                 static["lane_sin"], static["lane_mask"], cfg.num_heads, cfg.head_dim,
                                 cfg.rope_dim // 2, cfg.qk_norm_eps, lam=lam)
    return _linear(out, attn["to_out"]["weight"])


def same_l_attention(x: torch.Tensor, block: dict, cfg: SameConfig, lam: torch.Tensor | None = None,
                     pre_norm: dict | None = None) -> torch.Tensor:
    """`same_l._attention` (same_l.py:151-161). `block["self_attn"]` holds `to_qkv`, `q_norm`/`k_norm` DyT dicts
    and `to_out`; `block["rope_inv_freq"]`. x is `_attention`'s input (`_block` has applied its DyT pre-norm)
    unless `pre_norm` (`block["pre_norm"]`) is given: x is then the block input and the pre-norm runs inside the
    front end (same_l.py:191).

    With d_model <= 512 and window <= 128 the projection runs as the one-GEMM front end (pre-norm, `to_qkv`,
    q/k DyT + RoPE) and the band kernel reads its prepared output; otherwise `to_qkv` is a bf16 matmul and the
    band kernel prepares q/k itself. `to_out` is a bf16 matmul."""
    _require_cuda(cfg.attention)
    attn = block["self_attn"]
    window = cfg.sub_chunk_size
    if _band.fused_front_end_ok(x.shape[-1], window):
        out = _band.same_l_attention_x(x, attn["to_qkv"]["weight"], attn["q_norm"], attn["k_norm"],
                                       block["rope_inv_freq"], cfg.num_heads, window, pre_norm=pre_norm, lam=lam)
    else:
        if pre_norm is not None:  # `_dyt(x, pre_norm).astype(compute)` in fp32
            f32 = torch.float32
            alpha = torch.as_tensor(pre_norm["alpha"], dtype=f32, device=x.device)
            gamma = torch.as_tensor(pre_norm["gamma"], dtype=f32, device=x.device)
            beta = torch.as_tensor(pre_norm["beta"], dtype=f32, device=x.device)
            x = (gamma * torch.tanh(alpha * x.to(f32)) + beta).to(x.dtype)
        qkv = _linear(x, attn["to_qkv"]["weight"])
        out = _band.band_attention(qkv, attn["q_norm"], attn["k_norm"], block["rope_inv_freq"], cfg.num_heads,
                                   cfg.dim_heads, window, lam=lam)
    return _linear(out, attn["to_out"]["weight"])


class DiTFeedForward:
    """`dit._feed_forward` with the GLU projections quantised once (W8A8) or kept bf16."""

    def __init__(self, ff: dict, cfg: DiTConfig):
        self.w8a8 = cfg.ff_quant == "w8a8"
        g, o = ff["glu_proj"], ff["proj_out"]
        if self.w8a8:
            self.glu = W8A8Linear(g["weight"], g.get("bias"))
            self.out = W8A8Linear(o["weight"], o.get("bias"))
        else:
            self.glu = lambda x: _linear(x, g["weight"], g.get("bias"))  # noqa: E731
            self.out = lambda x: _linear(x, o["weight"], o.get("bias"))  # noqa: E731

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        value, gate = self.glu(x).chunk(2, dim=-1)
        return self.out(value * torch.nn.functional.silu(gate))
