"""B200 drop-in for the DiT's differential cross-attention (`sa3jax.dit._cross_attention`, dit.py:203-215):
q RMSNorm -> `SDPA(q, k, v) - SDPA(q_diff, k_diff, v)` over the hoisted context keys, no RoPE, no mask
(`_attend` / `_attend_out`, dit.py:131-176), as one sm_100a kernel through the C ABI (`hb_cross_diff_attn`).

* `cross_kv(kv, k_weight, num_heads, eps)` -> the hoisted `to_kv` output with k and k_diff RMS-normed, as the
  reference's `_cross_kv` hoists them once per clip (dit.py:274-284);
* `cross_attention(q, kv, q_weight, k_weight, num_heads, head_dim, eps)` -> `(B, Lq, H * 64)`, the merged
  attention before `to_out`. `k_weight=None` when `kv` is already k-normed (the hoisted form).

`ValueError` on unsupported shapes (head_dim other than 64, more than 384 context tokens).
"""
from __future__ import annotations

import torch

from hummingbird_b200 import _lib
from hummingbird_b200._tensors import check_cuda, ptr, stream_handle

MAX_CONTEXT = 384


def cross_kv(kv: torch.Tensor, k_weight: torch.Tensor, num_heads: int, eps: float, head_dim: int = 64) -> torch.Tensor:
    """`(B, Lkv, 3 * H * 64)` `to_kv` output -> the same layout with k and k_diff RMS-normed in fp32 and rounded
    to bf16, v as is (dit.py:122-128, 274-284). Once per clip, so plain torch ops."""
    if kv.dim() != 3 or kv.shape[-1] != 3 * num_heads * head_dim:
        raise ValueError(f"kv must be (B, Lkv, 3 * H * 64), got {tuple(kv.shape)}")
    width = num_heads * head_dim
    keys = kv[..., :2 * width].float().unflatten(-1, (2 * num_heads, head_dim))
    keys = keys * torch.rsqrt(keys.pow(2).mean(-1, keepdim=True) + eps) * k_weight.float()
    return torch.cat([keys.flatten(-2).to(torch.bfloat16), kv[..., 2 * width:].to(torch.bfloat16)], -1).contiguous()


def cross_attention(q: torch.Tensor, kv: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor | None,
                    num_heads: int, head_dim: int = 64, eps: float = 1e-6, *, lam: torch.Tensor | None = None,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """`(B, Lq, 2 * H * 64)` `to_q` output and `(B, Lkv, 3 * H * 64)` `to_kv` output -> `(B, Lq, H * 64)`."""
    if head_dim != 64:
        raise ValueError(f"cross_attention needs head_dim 64 (head_dim={head_dim})")
    width = num_heads * head_dim
    if q.dim() != 3 or q.dtype != torch.bfloat16 or q.shape[-1] != 2 * width:
        raise ValueError(f"q must be bf16 (B, Lq, 2 * H * 64), got {tuple(q.shape)} {q.dtype}")
    if kv.dim() != 3 or kv.dtype != torch.bfloat16 or kv.shape[-1] != 3 * width or kv.shape[0] != q.shape[0]:
        raise ValueError(f"kv must be bf16 (B, Lkv, 3 * H * 64), got {tuple(kv.shape)} {kv.dtype}")
    batch, q_len, _ = q.shape
    kv_len = kv.shape[1]
    if not 1 <= kv_len <= MAX_CONTEXT:
        raise ValueError(f"cross_attention takes 1..{MAX_CONTEXT} context tokens, got {kv_len}")
    check_cuda(q, kv, q_weight)
    q = q if q.stride(-1) == 1 and q.stride(0) == q.stride(1) * q_len and q.stride(1) % 8 == 0 else q.contiguous()
    kv = kv if kv.stride(-1) == 1 and kv.stride(0) == kv.stride(1) * kv_len and kv.stride(1) % 8 == 0 \
        else kv.contiguous()
    q_weight = q_weight.to(torch.float32).contiguous()
    if k_weight is not None:
        k_weight = k_weight.to(device=q.device, dtype=torch.float32).contiguous()
    if lam is not None:
        lam = lam.to(device=q.device, dtype=torch.float32).contiguous()
    if out is None:
        out = torch.empty(batch, q_len, width, dtype=torch.bfloat16, device=q.device)
    _lib.call("hb_cross_diff_attn", ptr(q), q.stride(1), ptr(kv), kv.stride(1), ptr(q_weight), ptr(k_weight),
              ptr(lam), ptr(out), out.stride(1), batch, q_len, kv_len, num_heads, head_dim, float(eps),
              stream_handle(q.device))
    return out
