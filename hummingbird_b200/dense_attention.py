"""B200 drop-in for `sa3jax.dense_attention` (dense_attention.py:97-153): the DiT's fused differential
self-attention, RMSNorm -> RoPE -> value mask -> two softmax branches -> subtract, on sm_100a.

Same entry points, argument meaning and errors as the reference:

* `tables(length, inv_freq, valid, head_dim, compute)` -> lane cos / signed-sin `(L, 128)` fp32 and lane
  V-mask `(B, L, 128)` (dense_attention.py:97-101, band_attention.py:43-58);
* `dense_attention(qkv, q_weight, k_weight, cos, sin, mask, num_heads, head_dim, half, eps)` ->
  `(B, L, H * 64)` (dense_attention.py:104-153); `ValueError` on unsupported shapes.

Tensors are torch CUDA tensors; the work runs on the current CUDA stream through the C ABI
(`hb_dense_diff_attn`). Additions over the reference: `lam` (per-pair lambda of `A - lambda * B`;
None = 1, the reference) and `pair_begin`/`pair_count` (head-pair sharding).
"""
from __future__ import annotations

import torch

from hummingbird_b200 import _lib
from hummingbird_b200._tensors import check_cuda, ptr, stream_handle, workspace

LANES = 128


def rope_tables(length: int, inv_freq: torch.Tensor, head_dim: int = 64, offset: int = 0):
    """`(length, 128)` fp32 cos and signed-sin lane tables for two 64-dim heads (band_attention.py:43-58):
    lane l -> dim d = l % 64 rotates with frequency d % half when d < 2 * half; angles are
    fp32(arange) * fp32(inv_freq), bit-identical to the reference's `_rope_tables`."""
    inv_freq = inv_freq.to(torch.float32)
    half = inv_freq.shape[0]
    dim = torch.arange(LANES, device=inv_freq.device) % head_dim
    rotary = dim < 2 * half
    freq = torch.where(rotary, inv_freq[dim % half], torch.zeros((), device=inv_freq.device))
    sign = torch.where(dim < half, -1.0, 1.0).to(inv_freq.device) * rotary
    angles = torch.arange(offset, offset + length, dtype=torch.float32, device=inv_freq.device)[:, None] * freq[None, :]
    return torch.cos(angles), torch.sin(angles) * sign


def tables(length: int, inv_freq: torch.Tensor, valid: torch.Tensor, head_dim: int = 64,
           compute: torch.dtype = torch.bfloat16):
    """Per-clip inputs (dense_attention.py:97-101): lane cos / signed-sin `(L, 128)` fp32 and the lane
    V-mask `(B, L, 128)` in the compute dtype."""
    cos, sin = rope_tables(length, inv_freq, head_dim)
    mask = valid.to(compute)[:, :, None].expand(*valid.shape, LANES)
    return cos, sin, mask


def workspace_bytes(batch: int, length: int, pair_count: int) -> int:
    import ctypes
    n = ctypes.c_size_t(0)
    _lib.call("hb_dense_workspace_bytes", batch, length, pair_count, ctypes.byref(n))
    return int(n.value)


def dense_attention(qkv: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor, cos: torch.Tensor,
                    sin: torch.Tensor, mask: torch.Tensor, num_heads: int, head_dim: int, half: int, eps: float, *,
                    lam: torch.Tensor | None = None, pair_begin: int = 0, pair_count: int | None = None,
                    out: torch.Tensor | None = None, ws: torch.Tensor | None = None) -> torch.Tensor:
    """`(B, L, 5 * H * D)` DiT `to_qkv` output -> `(B, L, 2 * pair_count * D)` differential self-attention."""
    if head_dim * 2 != LANES:
        raise ValueError(f"dense_attention needs head_dim 64 (head_dim={head_dim})")
    if qkv.dim() != 3 or qkv.dtype != torch.bfloat16 or qkv.shape[-1] != 5 * num_heads * head_dim:
        raise ValueError(f"qkv must be bf16 (B, L, 5 * H * 64), got {tuple(qkv.shape)} {qkv.dtype}")
    batch, length, _ = qkv.shape
    pairs = num_heads // 2
    pair_count = pairs - pair_begin if pair_count is None else pair_count
    check_cuda(qkv, q_weight, k_weight, cos, sin, mask)
    qkv = qkv if qkv.stride(-1) == 1 and qkv.stride(0) == qkv.stride(1) * length else qkv.contiguous()
    q_weight = q_weight.to(torch.float32).contiguous()
    k_weight = k_weight.to(torch.float32).contiguous()
    cos = cos.to(torch.float32)
    sin = sin.to(torch.float32)
    if cos.stride(-1) != 1 or sin.stride(-1) != 1 or cos.stride(0) != sin.stride(0) or cos.shape[0] < length:
        cos, sin = cos.contiguous(), sin.contiguous()
    if mask.dim() == 2:
        mask = mask[:, :, None]
    mask = mask.to(torch.bfloat16)
    if lam is not None:
        lam = lam.to(device=qkv.device, dtype=torch.float32).contiguous()
    width = 2 * pair_count * head_dim
    if out is None:
        out = torch.empty(batch, length, width, dtype=torch.bfloat16, device=qkv.device)
    need = workspace_bytes(batch, length, pair_count)
    ws = workspace(need, qkv.device) if ws is None else ws
    _lib.call("hb_dense_diff_attn", ptr(qkv), qkv.stride(1), ptr(q_weight), ptr(k_weight), ptr(cos), ptr(sin),
              cos.stride(0), ptr(mask), mask.stride(0), mask.stride(1), ptr(lam), ptr(out), out.stride(1), batch,
              length, num_heads, head_dim, half, float(eps), pair_begin, pair_count, ptr(ws), ws.numel(),
              stream_handle(qkv.device))
    return out
