"""The elementwise glue of a DiT block as fused sm_100a row kernels (`hb_dit_residual_norm`, `hb_glu_rows`,
`hb_head_rms_norm`): the steps `sa3jax.dit._block` (dit.py:224-250), `_feed_forward` (dit.py:218-221) and
`_attend`'s q norm (dit.py:150-176) run as separate XLA ops. Torch CUDA tensors, current stream, no CPU path.
"""
from __future__ import annotations

import torch

from hummingbird_b200 import _lib
from hummingbird_b200._tensors import check_cuda, ptr, stream_handle


def _rows(t: torch.Tensor) -> torch.Tensor:
    """`(..., d)` bf16 with unit stride in the last dim and uniform row stride, viewed as `(rows, d)`."""
    if t.dtype != torch.bfloat16:
        raise ValueError("the DiT glue kernels take bf16 tensors")
    flat = t.reshape(-1, t.shape[-1])
    if flat.stride(-1) != 1:
        raise ValueError("rows must be contiguous in their last dim")
    return flat


def residual_norm(h: torch.Tensor, *, y: torch.Tensor | None = None, gate: torch.Tensor | None = None,
                  local: torch.Tensor | None = None, local_row0: int = 0, weight: torch.Tensor | None = None,
                  scale: torch.Tensor | None = None, shift: torch.Tensor | None = None, eps: float = 1e-5,
                  out: torch.Tensor | None = None, quantize: bool = False):
    """In place on `h` `(B, T, d)`: `h += y * sigmoid(1 - gate)` (gate `(B, d)`, optional), `h[:, t >= local_row0]
    += local`; then, if `weight` is given, returns `RMSNorm(h) * weight * (1 + scale) + shift` (scale, shift
    `(B, d)`, optional). `gate`, `scale`, `shift` may be column slices of one `(B, k * d)` tensor. With
    `quantize`, that result comes per row in int8 form for a W8A8 GEMM: `(q (B * T, d) int8, scale (B * T,) fp32)`,
    exactly `w8a8.quantize_rows` of the bf16 result."""
    bsz, t, d = h.shape
    if not h.is_contiguous():
        raise ValueError("h must be contiguous")
    check_cuda(h)
    cond = [c for c in (gate, scale, shift) if c is not None]
    ldc = cond[0].stride(0) if cond else d
    for c in cond:
        if c.shape != (bsz, d) or c.stride() != (ldc, 1) or c.dtype != torch.bfloat16:
            raise ValueError("gate / scale / shift must be (B, d) bf16 rows of one common stride")
    y2 = None if y is None else _rows(y)
    if quantize:
        if weight is None:
            raise ValueError("the quantised output is the normalised x: weight is required")
        q = torch.empty(bsz * t, d, dtype=torch.int8, device=h.device)
        qs = torch.empty(bsz * t, dtype=torch.float32, device=h.device)
        _lib.call("hb_dit_residual_norm_int8", ptr(h), d, ptr(y2), 0 if y2 is None else y2.stride(0), ptr(gate),
                  ptr(scale), ptr(shift), ldc, ptr(local), local_row0, ptr(weight), ptr(q), d, ptr(qs), bsz * t, t, d,
                  float(eps), stream_handle(h.device))
        return q, qs
    x = None
    if weight is not None:
        x = torch.empty_like(h) if out is None else out
    _lib.call("hb_dit_residual_norm", ptr(h), d, ptr(y2), 0 if y2 is None else y2.stride(0), ptr(gate), ptr(scale),
              ptr(shift), ldc, ptr(local), local_row0, ptr(weight), ptr(x), d, bsz * t, t, d, float(eps),
              stream_handle(h.device))
    return x


def glu(g: torch.Tensor, *, quantize: bool = False):
    """`value * silu(gate)` of a GLU projection `(..., 2F)` (value first): bf16 `(..., F)`, or with
    `quantize` the per-row int8 form `(q (rows, F) int8, scale (rows,) fp32)` for `w8a8_gemm`."""
    g2 = _rows(g)
    check_cuda(g2)
    rows, two_f = g2.shape
    f = two_f // 2
    if quantize:
        q = torch.empty(rows, f, dtype=torch.int8, device=g.device)
        s = torch.empty(rows, dtype=torch.float32, device=g.device)
        _lib.call("hb_glu_rows", ptr(g2), g2.stride(0), rows, f, None, 0, ptr(q), q.stride(0), ptr(s),
                  stream_handle(g.device))
        return q, s
    z = torch.empty(*g.shape[:-1], f, dtype=torch.bfloat16, device=g.device)
    _lib.call("hb_glu_rows", ptr(g2), g2.stride(0), rows, f, ptr(z), f, None, 0, None, stream_handle(g.device))
    return z


def head_rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm over every 64-dim head of `x` `(..., heads * 64)` with a bf16 `(64,)` weight."""
    x2 = _rows(x)
    check_cuda(x2)
    rows, width = x2.shape
    if width % 64:
        raise ValueError("the row width must be a multiple of 64")
    out = torch.empty(*x.shape, dtype=torch.bfloat16, device=x.device)
    weight = weight.to(torch.bfloat16).contiguous()
    _lib.call("hb_head_rms_norm", ptr(x2), x2.stride(0), rows, width // 64, ptr(weight), float(eps), ptr(out),
              width, stream_handle(x.device))
    return out
