"""W8A8 int8 linear for the DiT MLP on sm_100a (tcgen05 `kind::i8`, int32 accumulation in TMEM).

The reference has no int8 path: `dit._feed_forward` calls `dit._linear(x, W, b)` = `x @ W^T + b` in bf16
(dit.py:33-36, 218-221). `W8A8Linear` is the drop-in for those calls when `DiTConfig.ff_quant == "w8a8"`:
weights are quantised once per output channel, activations per token on every call.
"""
from __future__ import annotations

import torch

from hummingbird_b200 import _lib
from hummingbird_b200._tensors import check_cuda, ptr, stream_handle


def quantize_rows(x: torch.Tensor, q: torch.Tensor | None = None, scale: torch.Tensor | None = None):
    """bf16 `(R, K)` -> (int8 `(R, K)`, fp32 `(R,)`): scale = absmax / 127 (1 if the row is zero),
    q = clamp(rint(x / scale), -127, 127)."""
    if x.dim() != 2 or x.dtype != torch.bfloat16:
        raise ValueError("quantize_rows expects a 2-D bf16 tensor")
    check_cuda(x)
    x = x if x.stride(1) == 1 else x.contiguous()
    rows, k = x.shape
    q = torch.empty(rows, k, dtype=torch.int8, device=x.device) if q is None else q
    scale = torch.empty(rows, dtype=torch.float32, device=x.device) if scale is None else scale
    _lib.call("hb_quant_rows_int8", ptr(x), x.stride(0), rows, k, ptr(q), q.stride(0), ptr(scale),
              stream_handle(x.device))
    return q, scale


def w8a8_gemm(qx: torch.Tensor, sx: torch.Tensor, qw: torch.Tensor, sw: torch.Tensor,
              bias: torch.Tensor | None = None, *, out: torch.Tensor | None = None,
              acc_out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 `((float)(qx @ qw^T) * sx[:, None]) * sw[None, :] + bias` with int32 accumulation."""
    check_cuda(qx, sx, qw, sw)
    m, k = qx.shape
    n = qw.shape[0]
    if qw.shape[1] != k:
        raise ValueError("qx and qw must share K")
    if bias is not None:
        bias = bias.to(torch.bfloat16).contiguous()
    out = torch.empty(m, n, dtype=torch.bfloat16, device=qx.device) if out is None else out
    _lib.call("hb_w8a8_gemm", ptr(qx), qx.stride(0), ptr(sx), ptr(qw), qw.stride(0), ptr(sw), ptr(bias), ptr(out),
              out.stride(0), ptr(acc_out), 0 if acc_out is None else acc_out.stride(0), m, n, k,
              stream_handle(qx.device))
    return out


class W8A8Linear:
    """`nn.Linear` with weight `[out, in]` (the checkpoint layout, dit.py:34) run as W8A8."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None = None):
        self.qw, self.sw = quantize_rows(weight.to(torch.bfloat16).contiguous())
        self.bias = None if bias is None else bias.to(torch.bfloat16).contiguous()
        self.out_features, self.in_features = weight.shape

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.in_features).to(torch.bfloat16)
        qx, sx = quantize_rows(x2)
        return w8a8_gemm(qx, sx, self.qw, self.sw, self.bias).reshape(*lead, self.out_features)


def glu_interleave(t: torch.Tensor) -> torch.Tensor:
    """Rows (dim 0) of a GLU projection `[value (F) | gate (F)]` reordered in blocks of 128: value rows
    [128 t, 128 t + 128), then gate rows [F + 128 t, F + 128 t + 128), for t = 0 .. F / 128 - 1 — the order
    `hb_w8a8_gemm_glu` reads (each 256-column output tile holds matching value and gate columns)."""
    two_f = t.shape[0]
    f = two_f // 2
    if two_f % 256:
        raise ValueError("the GLU width F must be a multiple of 128")
    blocks = t.reshape(2, f // 128, 128, *t.shape[1:])
    return blocks.transpose(0, 1).reshape(two_f, *t.shape[1:]).contiguous()


def w8a8_gemm_glu(qx: torch.Tensor, sx: torch.Tensor, qw: torch.Tensor, sw: torch.Tensor,
                  bias: torch.Tensor | None = None, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """z = value * silu(gate) of the W8A8 GEMM `qx @ qw^T` whose weight rows are in `glu_interleave` order."""
    check_cuda(qx, sx, qw, sw)
    m, k = qx.shape
    f = qw.shape[0] // 2
    if qw.shape[1] != k:
        raise ValueError("qx and qw must share K")
    if bias is not None:
        bias = bias.to(torch.bfloat16).contiguous()
    out = torch.empty(m, f, dtype=torch.bfloat16, device=qx.device) if out is None else out
    _lib.call("hb_w8a8_gemm_glu", ptr(qx), qx.stride(0), ptr(sx), ptr(qw), qw.stride(0), ptr(sw), ptr(bias), ptr(out),
              out.stride(0), m, f, k, stream_handle(qx.device))
    return out


class W8A8GluLinear:
    """The MLP's GLU projection (`glu_proj`, weight `[2F, in]` = [value | gate] rows) run as W8A8 with
    `value * silu(gate)` in the GEMM epilogue: `__call__(x)` returns z `[..., F]` in bf16."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None = None):
        w = glu_interleave(weight.to(torch.bfloat16))
        self.qw, self.sw = quantize_rows(w)
        self.bias = None if bias is None else glu_interleave(bias.to(torch.bfloat16))
        self.out_features, self.in_features = weight.shape[0] // 2, weight.shape[1]

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.in_features).to(torch.bfloat16)
        qx, sx = quantize_rows(x2)
        return w8a8_gemm_glu(qx, sx, self.qw, self.sw, self.bias).reshape(*lead, self.out_features)

    def quantized(self, qx: torch.Tensor, sx: torch.Tensor) -> torch.Tensor:
        """z `(rows, F)` from an activation already quantised per row (`quantize_rows` form)."""
        return w8a8_gemm_glu(qx, sx, self.qw, self.sw, self.bias)
