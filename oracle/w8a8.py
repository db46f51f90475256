"""W8A8 int8 GEMM oracle — test infrastructure. Parity UNPINNED against the reference (which has no int8 path).

The benchmark configs specify the path; the reference's site for it is `dit._feed_forward` ->
`dit._linear` (dit.py:33-36, 218-221), a bf16 `x @ W^T + b` with W stored `[out, in]`. The quantised
form fixed here, and reproduced bit for bit by the CUDA kernels:

* per row r of a bf16 matrix X `(R, K)`: `absmax = max_k |X[r, k]|` (exact), `scale = fp32(absmax) /
  fp32(127)` (one correctly rounded fp32 division; `scale = 1` when absmax is 0), `q = clamp(rint(fp32(X)
  / scale), -127, 127)` with a correctly rounded fp32 division and round-half-to-even. Activations are
  quantised per token (rows of X), weights per output channel (rows of W).
* `acc[m, n] = sum_k qx[m, k] * qw[n, k]` exactly in int32.
* `y[m, n] = bf16(fp32(fp32(fp32(acc) * sx[m]) * sw[n]) + fp32(bias[n]))`, each step one fp32 rounding
  (no fused multiply-add), int32 -> fp32 and fp32 -> bf16 round-to-nearest-even.
"""
from __future__ import annotations

import numpy as np

from oracle.common import bf16_bits_to_f32, f32_to_bf16_bits


def quantize_rows(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """fp32 view of a bf16 matrix `(R, K)` -> (int8 `(R, K)`, fp32 scales `(R,)`)."""
    x = np.asarray(x, np.float32)
    absmax = np.abs(x).max(axis=1).astype(np.float32)
    scale = (absmax / np.float32(127.0)).astype(np.float32)
    scale = np.where(absmax == 0, np.float32(1.0), scale).astype(np.float32)
    q = np.rint((x / scale[:, None]).astype(np.float32))
    return np.clip(q, -127, 127).astype(np.int8), scale


def int_matmul(qx: np.ndarray, qw: np.ndarray) -> np.ndarray:
    """Exact `qx @ qw^T` as int32 (fits for K <= 2^17). Computed as a float64 BLAS matmul, which is exact
    here: every product is an integer below 2^14 and every partial sum below 2^31 < 2^53."""
    assert qx.shape[1] <= (1 << 17)
    return (qx.astype(np.float64) @ qw.astype(np.float64).T).astype(np.int32)


def epilogue(acc: np.ndarray, sx: np.ndarray, sw: np.ndarray, bias_bits: np.ndarray | None) -> np.ndarray:
    """Fixed-order fp32 dequant + bias -> bf16 bit patterns `(M, N)` uint16."""
    f = acc.astype(np.float32)
    y = (f * np.asarray(sx, np.float32)[:, None]).astype(np.float32)
    y = (y * np.asarray(sw, np.float32)[None, :]).astype(np.float32)
    if bias_bits is not None:
        y = (y + bf16_bits_to_f32(bias_bits)[None, :]).astype(np.float32)
    return f32_to_bf16_bits(y)


def w8a8_linear(x_bits: np.ndarray, qw: np.ndarray, sw: np.ndarray, bias_bits: np.ndarray | None):
    """bf16 activations `(M, K)` (uint16 bits) -> (bf16 bits `(M, N)`, int32 acc, qx, sx)."""
    qx, sx = quantize_rows(bf16_bits_to_f32(x_bits))
    acc = int_matmul(qx, qw)
    return epilogue(acc, sx, sw, bias_bits), acc, qx, sx
