"""B200 drop-in for `sa3jax.band_attention` (band_attention.py:123-180): the SAME-L decoder's fused
differential sliding-window attention, DyT -> RoPE -> both band branches -> subtract, on sm_100a.

`band_attention(qkv, q_norm, k_norm, inv_freq, num_heads, head_dim, window)` has the reference's
signature and meaning (`q_norm`/`k_norm` are `{"alpha", "gamma", "beta"}` DyT parameters shared by both
branches); its Pallas tiling knobs (`rows`, `halo`, `sub`, `stack`, `interpret`) are accepted and ignored:
the sm_100a kernel tiles by 128 rows and walks only the key tiles inside the band. `ValueError` on
unsupported shapes, as the reference. Additions: `lam` (per-pair lambda; None = 1) and the sequence-shard
form `band_attention_shard` used with a halo exchange.

The front end of `same_l._attention` (same_l.py:151-161) runs as one GEMM here: `qkv_project` computes
`_linear(x, to_qkv)` (with `_block`'s DyT pre-norm on x when given, same_l.py:191) and, with `prepare`, the
q/k DyT + RoPE of the band kernel in its epilogue; `band_attention_prepared` then runs the band kernel without
its preparation stage. `same_l_attention_x` is the two together: x `(B, S, d)` -> band output `(B, S, H 64)`.
"""
from __future__ import annotations

import ctypes

import torch

from hummingbird_b200 import _lib
from hummingbird_b200._tensors import check_cuda, ptr, stream_handle, workspace


def pack_norm(norm: dict, device: torch.device) -> torch.Tensor:
    """`{"alpha": scalar, "gamma": (64,), "beta": (64,)}` -> fp32 `[alpha, gamma[64], beta[64]]`."""
    alpha = torch.as_tensor(norm["alpha"], dtype=torch.float32, device=device).reshape(-1)[:1]
    gamma = torch.as_tensor(norm["gamma"], dtype=torch.float32, device=device).reshape(-1)
    beta = torch.as_tensor(norm["beta"], dtype=torch.float32, device=device).reshape(-1)
    if gamma.numel() != 64 or beta.numel() != 64:
        raise ValueError("DyT gamma / beta must have 64 entries (head_dim 64)")
    return torch.cat([alpha, gamma, beta]).contiguous()


def workspace_bytes(batch: int, rows: int, pair_count: int, window: int, half: int) -> int:
    n = ctypes.c_size_t(0)
    _lib.call("hb_band_workspace_bytes", batch, rows, pair_count, window, half, ctypes.byref(n))
    return int(n.value)


def band_attention_shard(qkv: torch.Tensor, q_norm, k_norm, inv_freq: torch.Tensor, num_heads: int,
                         head_dim: int, window: int, *, q_begin: int, q_count: int, pos0: int,
                         lam: torch.Tensor | None = None, pair_begin: int = 0, pair_count: int | None = None,
                         out: torch.Tensor | None = None, ws: torch.Tensor | None = None,
                         stages: int = _lib.HB_STAGE_ALL) -> torch.Tensor:
    """Band attention over a buffer of `rows` consecutive sequence rows (a shard plus its halos):
    queries are buffer rows `[q_begin, q_begin + q_count)`, every buffer row is a key, and buffer row 0 sits
    at global position `pos0`. Returns `(B, q_count, 2 * pair_count * 64)` bf16. `stages` may issue only the
    preparation (HB_STAGE_PREPARE) or only the attention (HB_STAGE_ATTEND) half, on the same `ws`."""
    if head_dim != 64:
        raise ValueError(f"band_attention: need head_dim 64 (head_dim={head_dim})")
    if qkv.dim() != 3 or qkv.dtype != torch.bfloat16 or qkv.shape[-1] != 5 * num_heads * head_dim:
        raise ValueError(f"qkv must be bf16 (B, S, 5 * H * 64), got {tuple(qkv.shape)} {qkv.dtype}")
    check_cuda(qkv)
    batch, rows, _ = qkv.shape
    pair_count = num_heads // 2 - pair_begin if pair_count is None else pair_count
    qkv = qkv if qkv.stride(-1) == 1 and qkv.stride(0) == qkv.stride(1) * rows else qkv.contiguous()
    qn = q_norm if isinstance(q_norm, torch.Tensor) else pack_norm(q_norm, qkv.device)
    kn = k_norm if isinstance(k_norm, torch.Tensor) else pack_norm(k_norm, qkv.device)
    freqs = inv_freq.to(device=qkv.device, dtype=torch.float32).contiguous()
    if lam is not None:
        lam = lam.to(device=qkv.device, dtype=torch.float32).contiguous()
    if out is None:
        out = torch.empty(batch, q_count, 2 * pair_count * head_dim, dtype=torch.bfloat16, device=qkv.device)
    need = workspace_bytes(batch, rows, pair_count, window, freqs.shape[0])
    ws = workspace(need, qkv.device) if ws is None else ws
    _lib.call("hb_band_diff_attn", ptr(qkv), qkv.stride(1), ptr(qn), ptr(kn), ptr(freqs), freqs.shape[0], ptr(lam),
              ptr(out), out.stride(1), batch, rows, q_begin, q_count, pos0, num_heads, head_dim, window, pair_begin,
              pair_count, ptr(ws), ws.numel(), stages, stream_handle(qkv.device))
    return out


def band_attention(qkv: torch.Tensor, q_norm, k_norm, inv_freq: torch.Tensor, num_heads: int, head_dim: int,
                   window: int, *, rows: int = 1024, halo: int = 32, sub: int = 256, stack: bool = True,
                   interpret: bool = False, lam: torch.Tensor | None = None, out: torch.Tensor | None = None,
                   ws: torch.Tensor | None = None) -> torch.Tensor:
    """`(B, S, 5 * H * D)` projection output -> `(B, S, H * D)` differential band attention."""
    del rows, halo, sub, stack, interpret  # Pallas tiling knobs of the TPU kernel
    length = qkv.shape[1]
    return band_attention_shard(qkv, q_norm, k_norm, inv_freq, num_heads, head_dim, window, q_begin=0,
                                q_count=length, pos0=0, lam=lam, out=out, ws=ws)


def pack_pre_norm(norm: dict, d_model: int, device: torch.device) -> torch.Tensor:
    """The block's DyT `{"alpha": scalar, "gamma": (d,), "beta": (d,)}` -> fp32 `[alpha, gamma[d], beta[d]]`."""
    alpha = torch.as_tensor(norm["alpha"], dtype=torch.float32, device=device).reshape(-1)[:1]
    gamma = torch.as_tensor(norm["gamma"], dtype=torch.float32, device=device).reshape(-1)
    beta = torch.as_tensor(norm["beta"], dtype=torch.float32, device=device).reshape(-1)
    if gamma.numel() != d_model or beta.numel() != d_model:
        raise ValueError(f"pre-norm gamma / beta must have d_model = {d_model} entries")
    return torch.cat([alpha, gamma, beta]).contiguous()


def qkv_project(x: torch.Tensor, to_qkv: torch.Tensor, q_norm, k_norm, inv_freq: torch.Tensor, num_heads: int,
                *, pre_norm=None, prepare: bool = True, pos0: int = 0,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """`(B, S, d)` bf16 -> `(B, S, 5 H 64)` bf16: `_linear(x', to_qkv)` (same_l.py:157) with
    `x' = bf16(DyT(x, pre_norm))` when `pre_norm` is given (same_l.py:191), else x. With `prepare`, the q, k,
    q_diff, k_diff columns leave DyT'd and rotated (buffer row r at position `pos0 + r`), ready for
    `band_attention_prepared`. `to_qkv` is the checkpoint's `[5 H 64, d]` weight; d <= 512."""
    if x.dim() != 3 or x.dtype != torch.bfloat16:
        raise ValueError(f"x must be bf16 (B, S, d), got {tuple(x.shape)} {x.dtype}")
    check_cuda(x)
    batch, rows, d = x.shape
    n = 5 * num_heads * 64
    if to_qkv.dtype != torch.bfloat16 or tuple(to_qkv.shape) != (n, d):
        raise ValueError(f"to_qkv must be bf16 ({n}, {d}), got {tuple(to_qkv.shape)} {to_qkv.dtype}")
    # rows consecutive across the batch (the batch stride does not matter for one batch element)
    x = x if x.stride(-1) == 1 and (batch == 1 or x.stride(0) == x.stride(1) * rows) else x.contiguous()
    w = to_qkv if to_qkv.stride(-1) == 1 else to_qkv.contiguous()
    pre = None
    if pre_norm is not None:
        pre = pre_norm if isinstance(pre_norm, torch.Tensor) else pack_pre_norm(pre_norm, d, x.device)
    qn = kn = freqs = None
    half = 0
    if prepare:
        qn = q_norm if isinstance(q_norm, torch.Tensor) else pack_norm(q_norm, x.device)
        kn = k_norm if isinstance(k_norm, torch.Tensor) else pack_norm(k_norm, x.device)
        freqs = inv_freq.to(device=x.device, dtype=torch.float32).contiguous()
        half = freqs.shape[0]
    if out is None:
        out = torch.empty(batch, rows, n, dtype=torch.bfloat16, device=x.device)
    if out.stride(-1) != 1 or (batch > 1 and out.stride(0) != out.stride(1) * rows):
        raise ValueError("out must have unit column stride and consecutive rows across the batch")
    _lib.call("hb_band_qkv_project", ptr(x), x.stride(1), ptr(pre), ptr(w), w.stride(0), ptr(qn), ptr(kn), ptr(freqs),
              half, ptr(out), out.stride(1), batch, rows, pos0, d, num_heads, 64, 1 if prepare else 0,
              stream_handle(x.device))
    return out


def band_attention_prepared(qkv: torch.Tensor, num_heads: int, window: int, *, q_begin: int = 0,
                            q_count: int | None = None, lam: torch.Tensor | None = None, pair_begin: int = 0,
                            pair_count: int | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """`band_attention_shard` on the output of `qkv_project(..., prepare=True)`: the same result as the raw
    projection through `band_attention_shard`, without the preparation stage. Window <= 128."""
    if qkv.dim() != 3 or qkv.dtype != torch.bfloat16 or qkv.shape[-1] != 5 * num_heads * 64:
        raise ValueError(f"qkv must be bf16 (B, S, 5 * H * 64), got {tuple(qkv.shape)} {qkv.dtype}")
    check_cuda(qkv)
    batch, rows, _ = qkv.shape
    q_count = rows - q_begin if q_count is None else q_count
    pair_count = num_heads // 2 - pair_begin if pair_count is None else pair_count
    qkv = qkv if qkv.stride(-1) == 1 and qkv.stride(0) == qkv.stride(1) * rows else qkv.contiguous()
    if lam is not None:
        lam = lam.to(device=qkv.device, dtype=torch.float32).contiguous()
    if out is None:
        out = torch.empty(batch, q_count, 2 * pair_count * 64, dtype=torch.bfloat16, device=qkv.device)
    _lib.call("hb_band_diff_attn_prepared", ptr(qkv), qkv.stride(1), ptr(lam), ptr(out), out.stride(1), batch, rows,
              q_begin, q_count, num_heads, 64, window, pair_begin, pair_count, stream_handle(qkv.device))
    return out


def fused_front_end_ok(d_model: int, window: int) -> bool:
    """Whether `same_l_attention_x` takes the one-GEMM front end (d_model <= 512, window <= 128)."""
    return d_model % 64 == 0 and 64 <= d_model <= 512 and 0 <= window <= 128


def same_l_attention_x(x: torch.Tensor, to_qkv: torch.Tensor, q_norm, k_norm, inv_freq: torch.Tensor,
                       num_heads: int, window: int, *, pre_norm=None, lam: torch.Tensor | None = None,
                       qkv: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """`same_l._attention` up to `to_out` (same_l.py:151-161): x `(B, S, d)` -> `(B, S, H 64)`, through the
    one-GEMM front end and the band kernel without its preparation stage (`qkv` is an optional `(B, S, 5 H 64)`
    buffer for the prepared projection)."""
    if not fused_front_end_ok(x.shape[-1], window):
        raise ValueError(f"same_l_attention_x: needs d_model a multiple of 64 in [64, 512] and window <= 128 "
                         f"(d_model={x.shape[-1]}, window={window})")
    qkv = qkv_project(x, to_qkv, q_norm, k_norm, inv_freq, num_heads, pre_norm=pre_norm, prepare=True, out=qkv)
    return band_attention_prepared(qkv, num_heads, window, lam=lam, out=out)


_STREAMS: dict[int, tuple] = {}


def _copy_streams(device: torch.device):
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _STREAMS:
        _STREAMS[idx] = (torch.cuda.Stream(device), torch.cuda.Stream(device))
    return _STREAMS[idx]


def band_attention_from_host(qkv_host: torch.Tensor, q_norm, k_norm, inv_freq: torch.Tensor, num_heads: int,
                             head_dim: int, window: int, *, lam: torch.Tensor | None = None,
                             out_host: torch.Tensor | None = None, dev_in: torch.Tensor | None = None,
                             dev_out: torch.Tensor | None = None, layout: dict | None = None, comm=None,
                             chunk_rows: int = 8192) -> torch.Tensor:
    """Band attention of a projection held in pinned HOST memory, streamed through the GPU.

    `qkv_host` `(B, R, 5 H 64)` bf16 pinned; the result goes to `out_host` `(B, R, H 64)` (pinned). Rows are
    copied to the device in chunks on one copy stream; the queries of a chunk run (on the current stream) as
    soon as their rows and the `window` rows after them have landed (whole 128-row key tiles); finished rows
    go back on a second copy stream, so the two copy directions and the kernel overlap. Returns `out_host`;
    the current stream is ordered after the last copy back (synchronise it before reading the result).

    With `layout` (`parallel.band_layout`) and `comm` the rows are this rank's shard of a longer sequence:
    the rows its neighbours need go first, then the halo exchange runs on the device, then the rest streams."""
    if qkv_host.is_cuda or qkv_host.dim() != 3:
        raise ValueError("qkv_host must be a (B, R, 5 * H * 64) host tensor")
    device = torch.device("cuda", torch.cuda.current_device())
    batch, own, width = qkv_host.shape
    before = layout["before"] if layout else 0
    after = layout["after"] if layout else 0
    rows = before + own + after
    out_w = num_heads * head_dim
    if out_host is None:
        out_host = torch.empty(batch, own, out_w, dtype=torch.bfloat16).pin_memory()
    if dev_in is None:
        dev_in = torch.empty(batch, rows, width, dtype=torch.bfloat16, device=device)
    if dev_out is None:
        dev_out = torch.empty(batch, own, out_w, dtype=torch.bfloat16, device=device)
    qn = q_norm if isinstance(q_norm, torch.Tensor) else pack_norm(q_norm, device)
    kn = k_norm if isinstance(k_norm, torch.Tensor) else pack_norm(k_norm, device)
    main = torch.cuda.current_stream(device)
    s_in, s_out = _copy_streams(device)
    s_in.wait_stream(main)
    s_out.wait_stream(main)
    pos0 = layout["pos0"] if layout else 0
    chunk = max(128, chunk_rows // 128 * 128)
    first = [0] * batch  # own rows [0, first[b]) are already on the device
    if layout and layout["world"] > 1:
        # the rows the neighbours need go first (every batch element), then one halo exchange on the device
        from hummingbird_b200 import parallel as par
        w, rk, length, win = layout["world"], comm.rank, layout["length"], layout["window"]
        nl = par.band_layout(length, w, rk - 1, win)["after"] if rk > 0 else 0
        nr = par.band_layout(length, w, rk + 1, win)["before"] if rk < w - 1 else 0
        with torch.cuda.stream(s_in):
            for b in range(batch):
                dev_in[b, before:before + nl].copy_(qkv_host[b, :nl], non_blocking=True)
                dev_in[b, before + own - nr:before + own].copy_(qkv_host[b, own - nr:], non_blocking=True)
        main.wait_stream(s_in)
        comm.halo_exchange(dev_in, layout)
        first = [nl] * batch
    for b in range(batch):
        copied = first[b]
        for c0 in range(0, own, chunk):
            c1 = min(own, c0 + chunk)
            # whole key tiles up to `window` rows past the chunk (buffer coordinates), within the own rows
            need = min(own, -(-(before + c1 + window) // 128) * 128 - before)
            if need > copied:
                with torch.cuda.stream(s_in):
                    dev_in[b, before + copied:before + need].copy_(qkv_host[b, copied:need], non_blocking=True)
                main.wait_stream(s_in)
                copied = need
            band_attention_shard(dev_in[b:b + 1], qn, kn, inv_freq, num_heads, head_dim, window,
                                 q_begin=before + c0, q_count=c1 - c0, pos0=pos0, lam=lam,
                                 out=dev_out[b:b + 1, c0:c1])
            s_out.wait_stream(main)
            with torch.cuda.stream(s_out):
                out_host[b, c0:c1].copy_(dev_out[b, c0:c1], non_blocking=True)
    main.wait_stream(s_out)
    return out_host



def same_l_attention_from_host(x_host: torch.Tensor, to_qkv: torch.Tensor, q_norm, k_norm, inv_freq: torch.Tensor,
                               num_heads: int, window: int, *, to_out: torch.Tensor | None = None, pre_norm=None,
                               lam: torch.Tensor | None = None, out_host: torch.Tensor | None = None,
                               dev_x: torch.Tensor | None = None, dev_qkv: torch.Tensor | None = None,
                               dev_att: torch.Tensor | None = None, dev_out: torch.Tensor | None = None,
                               layout: dict | None = None, comm=None, chunk_rows: int = 16384) -> torch.Tensor:
    """`same_l._attention` (same_l.py:151-161) of a layer input held in pinned HOST memory: x `(B, R, d)` bf16
    streams to the device in chunks; each chunk's rows go through the one-GEMM front end (`qkv_project`,
    prepared, at their sequence positions); a chunk's queries run through the band kernel once the rows up to
    `window` past them are projected; with `to_out` (`[H 64, H 64]`, the checkpoint's `[out, in]`) the output
    projection follows on the chunk; finished rows go back to `out_host` `(B, R, H 64)` (pinned) on a second copy
    stream. Only x and the output cross PCIe (the projection never does). Returns `out_host`; the current stream
    is ordered after the last copy back.

    With `layout` (`parallel.band_layout`) and `comm` the rows are this rank's shard of a longer sequence: the
    rows the neighbours need are projected first and their prepared projections exchanged on the device (the
    halo rows keep the positions their owner gave them), then the rest streams."""
    if x_host.is_cuda or x_host.dim() != 3:
        raise ValueError("x_host must be a (B, R, d) host tensor")
    device = torch.device("cuda", torch.cuda.current_device())
    batch, own, d = x_host.shape
    if not fused_front_end_ok(d, window):
        raise ValueError(f"same_l_attention_from_host: needs d_model a multiple of 64 in [64, 512] and window <= 128 "
                         f"(d_model={d}, window={window})")
    before = layout["before"] if layout else 0
    after = layout["after"] if layout else 0
    rows = before + own + after
    width, out_w = 5 * num_heads * 64, num_heads * 64
    if out_host is None:
        out_host = torch.empty(batch, own, out_w, dtype=torch.bfloat16).pin_memory()
    if dev_x is None:
        dev_x = torch.empty(batch, own, d, dtype=torch.bfloat16, device=device)
    if dev_qkv is None:
        dev_qkv = torch.empty(batch, rows, width, dtype=torch.bfloat16, device=device)
    if dev_att is None:
        dev_att = torch.empty(batch, own, out_w, dtype=torch.bfloat16, device=device)
    if to_out is not None and dev_out is None:
        dev_out = torch.empty(batch, own, out_w, dtype=torch.bfloat16, device=device)
    qn = q_norm if isinstance(q_norm, torch.Tensor) else pack_norm(q_norm, device)
    kn = k_norm if isinstance(k_norm, torch.Tensor) else pack_norm(k_norm, device)
    pre = None
    if pre_norm is not None:
        pre = pre_norm if isinstance(pre_norm, torch.Tensor) else pack_pre_norm(pre_norm, d, device)
    freqs = inv_freq.to(device=device, dtype=torch.float32).contiguous()
    main = torch.cuda.current_stream(device)
    s_in, s_out = _copy_streams(device)
    s_in.wait_stream(main)
    s_out.wait_stream(main)
    pos_base = (layout["pos0"] if layout else 0) + before  # global position of own row 0

    def project(b: int, r0: int, r1: int) -> None:  # own rows [r0, r1) of batch b, already on the device
        qkv_project(dev_x[b:b + 1, r0:r1], to_qkv, qn, kn, freqs, num_heads, pre_norm=pre, prepare=True,
                    pos0=pos_base + r0, out=dev_qkv[b:b + 1, before + r0:before + r1])

    def fetch(b: int, r0: int, r1: int) -> None:
        with torch.cuda.stream(s_in):
            dev_x[b, r0:r1].copy_(x_host[b, r0:r1], non_blocking=True)

    chunk = max(128, chunk_rows // 128 * 128)
    nl = nr = 0  # own rows the left / right neighbour needs (projected first when sharded)
    if layout and layout["world"] > 1:
        # the rows the neighbours need first (every batch element), projected, then one halo exchange
        from hummingbird_b200 import parallel as par
        w, rk, length, win = layout["world"], comm.rank, layout["length"], layout["window"]
        nl = par.band_layout(length, w, rk - 1, win)["after"] if rk > 0 else 0
        nr = par.band_layout(length, w, rk + 1, win)["before"] if rk < w - 1 else 0
        for b in range(batch):
            if nl:
                fetch(b, 0, nl)
            if nr:
                fetch(b, own - nr, own)
        main.wait_stream(s_in)
        for b in range(batch):
            if nl:
                project(b, 0, nl)
            if nr:
                project(b, own - nr, own)
        comm.halo_exchange(dev_qkv, layout)
    for b in range(batch):
        done, tail_done = nl, own - nr  # own rows [0, done) and [tail_done, own) are projected
        for c0 in range(0, own, chunk):
            c1 = min(own, c0 + chunk)
            # whole key tiles up to `window` rows past the chunk (buffer coordinates), within the own rows
            need = min(own, -(-(before + c1 + window) // 128) * 128 - before)
            hi = min(need, tail_done)
            if hi > done:
                fetch(b, done, hi)
                main.wait_stream(s_in)
                project(b, done, hi)
                done = hi
            band_attention_prepared(dev_qkv[b:b + 1], num_heads, window, q_begin=before + c0, q_count=c1 - c0,
                                    lam=lam, out=dev_att[b:b + 1, c0:c1])
            res = dev_att
            if to_out is not None:
                torch.matmul(dev_att[b, c0:c1], to_out.t(), out=dev_out[b, c0:c1])
                res = dev_out
            s_out.wait_stream(main)
            with torch.cuda.stream(s_out):
                out_host[b, c0:c1].copy_(res[b, c0:c1], non_blocking=True)
    main.wait_stream(s_out)
    return out_host
