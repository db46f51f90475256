"""Torch plumbing for the ctypes calls: raw pointers, the current stream, workspaces."""
from __future__ import annotations

import torch


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def check_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError("hummingbird_b200 operators run on CUDA tensors only (there is no CPU path)")


_WS: dict[tuple[int, int], torch.Tensor] = {}


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """A per-device cached uint8 workspace of at least `nbytes` (grown on demand, never shrunk).

    Calls on one device and stream reuse it back to back; callers that run operators concurrently on
    several streams pass their own `ws=` buffers instead."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, 0)
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WS[key] = buf
    return buf
