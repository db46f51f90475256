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


_WS: dict[int, torch.Tensor] = {}
_WS_RETIRED: list[torch.Tensor] = []


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """A per-device cached uint8 workspace of at least `nbytes` (grown on demand).

    Calls on one device and stream reuse it back to back; callers that run operators concurrently on
    several streams pass their own `ws=` buffers instead. A buffer that is outgrown is kept alive, not
    freed: a CUDA graph captured earlier may still hold its address."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _WS.get(idx)
    if buf is None or buf.numel() < nbytes:
        if buf is not None:
            _WS_RETIRED.append(buf)
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WS[idx] = buf
    return buf
