"""The multi-GPU exchanges through the library's own NCCL C ABI (`libhb_comm.so`, include/hb_comm.h):
band-attention halo send/recv and the dense head-pair all-gather, with host-side deadlines.

`HbComm` wraps one communicator. The id is created by rank 0 and handed to the other ranks over an existing
torch.distributed group (any backend); after that the data path runs through the C ABI only.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import torch

from hummingbird_b200._lib import HB_ERR_SHAPE, HB_OK, HbError

COMM_LIB_PATH = Path(__file__).resolve().parent / "libhb_comm.so"
ID_BYTES = 128

_p, _i, _i64 = C.c_void_p, C.c_int, C.c_int64
SIGNATURES: dict[str, list] = {
    "hb_comm_unique_id": [_p],
    "hb_comm_init": [_p, _i, _i, _i, C.POINTER(_p)],
    "hb_comm_halo_exchange": [_p, _p, _i, _i64, _i64, _i, _i, _i, _i, _i, _i, _p],
    "hb_comm_allgather_pairs": [_p, _p, _i64, _i64, C.POINTER(_i64), _p, _p, _i64, _i, _p],
    "hb_comm_abort": [_p],
    "hb_comm_destroy": [_p],
    "hb_comm_size": [_p, C.POINTER(_i), C.POINTER(_i)],
}
_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """Load `libhb_comm.so` once; raise if it is missing (there is no other exchange path behind it)."""
    global _lib
    if _lib is None:
        if not COMM_LIB_PATH.exists():
            raise RuntimeError(f"{COMM_LIB_PATH} is missing: build it with `python -m hummingbird_b200.build`")
        handle = C.CDLL(str(COMM_LIB_PATH))
        for name, args in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = C.c_int
        _lib = handle
    return _lib


def _call(name: str, *args) -> None:
    code = getattr(lib(), name)(*args)
    if code == HB_ERR_SHAPE:
        raise ValueError(f"{name}: unsupported shape or argument")
    if code != HB_OK:
        raise HbError(name, code)


def unique_id() -> bytes:
    buf = C.create_string_buffer(ID_BYTES)
    _call("hb_comm_unique_id", buf)
    return buf.raw


class HbComm:
    """One NCCL communicator over `world` ranks (one per GPU), created through the C ABI."""

    def __init__(self, rank: int, world: int, *, uid: bytes | None = None, group=None, timeout_ms: int = 60_000):
        if uid is None:
            import torch.distributed as dist
            box = [unique_id() if rank == 0 else None]
            dist.broadcast_object_list(box, src=0, group=group)
            uid = box[0]
        self.rank, self.world, self.timeout_ms = rank, world, timeout_ms
        handle = C.c_void_p()
        _call("hb_comm_init", C.create_string_buffer(uid, ID_BYTES), world, rank, timeout_ms, C.byref(handle))
        self._h = handle

    def halo_exchange(self, buf: torch.Tensor, layout: dict) -> None:
        """Fill the halo rows of `buf` `(B, rows, width)` laid out as `parallel.band_layout`, on the current stream."""
        from hummingbird_b200 import parallel as par
        b, rows, width = buf.shape
        if not buf.is_contiguous():
            raise ValueError("halo_exchange needs a contiguous buffer")
        rb = width * buf.element_size()
        world, length, window = layout["world"], layout["length"], layout["window"]
        send_left = par.band_layout(length, world, self.rank - 1, window)["after"] if self.rank > 0 else 0
        send_right = par.band_layout(length, world, self.rank + 1, window)["before"] if self.rank < world - 1 else 0
        _call("hb_comm_halo_exchange", self._h, buf.data_ptr(), b, rows * rb, rb, layout["before"], layout["q_count"],
              layout["after"], send_left, send_right, self.timeout_ms,
              torch.cuda.current_stream(buf.device).cuda_stream)

    def gather_pairs(self, local: torch.Tensor, pairs: int) -> torch.Tensor:
        """All-gather head-pair pieces `(B, L, (p1 - p0) * 128)` into `(B, L, pairs * 128)` (uneven splits allowed)."""
        from hummingbird_b200 import parallel as par
        b, length, w = local.shape
        es = local.element_size()
        widths = [(p1 - p0) * 128 * es for p0, p1 in (par.shard_pairs(pairs, self.world, r) for r in range(self.world))]
        local = local.contiguous()
        out = local.new_empty(b, length, pairs * 128)
        gathered = torch.empty(self.world * b * length * max(widths), dtype=torch.uint8, device=local.device)
        arr = (C.c_int64 * self.world)(*widths)
        _call("hb_comm_allgather_pairs", self._h, local.data_ptr(), w * es, b * length, arr, gathered.data_ptr(),
              out.data_ptr(), pairs * 128 * es, self.timeout_ms, torch.cuda.current_stream(local.device).cuda_stream)
        return out

    def close(self) -> None:
        if self._h:
            _call("hb_comm_destroy", self._h)
            self._h = None

    def abort(self) -> None:
        if self._h:
            _call("hb_comm_abort", self._h)
            self._h = None
