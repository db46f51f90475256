"""ctypes binding of `libhb_b200.so` (the C ABI declared in `include/hb_b200.h`).

There is no fallback: if the library is missing or fails to load, every operator raises. The library
is built in-tree by `python -m hummingbird_b200.build` (or `__graft_entry__.build()`).
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libhb_b200.so"

HB_OK, HB_ERR_SHAPE, HB_ERR_ALIGN, HB_ERR_ARCH, HB_ERR_LAUNCH = 0, 1, 2, 3, 4
HB_ERR_DEVICE, HB_ERR_TIMEOUT, HB_ERR_WORKSPACE, HB_ERR_NCCL, HB_ERR_NULL = 5, 6, 7, 8, 9
HB_STAGE_PREPARE, HB_STAGE_ATTEND, HB_STAGE_ALL = 1, 2, 3
_NAMES = {0: "ok", 1: "unsupported shape", 2: "misaligned pointer or stride", 3: "device is not sm_100",
          4: "CUDA launch failed", 5: "device error", 6: "device-side wait timed out", 7: "workspace too small",
          8: "collective failed", 9: "null pointer"}

_p, _i, _i64, _f, _sz = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t

# name -> argtypes, exactly the prototypes of include/hb_b200.h
SIGNATURES: dict[str, list] = {
    "hb_version": [],
    "hb_device_status": [C.POINTER(C.c_uint), _p],
    "hb_dense_workspace_bytes": [_i, _i, _i, C.POINTER(_sz)],
    "hb_dense_diff_attn": [_p, _i64, _p, _p, _p, _p, _i64, _p, _i64, _i64, _p, _p, _i64, _i, _i, _i, _i, _i, _f,
                           _i, _i, _p, _sz, _p],
    "hb_dense_noalloc_max_bytes": [C.POINTER(_sz)],
    "hb_dense_diff_attn_noalloc": [_p, _i64, _p, _p, _p, _p, _i64, _p, _i64, _i64, _p, _p, _i64, _i, _i, _i, _i, _i,
                                   _f, _i, _i, _p],
    "hb_cross_diff_attn": [_p, _i64, _p, _i64, _p, _p, _p, _p, _i64, _i, _i, _i, _i, _i, _f, _p],
    "hb_band_workspace_bytes": [_i, _i, _i, _i, _i, C.POINTER(_sz)],
    "hb_band_diff_attn": [_p, _i64, _p, _p, _p, _i, _p, _p, _i64, _i, _i, _i, _i, _i64, _i, _i, _i, _i, _i, _p, _sz,
                          _i, _p],
    "hb_band_qkv_project": [_p, _i64, _p, _p, _i64, _p, _p, _p, _i, _p, _i64, _i, _i, _i64, _i, _i, _i, _i, _p],
    "hb_band_diff_attn_prepared": [_p, _i64, _p, _p, _i64, _i, _i, _i, _i, _i, _i, _i, _i, _i, _p],
    "hb_quant_rows_int8": [_p, _i64, _i, _i, _p, _i64, _p, _p],
    "hb_w8a8_gemm": [_p, _i64, _p, _p, _i64, _p, _p, _p, _i64, _p, _i64, _i, _i, _i, _p],
    "hb_w8a8_gemm_glu": [_p, _i64, _p, _p, _i64, _p, _p, _p, _i64, _i, _i, _i, _p],
    "hb_dit_residual_norm": [_p, _i64, _p, _i64, _p, _p, _p, _i64, _p, _i, _p, _p, _i64, _i, _i, _i, _f, _p],
    "hb_dit_residual_norm_int8": [_p, _i64, _p, _i64, _p, _p, _p, _i64, _p, _i, _p, _p, _i64, _p, _i, _i, _i, _f, _p],
    "hb_glu_rows": [_p, _i64, _i, _i, _p, _i64, _p, _i64, _p, _p],
    "hb_head_rms_norm": [_p, _i64, _i, _i, _p, _f, _p, _i64, _p],
}

_lib: C.CDLL | None = None


class HbError(RuntimeError):
    def __init__(self, fn: str, code: int):
        super().__init__(f"{fn} failed: status {code} ({_NAMES.get(code, 'unknown')})")
        self.code = code


def lib() -> C.CDLL:
    """Load the library once; raise if it is missing (no fallback path exists)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m hummingbird_b200.build`")
        handle = C.CDLL(str(LIB_PATH))
        for name, args in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = C.c_int
        _lib = handle
    return _lib


def call(name: str, *args) -> None:
    """Call an entry point; HB_ERR_SHAPE becomes ValueError (as the reference raises), others HbError."""
    code = getattr(lib(), name)(*args)
    if code == HB_ERR_SHAPE:
        raise ValueError(f"{name}: unsupported shape or argument")
    if code != HB_OK:
        raise HbError(name, code)


def device_status(stream: int = 0) -> int:
    """Read and clear the device status word (nonzero after a device-side timeout)."""
    v = C.c_uint(0)
    call("hb_device_status", C.byref(v), stream)
    return int(v.value)
