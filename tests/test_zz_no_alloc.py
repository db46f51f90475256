"""The allocation-free dense attention entry point, `hb_dense_diff_attn_noalloc`, called through the C ABI.

It exists for callers that cannot allocate device memory or hand the library a workspace, such as a
handler running inside a runtime that has already reserved most of the GPU's memory for its own allocator,
or code that must not let cudaMalloc / cudaFree synchronise the device. Its scratch is one fixed array inside
the library, so these tests check that (1) two calls in a row, with different problems, each give the same
output as the workspace entry point `hb_dense_diff_attn` (the second call runs over the scratch contents the
first one left behind), and (2) a problem too large for the fixed scratch is refused before any launch.

The file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch

from gpu_util import check_attn, f32_cuda, to_np


def _noalloc_args(w, cos, sin, mask, q_w, k_w, lam, out, pair_begin=0, pair_count=None):
    batch, length, _ = w.qkv.shape
    pair_count = w.heads // 2 if pair_count is None else pair_count
    return (w.qkv.data_ptr(), w.qkv.stride(1), q_w.data_ptr(), k_w.data_ptr(), cos.data_ptr(), sin.data_ptr(),
            cos.stride(0), mask.data_ptr(), mask.stride(0), mask.stride(1), lam.data_ptr(), out.data_ptr(),
            out.stride(1), batch, length, w.heads, 64, w.half, ctypes.c_float(w.eps), pair_begin, pair_count,
            torch.cuda.current_stream().cuda_stream)


def test_noalloc_rejects_problems_larger_than_its_scratch():
    """Host-side refusal: no pointer is dereferenced and nothing is launched (runs without a GPU)."""
    from hummingbird_b200 import _lib, build
    build.build()
    lib = _lib.lib()
    cap = ctypes.c_size_t(0)
    assert lib.hb_dense_noalloc_max_bytes(ctypes.byref(cap)) == _lib.HB_OK
    need = ctypes.c_size_t(0)
    assert lib.hb_dense_workspace_bytes(8, 4096, 8, ctypes.byref(need)) == _lib.HB_OK
    assert need.value > cap.value
    fake = 1 << 20  # aligned, never dereferenced: the size check comes first
    rc = lib.hb_dense_diff_attn_noalloc(fake, 5120, fake, fake, fake, fake, 128, fake, 4096, 1, None, fake, 1024, 8,
                                        4096, 16, 64, 32, ctypes.c_float(1e-6), 0, 8, None)
    assert rc == _lib.HB_ERR_WORKSPACE


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_twice(cuda_lib):
    from hummingbird_b200 import _lib
    from hummingbird_b200 import dense_attention as hb
    from hummingbird_b200.workloads import dense_inputs
    problems = [dict(seed=0),  # config 1: B=1, L=646, 16 heads
                dict(seed=9, batch=2, length=300, d_model=512, heads=8, masked_tail=17)]
    for kw in problems:
        w = dense_inputs("cuda", **kw)
        batch, length, _ = w.qkv.shape
        cos, sin, mask = hb.tables(length, f32_cuda(w.inv_freq), f32_cuda(w.valid))
        q_w, k_w, lam = f32_cuda(w.q_weight), f32_cuda(w.k_weight), f32_cuda(w.lam)
        ref = hb.dense_attention(w.qkv, q_w, k_w, cos, sin, mask, w.heads, 64, w.half, w.eps, lam=lam)
        out = torch.full_like(ref, float("nan"))
        _lib.call("hb_dense_diff_attn_noalloc", *_noalloc_args(w, cos, sin, mask, q_w, k_w, lam, out))
        torch.cuda.synchronize()
        check_attn(to_np(out), to_np(ref), max_abs=2e-2, mean_abs=2e-3)
        assert np.array_equal(to_np(out), to_np(ref))  # same kernels on the same inputs: identical bits
    assert _lib.device_status() == 0


@pytest.mark.gpu
def test_noalloc_head_pair_shard_and_scratch_boundary(cuda_lib):
    """A head-pair shard with lambda (pair_begin > 0, output at that pair's columns) and a problem whose prepared
    tiles take 63.75 MiB of the 64 MiB scratch (B=1, L=6,528, 16 heads): both bit-equal to the workspace entry
    point, so the size check admits exactly what the scratch holds and the shard offsets are applied."""
    from hummingbird_b200 import _lib
    from hummingbird_b200 import dense_attention as hb
    from hummingbird_b200.workloads import dense_inputs
    w = dense_inputs("cuda", seed=5, batch=1, length=6528, d_model=1024, heads=16, masked_tail=64)
    need = ctypes.c_size_t(0)
    cap = ctypes.c_size_t(0)
    assert cuda_lib.hb_dense_workspace_bytes(1, 6528, 8, ctypes.byref(need)) == _lib.HB_OK
    assert cuda_lib.hb_dense_noalloc_max_bytes(ctypes.byref(cap)) == _lib.HB_OK
    assert cap.value - (1 << 20) < need.value <= cap.value
    cos, sin, mask = hb.tables(6528, f32_cuda(w.inv_freq), f32_cuda(w.valid))
    q_w, k_w, lam = f32_cuda(w.q_weight), f32_cuda(w.k_weight), f32_cuda(w.lam)
    ref = hb.dense_attention(w.qkv, q_w, k_w, cos, sin, mask, w.heads, 64, w.half, w.eps, lam=lam)
    out = torch.full_like(ref, float("nan"))
    _lib.call("hb_dense_diff_attn_noalloc", *_noalloc_args(w, cos, sin, mask, q_w, k_w, lam, out))
    torch.cuda.synchronize()
    assert np.array_equal(to_np(out), to_np(ref))
    # pairs 3..6 of 8 into a buffer holding only those pairs' columns
    shard = torch.full((1, 6528, 4 * 128), float("nan"), dtype=torch.bfloat16, device="cuda")
    _lib.call("hb_dense_diff_attn_noalloc", *_noalloc_args(w, cos, sin, mask, q_w, k_w, lam, shard, pair_begin=3,
                                                           pair_count=4))
    torch.cuda.synchronize()
    assert np.array_equal(to_np(shard), to_np(ref[:, :, 3 * 128:7 * 128]))
    assert _lib.device_status() == 0
