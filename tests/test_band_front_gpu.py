"""GPU parity: the SAME-L attention front end in one GEMM (`hb_band_qkv_project`: block DyT pre-norm ->
`to_qkv` -> q/k DyT + RoPE) and the band kernel on its prepared output (`hb_band_diff_attn_prepared`).

* The projection (prepare = 0) against `oracle.band.front_end` (`same_l._block`'s `_dyt(x, pre_norm)` cast to
  bf16, then `_linear(x, to_qkv)`, same_l.py:52-69, 157, 191): without the pre-norm every entry within one bf16
  rounding of the exact product plus the fp32 summation bound K 2^-24 sum|x w| (entries whose dot product
  nearly cancels carry that absolute error, many ulps of a tiny result), and equal on all but a tiny share; with
  the pre-norm, within a relative L2 error of 2e-3 (the kernel's tanh is the hardware approximation, relative
  error ~2^-11, which moves some bf16 roundings of x').
* The prepared path against the raw path: bit-identical outputs (the projection's epilogue runs the band
  kernel's own DyT / RoPE arithmetic), for ragged lengths, two batch elements, windows 0 / 17 / 128, head-pair
  ranges, query ranges and sequence shards projected at their own positions, and at config 2's full size.
* x -> out against the oracle at the attention tolerance, on the golden windows and on sampled config-2 blocks.
"""
import numpy as np
import pytest
import torch

from gpu_util import check_attn, f32_cuda, to_np
from oracle import band as oband

pytestmark = pytest.mark.gpu


def _inputs(**kw):
    from hummingbird_b200.workloads import band_layer_inputs
    return band_layer_inputs("cuda", **kw)


@pytest.mark.parametrize("batch,length,d_model,heads", [(1, 1000, 512, 8), (2, 300, 256, 4), (1, 129, 64, 2)])
def test_projection_matches_oracle(batch, length, d_model, heads, cuda_lib):
    from hummingbird_b200.band_attention import qkv_project
    w = _inputs(batch=batch, length=length, d_model=d_model, heads=heads)
    x, wt = to_np(w.x).astype(np.float64), to_np(w.to_qkv).astype(np.float64)
    raw = to_np(qkv_project(w.x, w.to_qkv, None, None, None, heads, prepare=False)).astype(np.float64)
    ref = oband.front_end(x, wt)
    exact = x @ wt.T
    bound = 2.0 ** -8 * np.abs(exact) + d_model * 2.0 ** -24 * (np.abs(x) @ np.abs(wt).T) + 1e-30
    assert np.all(np.abs(raw - exact) <= bound), np.max(np.abs(raw - exact) / bound)
    assert np.mean(raw != ref) < 2e-3, np.mean(raw != ref)
    # with the block pre-norm
    raw = qkv_project(w.x, w.to_qkv, None, None, None, heads, pre_norm=w.pre_norm, prepare=False)
    ref = oband.front_end(to_np(w.x), to_np(w.to_qkv), w.pre_norm)
    got = to_np(raw).astype(np.float64)
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    print(f"projection with pre-norm: relative L2 {rel:.2e}")
    assert rel < 2e-3, rel


@pytest.mark.parametrize("window", [0, 17, 128])
def test_prepared_equals_raw_path_bit_for_bit(window, cuda_lib):
    from hummingbird_b200.band_attention import (band_attention_prepared, band_attention_shard, pack_norm,
                                                 qkv_project)
    w = _inputs(batch=2, length=1000, d_model=256, heads=4, window=window)
    freqs = f32_cuda(w.inv_freq)
    qn, kn = pack_norm(w.q_norm, "cuda"), pack_norm(w.k_norm, "cuda")
    lam = f32_cuda(w.lam)
    raw = qkv_project(w.x, w.to_qkv, qn, kn, freqs, w.heads, pre_norm=w.pre_norm, prepare=False)
    prep = qkv_project(w.x, w.to_qkv, qn, kn, freqs, w.heads, pre_norm=w.pre_norm, prepare=True)
    # v columns are untouched by the preparation
    sec = w.heads * 64
    assert torch.equal(raw[..., 2 * sec:3 * sec], prep[..., 2 * sec:3 * sec])
    for kw in (dict(), dict(pair_begin=1, pair_count=1), dict(q_begin=130, q_count=500)):
        q_begin, q_count = kw.get("q_begin", 0), kw.get("q_count", 1000)
        pb, pc = kw.get("pair_begin", 0), kw.get("pair_count", None)
        a = band_attention_shard(raw, qn, kn, freqs, w.heads, 64, window, q_begin=q_begin, q_count=q_count, pos0=0,
                                 lam=lam, pair_begin=pb, pair_count=pc)
        b = band_attention_prepared(prep, w.heads, window, q_begin=q_begin, q_count=q_count, lam=lam, pair_begin=pb,
                                    pair_count=pc)
        assert torch.equal(a, b), kw


def test_prepared_sequence_shards(cuda_lib):
    """Each shard's rows plus `window` halo rows each side, projected at their own positions (`pos0`): the
    prepared band kernel on the owned queries equals the raw projection of the same buffer through
    `band_attention_shard` bit for bit, and the concatenated shards match the unsharded oracle. (Shards start
    their 128-row key tiles at their first buffer row, so their online-softmax order differs from the unsharded
    call's: shards are compared with the oracle, not bit for bit with the unsharded output.)"""
    from hummingbird_b200.band_attention import band_attention_prepared, band_attention_shard, qkv_project
    window, length = 128, 1100
    w = _inputs(length=length, d_model=256, heads=4, window=window)
    freqs, lam = f32_cuda(w.inv_freq), f32_cuda(w.lam)
    bounds = np.linspace(0, length, 4).astype(int)
    parts = []
    for s0, s1 in zip(bounds[:-1], bounds[1:]):
        lo, hi = max(0, s0 - window), min(length, s1 + window)
        xs = w.x[:, lo:hi]
        prep = qkv_project(xs, w.to_qkv, w.q_norm, w.k_norm, freqs, w.heads, pre_norm=w.pre_norm, pos0=lo)
        raw = qkv_project(xs, w.to_qkv, None, None, None, w.heads, pre_norm=w.pre_norm, prepare=False)
        a = band_attention_prepared(prep, w.heads, window, q_begin=s0 - lo, q_count=s1 - s0, lam=lam)
        b = band_attention_shard(raw, w.q_norm, w.k_norm, freqs, w.heads, 64, window, q_begin=s0 - lo,
                                 q_count=s1 - s0, pos0=lo, lam=lam)
        assert torch.equal(a, b), (s0, s1)
        parts.append(to_np(a))
    qkv = oband.front_end(to_np(w.x), to_np(w.to_qkv), w.pre_norm)
    ref = oband.band_diff_attention(qkv, w.q_norm, w.k_norm, w.inv_freq, w.heads, window, lam=w.lam)
    check_attn(np.concatenate(parts, axis=1), ref)


@pytest.mark.parametrize("window,length", [(17, 204), (128, 384), (128, 1000)])
def test_front_end_against_oracle(window, length, cuda_lib):
    from hummingbird_b200.band_attention import same_l_attention_x
    w = _inputs(length=length, d_model=256, heads=4, window=window)
    out = same_l_attention_x(w.x, w.to_qkv, w.q_norm, w.k_norm, f32_cuda(w.inv_freq), w.heads, window,
                             pre_norm=w.pre_norm, lam=f32_cuda(w.lam))
    qkv = oband.front_end(to_np(w.x), to_np(w.to_qkv), w.pre_norm)
    ref = oband.band_diff_attention(qkv, w.q_norm, w.k_norm, w.inv_freq, w.heads, window, lam=w.lam)
    check_attn(to_np(out), ref)


def test_front_end_config2_full_length(cuda_lib):
    """Config 2 at full size through the front end (x (1, 82,688, 512), 8 heads, window 128): the prepared path
    equals the raw-projection path bit for bit over the whole output, and sampled query blocks match the oracle
    run on this projection."""
    from hummingbird_b200.band_attention import band_attention, qkv_project, same_l_attention_x
    w = _inputs()
    freqs, lam = f32_cuda(w.inv_freq), f32_cuda(w.lam)
    out = same_l_attention_x(w.x, w.to_qkv, w.q_norm, w.k_norm, freqs, w.heads, w.window, pre_norm=w.pre_norm,
                             lam=lam)
    raw = qkv_project(w.x, w.to_qkv, None, None, None, w.heads, pre_norm=w.pre_norm, prepare=False)
    assert torch.equal(out, band_attention(raw, w.q_norm, w.k_norm, freqs, w.heads, 64, w.window, lam=lam))
    qkv = to_np(raw)
    out = to_np(out)
    del raw
    rng = np.random.default_rng(0)
    starts = sorted({0, qkv.shape[1] - 384, *rng.integers(0, qkv.shape[1] - 384, 4).tolist()})
    for s in starts:
        lo, hi = max(0, s - w.window), min(qkv.shape[1], s + 384 + w.window)
        ref = oband.band_diff_attention(qkv[:, lo:hi], w.q_norm, w.k_norm, w.inv_freq, w.heads, w.window, lam=w.lam,
                                        offset=lo)
        check_attn(out[:, s:s + 384], ref[:, s - lo:s - lo + 384])


def test_front_end_config5_length(cuda_lib):
    """Config 5's decoder length (x (1, 261,888, 512), 8 heads, window 128): the front end's RoPE in the GEMM
    epilogue must give the band kernel's own preparation bit for bit at positions up to 261,887 too, so the
    prepared path equals the raw-projection path over the whole output; the last query block matches the oracle
    on this projection."""
    from hummingbird_b200.band_attention import band_attention, qkv_project, same_l_attention_x
    w = _inputs(length=261_888)
    freqs, lam = f32_cuda(w.inv_freq), f32_cuda(w.lam)
    out = same_l_attention_x(w.x, w.to_qkv, w.q_norm, w.k_norm, freqs, w.heads, w.window, pre_norm=w.pre_norm,
                             lam=lam)
    raw = qkv_project(w.x, w.to_qkv, None, None, None, w.heads, pre_norm=w.pre_norm, prepare=False)
    assert torch.equal(out, band_attention(raw, w.q_norm, w.k_norm, freqs, w.heads, 64, w.window, lam=lam))
    length = raw.shape[1]
    s = length - 384
    lo = s - w.window
    ref = oband.band_diff_attention(to_np(raw[:, lo:]), w.q_norm, w.k_norm, w.inv_freq, w.heads, w.window,
                                    lam=w.lam, offset=lo)
    check_attn(to_np(out[:, s:]), ref[:, s - lo:])


def test_layer_from_host_equals_device_call(cuda_lib):
    """`same_l_attention_from_host` (pinned host x streamed in 256-row chunks, projected per chunk at its
    positions, band kernel per chunk of queries, rows copied back) equals the device call `same_l_attention_x`
    bit for bit, for two batch elements; with `to_out` (a bf16 matmul per chunk) it matches the device call
    followed by one `to_out` matmul within a bf16 rounding (the library may pick another GEMM per row count)."""
    from hummingbird_b200.band_attention import same_l_attention_from_host, same_l_attention_x
    w = _inputs(batch=2, length=1000, d_model=256, heads=4)
    freqs, lam = f32_cuda(w.inv_freq), f32_cuda(w.lam)
    g = torch.Generator(device="cuda").manual_seed(5)
    to_out = (torch.randn(256, 256, generator=g, device="cuda") / 16).to(torch.bfloat16)
    dev = same_l_attention_x(w.x, w.to_qkv, w.q_norm, w.k_norm, freqs, w.heads, w.window, pre_norm=w.pre_norm,
                             lam=lam)
    x_host = w.x.cpu().pin_memory()
    kw = dict(pre_norm=w.pre_norm, lam=lam, chunk_rows=256)
    out = same_l_attention_from_host(x_host, w.to_qkv, w.q_norm, w.k_norm, freqs, w.heads, w.window, **kw)
    torch.cuda.synchronize()
    assert torch.equal(out, dev.cpu())
    out = same_l_attention_from_host(x_host, w.to_qkv, w.q_norm, w.k_norm, freqs, w.heads, w.window, to_out=to_out,
                                     **kw)
    torch.cuda.synchronize()
    ref = torch.stack([dev[b] @ to_out.t() for b in range(2)]).float().cpu()
    assert torch.allclose(out.float(), ref, rtol=2 ** -7, atol=1e-6)
