"""GPU parity: the sm_100a band differential attention (through the C ABI) against the reference's golden
vectors and the fp32 oracle, including sequence shards with halos and the benchmark's full length."""
import numpy as np
import pytest
import torch

from conftest import load_golden
from gpu_util import bf16_cuda, check_attn, f32_cuda, fp32_tolerance, to_np
from oracle import band as oband
from oracle.common import bf16_bits_to_f32

BAND = ["band_w17_l204_partial", "band_w128_l384_full", "band_w17_l136_sharp"]
pytestmark = pytest.mark.gpu


def _norms(z):
    return ({"alpha": z["q_alpha"], "gamma": z["q_gamma"], "beta": z["q_beta"]},
            {"alpha": z["k_alpha"], "gamma": z["k_gamma"], "beta": z["k_beta"]})


@pytest.mark.parametrize("name", BAND)
def test_band_matches_reference_golden(name, cuda_lib):
    from hummingbird_b200.band_attention import band_attention
    z = load_golden(name)
    qn, kn = _norms(z)
    qkv = bf16_cuda(z["qkv_bits"])
    args = (bf16_bits_to_f32(z["qkv_bits"]), qn, kn, z["inv_freq"], int(z["heads"]), int(z["window"]))
    for lam, golden in ((None, z["out_ref"]),
                        (z["lam"], z["branch_a"] - np.repeat(z["lam"], 128)[None, None, :] * z["branch_b"])):
        out = to_np(band_attention(qkv, qn, kn, f32_cuda(z["inv_freq"]), int(z["heads"]), 64, int(z["window"]),
                                   lam=None if lam is None else f32_cuda(lam)))
        fused = oband.band_diff_attention(*args, lam=lam, fused_casts=True)
        check_attn(out, fused)
        check_attn(out, golden, *fp32_tolerance(fused, golden))


@pytest.mark.parametrize("window", [0, 17, 128, 300])
def test_band_windows_and_ragged_length(window, cuda_lib):
    from hummingbird_b200.band_attention import band_attention
    from hummingbird_b200.workloads import band_inputs
    w = band_inputs("cuda", seed=7, length=1000, d_model=256, heads=4, window=window)
    out = band_attention(w.qkv, w.q_norm, w.k_norm, f32_cuda(w.inv_freq), w.heads, 64, window, lam=f32_cuda(w.lam))
    ref = oband.band_diff_attention(to_np(w.qkv), w.q_norm, w.k_norm, w.inv_freq, w.heads, window, lam=w.lam)
    check_attn(to_np(out), ref)


@pytest.mark.parametrize("shards", [2, 3])
def test_band_sequence_shards_with_halo(shards, cuda_lib):
    """Each shard sees its rows plus `window` halo rows each side (what the NCCL halo exchange delivers);
    the concatenated shard outputs must match the unsharded oracle."""
    from hummingbird_b200.band_attention import band_attention_shard
    from hummingbird_b200.workloads import band_inputs
    window, length = 128, 1100
    w = band_inputs("cuda", seed=8, length=length, d_model=256, heads=4, window=window)
    ref = oband.band_diff_attention(to_np(w.qkv), w.q_norm, w.k_norm, w.inv_freq, w.heads, window, lam=w.lam)
    bounds = np.linspace(0, length, shards + 1).astype(int)
    parts = []
    for s0, s1 in zip(bounds[:-1], bounds[1:]):
        lo, hi = max(0, s0 - window), min(length, s1 + window)
        buf = w.qkv[:, lo:hi].contiguous()
        parts.append(to_np(band_attention_shard(buf, w.q_norm, w.k_norm, f32_cuda(w.inv_freq), w.heads, 64, window,
                                                q_begin=s0 - lo, q_count=s1 - s0, pos0=lo, lam=f32_cuda(w.lam))))
    check_attn(np.concatenate(parts, axis=1), ref)


def test_band_config2_full_length(cuda_lib):
    """Config 2 at full size (L=82,688, 8 heads, window 128) against the oracle on sampled query blocks."""
    from hummingbird_b200.band_attention import band_attention
    from hummingbird_b200.workloads import band_inputs
    w = band_inputs("cuda")
    out = to_np(band_attention(w.qkv, w.q_norm, w.k_norm, f32_cuda(w.inv_freq), w.heads, 64, w.window,
                               lam=f32_cuda(w.lam)))
    qkv = to_np(w.qkv)
    rng = np.random.default_rng(0)
    starts = sorted({0, qkv.shape[1] - 384, *rng.integers(0, qkv.shape[1] - 384, 6).tolist()})
    for s in starts:
        lo, hi = max(0, s - w.window), min(qkv.shape[1], s + 384 + w.window)
        ref = oband.band_diff_attention(qkv[:, lo:hi], w.q_norm, w.k_norm, w.inv_freq, w.heads, w.window, lam=w.lam,
                                        offset=lo)
        check_attn(out[:, s:s + 384], ref[:, s - lo:s - lo + 384])


def test_band_config5_length(cuda_lib):
    """Config 5's decoder length (L=261,888, the 380 s song; 8 heads, window 128) against the oracle on sampled
    query blocks, the last block included. RoPE angles reach fp32(261,887) * inv_freq here, so this checks the
    angle reduction far beyond config 2's positions. Only the sampled rows are copied to the host."""
    from hummingbird_b200.band_attention import band_attention
    from hummingbird_b200.workloads import band_inputs
    w = band_inputs("cuda", length=261_888)
    out = band_attention(w.qkv, w.q_norm, w.k_norm, f32_cuda(w.inv_freq), w.heads, 64, w.window, lam=f32_cuda(w.lam))
    length = w.qkv.shape[1]
    rng = np.random.default_rng(5)
    starts = sorted({0, length // 2, length - 384, *rng.integers(200_000, length - 384, 3).tolist()})
    for s in starts:
        lo, hi = max(0, s - w.window), min(length, s + 384 + w.window)
        ref = oband.band_diff_attention(to_np(w.qkv[:, lo:hi]), w.q_norm, w.k_norm, w.inv_freq, w.heads, w.window,
                                        lam=w.lam, offset=lo)
        check_attn(to_np(out[:, s:s + 384]), ref[:, s - lo:s - lo + 384])


def test_band_from_host_streamed_equals_device_call(cuda_lib):
    """The host-streamed API (chunks of rows copied in, computed, copied out on overlapping streams) gives
    the same bits as one device call, for B=2 and a chunk size that does not divide the length."""
    from hummingbird_b200 import band_attention as hb
    from hummingbird_b200.workloads import band_inputs
    w = band_inputs("cuda", seed=8, batch=2, length=3000, d_model=256, heads=4, window=128)
    freqs, lam = torch.from_numpy(w.inv_freq).cuda(), torch.from_numpy(w.lam).cuda()
    ref = hb.band_attention(w.qkv, w.q_norm, w.k_norm, freqs, w.heads, 64, w.window, lam=lam)
    host = w.qkv.cpu().pin_memory()
    out = hb.band_attention_from_host(host, w.q_norm, w.k_norm, freqs, w.heads, 64, w.window, lam=lam,
                                      chunk_rows=700)
    torch.cuda.synchronize()
    assert torch.equal(out, ref.cpu())
