"""GPU parity: the sm_100a dense differential attention (through the C ABI) against the reference's golden
vectors and the fp32 oracle. Tolerance: max-abs 2e-2, mean-abs 2e-3 (the attention tolerance), plus the bf16 rounding
of outputs larger than 1."""
import numpy as np
import pytest
import torch

from conftest import load_golden
from gpu_util import bf16_cuda, check_attn, f32_cuda, fp32_tolerance, to_np
from oracle import dense as odense
from oracle.common import bf16_bits_to_f32

DENSE = ["dense_h4_l200_full", "dense_h2_l130_partial", "dense_h2_l257_sharp"]
pytestmark = pytest.mark.gpu


def _run(z, lam=None, **kw):
    from hummingbird_b200 import dense_attention as hb
    qkv = bf16_cuda(z["qkv_bits"])
    length = qkv.shape[1]
    cos, sin, mask = hb.tables(length, f32_cuda(z["inv_freq"]), f32_cuda(z["valid"]))
    out = hb.dense_attention(qkv, f32_cuda(z["q_weight"]), f32_cuda(z["k_weight"]), cos, sin, mask,
                             int(z["heads"]), 64, int(z["half"]), float(z["eps"]),
                             lam=None if lam is None else f32_cuda(lam), **kw)
    torch.cuda.synchronize()
    return to_np(out)


@pytest.mark.parametrize("name", DENSE)
def test_dense_matches_reference_golden(name, cuda_lib):
    """Against the reference's fp32 XLA output (golden) and the fused kernel's cast points (oracle)."""
    z = load_golden(name)
    args = (bf16_bits_to_f32(z["qkv_bits"]), z["q_weight"], z["k_weight"], z["inv_freq"], z["valid"],
            int(z["heads"]), float(z["eps"]))
    for lam, golden in ((None, z["out_ref"]),
                        (z["lam"], z["branch_a"] - np.repeat(z["lam"], 128)[None, None, :] * z["branch_b"])):
        out = _run(z, lam=lam)
        fused = odense.dense_diff_attention(*args, lam=lam, fused_casts=True)
        check_attn(out, fused)
        check_attn(out, golden, *fp32_tolerance(fused, golden))


def test_dense_lambda_zero_is_branch_a(cuda_lib):
    z = load_golden("dense_h2_l130_partial")
    check_attn(_run(z, lam=np.zeros(1, np.float32)), z["branch_a"])


def test_dense_identical_branches_cancel(cuda_lib):
    z = dict(load_golden("dense_h4_l200_full"))
    bits = z["qkv_bits"].reshape(2, 200, 5, 256)
    bits[:, :, 3] = bits[:, :, 0]
    bits[:, :, 4] = bits[:, :, 1]
    z["qkv_bits"] = bits.reshape(2, 200, 1280)
    assert np.abs(_run(z)).max() == 0.0


def test_dense_tables_without_16_byte_alignment(cuda_lib):
    """Lane tables whose rows are not 16-byte aligned take the prologue's scalar-load path: same bits."""
    from hummingbird_b200 import dense_attention as hb
    z = load_golden("dense_h4_l200_full")
    qkv = bf16_cuda(z["qkv_bits"])
    cos, sin, mask = hb.tables(200, f32_cuda(z["inv_freq"]), f32_cuda(z["valid"]))
    args = (f32_cuda(z["q_weight"]), f32_cuda(z["k_weight"]))
    ref = hb.dense_attention(qkv, *args, cos, sin, mask, 4, 64, 32, float(z["eps"]))
    pad_c = torch.zeros(200, 129, device="cuda")
    pad_s = torch.zeros(200, 129, device="cuda")
    pad_c[:, 1:], pad_s[:, 1:] = cos, sin
    out = hb.dense_attention(qkv, *args, pad_c[:, 1:], pad_s[:, 1:], mask, 4, 64, 32, float(z["eps"]))
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


def test_dense_pair_sharding_matches_full(cuda_lib):
    z = load_golden("dense_h4_l200_full")
    full = _run(z, lam=z["lam"])
    part = _run(z, lam=z["lam"], pair_begin=1, pair_count=1)
    assert np.array_equal(part, full[..., 128:256])


def test_dense_config1_against_oracle(cuda_lib):
    from hummingbird_b200.workloads import dense_inputs
    from hummingbird_b200 import dense_attention as hb
    w = dense_inputs("cuda")
    cos, sin, mask = hb.tables(646, f32_cuda(w.inv_freq), f32_cuda(w.valid))
    out = hb.dense_attention(w.qkv, f32_cuda(w.q_weight), f32_cuda(w.k_weight), cos, sin, mask, w.heads, 64,
                             w.half, w.eps, lam=f32_cuda(w.lam))
    ref = odense.dense_diff_attention(to_np(w.qkv), w.q_weight, w.k_weight, w.inv_freq, w.valid, w.heads,
                                      w.eps, lam=w.lam)
    check_attn(to_np(out), ref)


def test_dense_long_sequence_against_oracle(cuda_lib):
    """B=2, L=2648 (the 120 s DiT self-attention length) on 4 heads: many key tiles, ragged tail."""
    from hummingbird_b200.workloads import dense_inputs
    from hummingbird_b200 import dense_attention as hb
    w = dense_inputs("cuda", seed=5, batch=2, length=2648, d_model=256, heads=4, masked_tail=100)
    cos, sin, mask = hb.tables(2648, f32_cuda(w.inv_freq), f32_cuda(w.valid))
    out = hb.dense_attention(w.qkv, f32_cuda(w.q_weight), f32_cuda(w.k_weight), cos, sin, mask, w.heads, 64,
                             w.half, w.eps, lam=f32_cuda(w.lam))
    ref = odense.dense_diff_attention(to_np(w.qkv), w.q_weight, w.k_weight, w.inv_freq, w.valid, w.heads,
                                      w.eps, lam=w.lam)
    check_attn(to_np(out), ref)


def test_dense_380s_length_against_oracle_on_sampled_rows(cuda_lib):
    """B=2, L=8,248 (the 380 s DiT self-attention length: 65 key tiles, ragged tail), 4 heads, lambda; the
    oracle on sampled query rows (first and last tiles, a middle block) against every key."""
    from hummingbird_b200.workloads import dense_inputs
    from hummingbird_b200 import dense_attention as hb
    length = 8248
    w = dense_inputs("cuda", seed=6, batch=2, length=length, d_model=256, heads=4, masked_tail=64)
    cos, sin, mask = hb.tables(length, f32_cuda(w.inv_freq), f32_cuda(w.valid))
    out = to_np(hb.dense_attention(w.qkv, f32_cuda(w.q_weight), f32_cuda(w.k_weight), cos, sin, mask, w.heads, 64,
                                   w.half, w.eps, lam=f32_cuda(w.lam)))
    assert np.isfinite(out).all()
    rows = np.r_[0:64, 4100:4164, length - 72:length]
    ref = odense.dense_diff_attention(to_np(w.qkv), w.q_weight, w.k_weight, w.inv_freq, w.valid, w.heads, w.eps,
                                      lam=w.lam, queries=rows)
    check_attn(out[:, rows], ref)


def test_dense_rejects_bad_shapes(cuda_lib):
    from hummingbird_b200 import dense_attention as hb
    qkv = torch.zeros(1, 8, 5 * 4 * 64, dtype=torch.bfloat16, device="cuda")
    cos = torch.ones(8, 128, device="cuda")
    mask = torch.ones(1, 8, dtype=torch.bfloat16, device="cuda")
    w = torch.ones(64, device="cuda")
    with pytest.raises(ValueError):
        hb.dense_attention(qkv, w, w, cos, cos, mask, 4, 64, 12, 1e-6)  # half not a multiple of 8
    with pytest.raises(ValueError):
        hb.dense_attention(qkv, w, w, cos, cos, mask, 4, 32, 16, 1e-6)  # head_dim 32
