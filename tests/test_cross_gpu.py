"""GPU parity: the sm_100a differential cross-attention (through the C ABI) against golden vectors made by the
reference's own `_cross_attention` and against the fp32 oracle. Tolerance: max-abs 2e-2, mean-abs 2e-3 (the
attention tolerance), plus the bf16 rounding of outputs larger than 1."""
import numpy as np
import pytest
import torch

from conftest import load_golden
from gpu_util import bf16_cuda, check_attn, f32_cuda, fp32_tolerance, to_np
from oracle import cross as ocross
from oracle.common import bf16_bits_to_f32

CROSS = ["cross_h4_q200_kv128", "cross_h2_q130_kv257_sharp"]
pytestmark = pytest.mark.gpu


def _inputs(seed, batch, q_len, kv_len, heads, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    q2 = (scale * torch.randn(batch, q_len, 2 * heads * 64, generator=g)).to(torch.bfloat16)
    kv = torch.randn(batch, kv_len, 3 * heads * 64, generator=g).to(torch.bfloat16)
    q_w = 1 + 0.02 * torch.randn(64, generator=g)
    k_w = 1 + 0.02 * torch.randn(64, generator=g)
    return q2, kv, q_w, k_w


def _run(q2, kv, q_w, k_w, heads, lam=None, eps=1e-6):
    from hummingbird_b200.cross_attention import cross_attention
    out = cross_attention(q2.cuda(), kv.cuda(), q_w.cuda(), None if k_w is None else k_w.cuda(), heads, 64, eps,
                          lam=None if lam is None else f32_cuda(lam))
    torch.cuda.synchronize()
    return to_np(out)


def _np(t):
    return t.float().numpy()


@pytest.mark.parametrize("name", CROSS)
def test_cross_matches_reference_golden(name, cuda_lib):
    """Against the reference's fp32 XLA output (golden) and the fused kernels' cast points (oracle)."""
    z = load_golden(name)
    heads = int(z["heads"])
    q2, kv = bf16_cuda(z["q_bits"]), bf16_cuda(z["kv_bits"])
    args = (bf16_bits_to_f32(z["q_bits"]), bf16_bits_to_f32(z["kv_bits"]), z["q_weight"], z["k_weight"], heads,
            float(z["eps"]))
    for lam, golden in ((None, z["out_ref"]),
                        (z["lam"], z["branch_a"] - np.repeat(z["lam"], 128)[None, None, :] * z["branch_b"])):
        out = _run(q2, kv, torch.from_numpy(z["q_weight"]), torch.from_numpy(z["k_weight"]), heads, lam=lam)
        fused = ocross.cross_diff_attention(*args, lam=lam, fused_casts=True)
        check_attn(out, fused)
        check_attn(out, golden, *fp32_tolerance(fused, golden))


def test_cross_lambda_zero_is_branch_a(cuda_lib):
    z = load_golden("cross_h4_q200_kv128")
    out = _run(bf16_cuda(z["q_bits"]), bf16_cuda(z["kv_bits"]), torch.from_numpy(z["q_weight"]),
               torch.from_numpy(z["k_weight"]), 4, lam=np.zeros(2, np.float32))
    check_attn(out, z["branch_a"])


def test_cross_identical_branches_cancel(cuda_lib):
    q2, kv, q_w, k_w = _inputs(1, 2, 300, 128, 2)
    q2[..., 128:] = q2[..., :128]
    kv[..., 128:256] = kv[..., :128]
    assert np.abs(_run(q2, kv, q_w, k_w, 2)).max() == 0.0


def test_cross_hoisted_keys_match_raw_keys(cuda_lib):
    """`cross_kv` (k-norm hoisted once, as the reference's `_cross_kv`) + k_weight=None against the oracle."""
    from hummingbird_b200.cross_attention import cross_kv
    q2, kv, q_w, k_w = _inputs(2, 2, 260, 128, 4)
    hoisted = cross_kv(kv.cuda(), k_w.cuda(), 4, 1e-6)
    out = _run(q2, hoisted.cpu(), q_w, None, 4)
    ref = ocross.cross_diff_attention(_np(q2), _np(kv), _np(q_w), _np(k_w), 4)
    check_attn(out, ref)
    check_attn(out, _run(q2, kv, q_w, k_w, 4))


@pytest.mark.parametrize("batch,q_len,kv_len,heads", [
    (1, 1, 1, 1),        # one query, one key, odd head count
    (3, 129, 127, 3),    # ragged query tile, partial key tile
    (1, 77, 384, 2),     # the longest context: three full key tiles
    (2, 40, 257, 2),     # the reference's 257-token conditioning: a key tile with one key
])
def test_cross_ragged_shapes(batch, q_len, kv_len, heads, cuda_lib):
    q2, kv, q_w, k_w = _inputs(3 + q_len, batch, q_len, kv_len, heads)
    ref = ocross.cross_diff_attention(_np(q2), _np(kv), _np(q_w), _np(k_w), heads)
    check_attn(_run(q2, kv, q_w, k_w, heads), ref)


def test_cross_dit_shape_against_oracle(cuda_lib):
    """The 120 s DiT's cross-attention: B=2, 2,648 queries, 16 heads, 128 context tokens (672 units over the
    SMs, several (batch, head) runs per CTA)."""
    q2, kv, q_w, k_w = _inputs(4, 2, 2648, 128, 16)
    lam = np.random.default_rng(4).uniform(0.2, 0.8, 8).astype(np.float32)
    ref = ocross.cross_diff_attention(_np(q2), _np(kv), _np(q_w), _np(k_w), 16, lam=lam)
    check_attn(_run(q2, kv, q_w, k_w, 16, lam=lam), ref)


def test_cross_long_context_many_runs(cuda_lib):
    """Three key tiles resident per run and run changes inside a CTA's unit range (320 units)."""
    q2, kv, q_w, k_w = _inputs(5, 1, 5000, 300, 8)
    ref = ocross.cross_diff_attention(_np(q2), _np(kv), _np(q_w), _np(k_w), 8)
    check_attn(_run(q2, kv, q_w, k_w, 8), ref)


def test_cross_rejects_unsupported_shapes(cuda_lib):
    from hummingbird_b200 import _lib
    from hummingbird_b200.cross_attention import cross_attention
    q2, kv, q_w, k_w = _inputs(6, 1, 16, 385, 2)
    with pytest.raises(ValueError):
        cross_attention(q2.cuda(), kv.cuda(), q_w.cuda(), k_w.cuda(), 2)
    with pytest.raises(ValueError):
        cross_attention(q2.cuda(), kv[:, :8].cuda(), q_w.cuda(), k_w.cuda(), 2, head_dim=128)
    q, kvd, qw = q2.cuda(), kv.cuda(), q_w.cuda()
    out = torch.empty(1, 16, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):  # the C ABI itself refuses more than 384 context tokens (HB_ERR_SHAPE)
        _lib.call("hb_cross_diff_attn", q.data_ptr(), q.stride(1), kvd.data_ptr(), kvd.stride(1), qw.data_ptr(),
                  None, None, out.data_ptr(), 128, 1, 16, 385, 2, 64, 1e-6, 0)
    with pytest.raises(_lib.HbError):  # misaligned row stride (HB_ERR_ALIGN)
        _lib.call("hb_cross_diff_attn", q.data_ptr(), 260, kvd.data_ptr(), kvd.stride(1), qw.data_ptr(),
                  None, None, out.data_ptr(), 128, 1, 16, 8, 2, 64, 1e-6, 0)
