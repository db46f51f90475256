"""CPU: pin the oracle against golden vectors produced by the reference's own XLA-path code
(tests/golden/make_golden.py), plus invariants that hold whatever the reference's rounding (lambda = 0,
identical branches, band vs dense, W8A8 integer exactness)."""
import numpy as np
import pytest

from conftest import load_golden
from oracle import band, cross, dense, w8a8
from oracle.common import bf16_bits_to_f32, check_close

DENSE = ["dense_h4_l200_full", "dense_h2_l130_partial", "dense_h2_l257_sharp"]
BAND = ["band_w17_l204_partial", "band_w128_l384_full", "band_w17_l136_sharp"]
CROSS = ["cross_h4_q200_kv128", "cross_h2_q130_kv257_sharp"]


def _band_norms(z):
    q = {"alpha": z["q_alpha"], "gamma": z["q_gamma"], "beta": z["q_beta"]}
    k = {"alpha": z["k_alpha"], "gamma": z["k_gamma"], "beta": z["k_beta"]}
    return q, k


@pytest.mark.parametrize("name", DENSE)
def test_dense_oracle_matches_reference(name):
    z = load_golden(name)
    qkv = bf16_bits_to_f32(z["qkv_bits"])
    args = (qkv, z["q_weight"], z["k_weight"], z["inv_freq"], z["valid"], int(z["heads"]), float(z["eps"]))
    out = dense.dense_diff_attention(*args)
    check_close(out, z["out_ref"], max_abs=1e-5, mean_abs=1e-6)
    a, b = dense.dense_branches(*args)
    check_close(dense.merge_heads(a), z["branch_a"], max_abs=1e-5, mean_abs=1e-6)
    check_close(dense.merge_heads(b), z["branch_b"], max_abs=1e-5, mean_abs=1e-6)
    # lambda: A - lambda * B against the reference's own branches
    lam = z["lam"]
    ref = z["branch_a"] - np.repeat(lam, 128)[None, None, :] * z["branch_b"]
    check_close(dense.dense_diff_attention(*args, lam=lam), ref, max_abs=1e-5, mean_abs=1e-6)


@pytest.mark.parametrize("name", CROSS)
def test_cross_oracle_matches_reference(name):
    z = load_golden(name)
    args = (bf16_bits_to_f32(z["q_bits"]), bf16_bits_to_f32(z["kv_bits"]), z["q_weight"], z["k_weight"],
            int(z["heads"]), float(z["eps"]))
    check_close(cross.cross_diff_attention(*args), z["out_ref"], max_abs=1e-5, mean_abs=1e-6)
    a, b = cross.cross_branches(*args)
    check_close(dense.merge_heads(a), z["branch_a"], max_abs=1e-5, mean_abs=1e-6)
    check_close(dense.merge_heads(b), z["branch_b"], max_abs=1e-5, mean_abs=1e-6)
    lam = z["lam"]
    ref = z["branch_a"] - np.repeat(lam, 128)[None, None, :] * z["branch_b"]
    check_close(cross.cross_diff_attention(*args, lam=lam), ref, max_abs=1e-5, mean_abs=1e-6)


def test_cross_oracle_hoisted_keys_and_invariants():
    """Pre-normed keys with k_weight=None give the same result; lambda = 0 is branch A; identical branches
    cancel exactly."""
    z = load_golden("cross_h4_q200_kv128")
    q2, kv = bf16_bits_to_f32(z["q_bits"]), bf16_bits_to_f32(z["kv_bits"]).astype(np.float64)
    args = (z["q_weight"], z["k_weight"], 4, 1e-6)
    full = cross.cross_diff_attention(q2, kv, *args)
    k, kd, v = np.split(kv, 3, axis=-1)
    normed = [dense.merge_heads(dense.rms_norm(t.reshape(2, 128, 4, 64).transpose(0, 2, 1, 3), z["k_weight"], 1e-6))
              for t in (k, kd)]
    hoisted = np.concatenate([*normed, v], -1)
    check_close(cross.cross_diff_attention(q2, hoisted, z["q_weight"], None, 4), full, max_abs=1e-6, mean_abs=1e-7)
    check_close(cross.cross_diff_attention(q2, kv, *args, lam=np.zeros(2, np.float32)), z["branch_a"],
                max_abs=1e-5, mean_abs=1e-6)
    qs, kvs = np.split(q2, 2, axis=-1), np.split(kv, 3, axis=-1)
    same = cross.cross_diff_attention(np.concatenate([qs[0], qs[0]], -1), np.concatenate([kvs[0], kvs[0], kvs[2]], -1),
                                      *args)
    assert np.abs(same).max() == 0.0


@pytest.mark.parametrize("name", BAND)
def test_band_oracle_matches_reference(name):
    z = load_golden(name)
    qkv = bf16_bits_to_f32(z["qkv_bits"])
    qn, kn = _band_norms(z)
    args = (qkv, qn, kn, z["inv_freq"], int(z["heads"]), int(z["window"]))
    check_close(band.band_diff_attention(*args), z["out_ref"], max_abs=1e-5, mean_abs=1e-6)
    a, b = band.band_branches(*args)
    check_close(dense.merge_heads(a), z["branch_a"], max_abs=1e-5, mean_abs=1e-6)
    lam = z["lam"]
    ref = z["branch_a"] - np.repeat(lam, 128)[None, None, :] * z["branch_b"]
    check_close(band.band_diff_attention(*args, lam=lam), ref, max_abs=1e-5, mean_abs=1e-6)


def test_dense_invariants():
    z = load_golden("dense_h2_l130_partial")
    qkv = bf16_bits_to_f32(z["qkv_bits"]).copy()
    args = (z["q_weight"], z["k_weight"], z["inv_freq"], z["valid"], 2, 1e-6)
    # lambda = 0 is plain attention on branch A
    out0 = dense.dense_diff_attention(qkv, *args, lam=np.zeros(1, np.float32))
    check_close(out0, z["branch_a"], max_abs=1e-5, mean_abs=1e-6)
    # identical branches with lambda = 1 cancel exactly
    sec = np.split(qkv, 5, axis=-1)
    same = np.concatenate([sec[0], sec[1], sec[2], sec[0], sec[1]], -1)
    assert np.abs(dense.dense_diff_attention(same, *args)).max() == 0.0


def test_band_window_covering_everything_is_dense_attention():
    z = load_golden("band_w17_l136_sharp")
    qkv = bf16_bits_to_f32(z["qkv_bits"])
    qn, kn = _band_norms(z)
    wide = band.band_diff_attention(qkv, qn, kn, z["inv_freq"], 2, window=10_000)
    a, b = band.band_branches(qkv, qn, kn, z["inv_freq"], 2, window=10_000)
    q, k, v, qd, kd = dense.split_heads(qkv, 2)
    cos, sin = dense.rope_cos_sin(qkv.shape[1], z["inv_freq"])
    full_a = dense.softmax_attend(dense.apply_rope(band.dyt(q, qn), cos, sin),
                                  dense.apply_rope(band.dyt(k, kn), cos, sin), v)
    check_close(dense.merge_heads(a), dense.merge_heads(full_a), max_abs=1e-9, mean_abs=1e-10)
    assert wide.shape == (1, 136, 128)


def test_w8a8_oracle_matches_integer_golden():
    z = load_golden("w8a8_m9_k96_n12")
    y, acc, qx, sx = w8a8.w8a8_linear(z["x_bits"], z["qw"], z["sw"], z["bias_bits"])
    assert np.array_equal(qx, z["qx"]) and np.array_equal(sx, z["sx"])
    assert np.array_equal(acc, z["acc"])
    assert np.array_equal(y, z["y_bits"])
    qw, sw = w8a8.quantize_rows(bf16_bits_to_f32(z["w_bits"]))
    assert np.array_equal(qw, z["qw"]) and np.array_equal(sw, z["sw"])


def test_quantize_rounding_rules():
    x = np.array([[127.0, 2.5, -3.5, 0.5, -0.5, 1.5, 126.5, -127.0],
                  [0, 0, 0, 0, 0, 0, 0, 0]], np.float32)
    q, s = w8a8.quantize_rows(x)
    assert s[0] == 1.0 and s[1] == 1.0
    assert q[0].tolist() == [127, 2, -4, 0, 0, 2, 126, -127]
    assert q[1].tolist() == [0] * 8


def _block_args(z):
    p = {k[2:]: bf16_bits_to_f32(v) for k, v in z.items() if k.startswith("p_")}
    h = bf16_bits_to_f32(z["h_bits"])
    valid = np.ones(h.shape[:2], np.float32)
    return (h, p, bf16_bits_to_f32(z["gcond_bits"]), z["kv_normed"], z["inv_freq"], valid), \
        dict(num_heads=int(z["heads"]), memory=int(z["memory"]), norm_eps=float(z["norm_eps"]),
             qk_eps=float(z["qk_eps"]))


def test_dit_block_oracle_matches_reference():
    """`oracle.dit_block` against the reference's own `dit._block` (dit.py:224-250) on random weights."""
    from oracle.dit_block import dit_block
    z = load_golden("dit_block_d256_l136")
    args, kw = _block_args(z)
    out = dit_block(*args, **kw)
    check_close(out, z["out_ref"], max_abs=1e-4, mean_abs=1e-5)


@pytest.mark.parametrize("mistake", ["gate_without_one_minus", "local_on_memory_rows", "no_adaln_shift"])
def test_dit_block_fixture_catches_order_mistakes(mistake, monkeypatch):
    """Each of these slips in the block's composition moves the output, on the memory rows or on the latent rows,
    by more than 3x the bf16 tolerance the GPU test of the composed block uses per row group, so that test would
    catch it. The mistakes are planted in the oracle, on the CPU."""
    from gpu_util import BLOCK_REL_TOL, block_rel_errors
    from oracle import dit_block as ob
    z = load_golden("dit_block_d256_l136")
    args, kw = _block_args(z)
    h, p, gcond, kv, freqs, valid = args
    if mistake == "gate_without_one_minus":
        monkeypatch.setattr(ob, "_sigmoid", lambda x: 1.0 / (1.0 + np.exp(x - 1.0)))  # sigmoid(gate), not of 1 - gate
    elif mistake == "local_on_memory_rows":
        kw = dict(kw, memory=0)
    else:
        gcond = gcond.copy()
        gcond[:, 256:512] = -p["to_scale_shift_gate"][256:512]  # cancels shift_self: x * (1 + scale) only
    out = ob.dit_block(h, p, gcond, kv, freqs, valid, **kw)
    worst = max(block_rel_errors(out, z["out_ref"], int(z["memory"])))
    assert worst > 3 * BLOCK_REL_TOL, f"{mistake}: relative change {worst:.3e} too small to be caught"
