"""Generate the golden vectors in `tests/golden/*.npz` by running the REFERENCE's own code.

JAX is not installable here, so `tests/golden/_jaxshim/jax` (a numpy stand-in for the few JAX calls on
the reference's XLA path) is put on `sys.path` and the reference package `sa3jax` is imported from the
reference checkout named by `$HB_REFERENCE` (required). The reference then runs in fp32
(`dtypes.FP32_PARITY`) through its own functions:

* dense: `sa3jax.dit._self_attention` (dit.py:185-200) with `DiTConfig(attention="xla", differential=True)`,
  identity `to_qkv` / `to_out` so the fixture holds exactly the kernel boundary `qkv -> merged out`;
  branches A and B separately through the same function with `differential=False` on `[q|k|v]` and
  `[q_diff|k_diff|v]`.
* band: `sa3jax.same_l._attention` (same_l.py:151-169) with `SameConfig(attention="xla")`,
  `stride = window - 1`, mask from `same_l._swa_mask`; branches A and B through `same_l._rope`,
  `_dyt` and `_sdpa` composed as `_attention` composes them (same_l.py:162-168).
* cross: `sa3jax.dit._cross_attention` (dit.py:203-215) over keys hoisted by `sa3jax.dit._cross_kv`
  (dit.py:274-284), identity `to_q` / `to_kv` / `to_out`; branches A and B with `differential=False`.
* w8a8: no reference exists; the accumulators come from a pure-Python integer dot product, independent
  of the numpy oracle.
* dit block: `sa3jax.dit._block` (dit.py:224-250) on one block with random weights, cross K/V from
  `sa3jax.dit._cross_kv` (dit.py:274-284).

Run from the repo root:  HB_REFERENCE=<path of a hummingbird checkout> python tests/golden/make_golden.py
This script (and only this script) reads the reference; the fixtures it writes are what tests use.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]


def _import_reference():
    ref = os.environ.get("HB_REFERENCE")
    if not ref or not (Path(ref) / "sa3jax").is_dir():
        raise SystemExit("set HB_REFERENCE to a checkout of kelechi-c/hummingbird (the directory holding sa3jax/)")
    sys.path.insert(0, str(HERE / "_jaxshim"))
    sys.path.insert(0, ref)
    from sa3jax import config, dit, dtypes, same_l  # noqa: E402
    return config, dit, dtypes, same_l


def _bf16(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    sys.path.insert(0, str(ROOT))
    from oracle.common import bf16_bits_to_f32, f32_to_bf16_bits
    bits = f32_to_bf16_bits(np.asarray(x, np.float32))
    return bits, bf16_bits_to_f32(bits)


def _inv_freq(half: int) -> np.ndarray:
    rot = 2 * half
    return (1.0 / (10000.0 ** (np.arange(0, rot, 2, dtype=np.float64) / rot))).astype(np.float32)


def dense_case(name, *, seed, batch, length, heads, half, w_scale=1.0, masked_tail=0):
    config, dit, dtypes, _ = _import_reference()
    rng = np.random.default_rng(seed)
    qkv_bits, qkv = _bf16(rng.standard_normal((batch, length, 5 * heads * 64)))
    q_w = (w_scale + 0.02 * rng.standard_normal(64)).astype(np.float32)
    k_w = (w_scale + 0.02 * rng.standard_normal(64)).astype(np.float32)
    lam = rng.uniform(0.2, 0.8, heads // 2).astype(np.float32)
    freqs = _inv_freq(half)
    valid = np.ones((batch, length), np.float32)
    if masked_tail:
        valid[0, length - masked_tail:] = 0.0
    f32 = dtypes.FP32_PARITY
    inner = heads * 64

    def run(x, differential):
        width = x.shape[-1]
        cfg = config.DiTConfig(embed_dim=inner, num_heads=heads, differential=differential, attention="xla")
        block = {"self_attn": {"to_qkv": {"weight": np.eye(width, dtype=np.float32)},
                               "q_norm": {"weight": q_w}, "k_norm": {"weight": k_w},
                               "to_out": {"weight": np.eye(inner, dtype=np.float32)}}}
        cos, sin = dit._rope_tables(length, freqs)
        static = {"cos": cos, "sin": sin, "v_mask": valid[:, None, :, None]}
        return dit._self_attention(x.astype(np.float32), block, static, cfg, f32)

    out = run(qkv, True)
    sec = np.split(qkv, 5, axis=-1)
    branch_a = run(np.concatenate([sec[0], sec[1], sec[2]], -1), False)
    branch_b = run(np.concatenate([sec[3], sec[4], sec[2]], -1), False)
    np.savez_compressed(HERE / f"{name}.npz", qkv_bits=qkv_bits, q_weight=q_w, k_weight=k_w, inv_freq=freqs,
                        valid=valid, lam=lam, heads=heads, half=half, eps=np.float32(1e-6),
                        out_ref=out.astype(np.float32), branch_a=branch_a.astype(np.float32),
                        branch_b=branch_b.astype(np.float32))
    print(f"{name}: out absmax {np.abs(out).max():.4f}")


def cross_case(name, *, seed, batch, q_len, kv_len, heads, w_scale=1.0):
    """`sa3jax.dit._cross_attention` (dit.py:203-215) on K/V hoisted by `sa3jax.dit._cross_kv` (dit.py:274-284),
    identity `to_q` / `to_kv` / `to_out`; branches A and B through the same function with `differential=False`."""
    config, dit, dtypes, _ = _import_reference()
    rng = np.random.default_rng(seed)
    inner = heads * 64
    q_bits, q2 = _bf16(rng.standard_normal((batch, q_len, 2 * inner)))
    kv_bits, kv = _bf16(rng.standard_normal((batch, kv_len, 3 * inner)))
    q_w = (w_scale + 0.02 * rng.standard_normal(64)).astype(np.float32)
    k_w = (w_scale + 0.02 * rng.standard_normal(64)).astype(np.float32)
    lam = rng.uniform(0.2, 0.8, heads // 2).astype(np.float32)
    f32 = dtypes.FP32_PARITY

    def run(q_in, kv_in, differential):
        cfg = config.DiTConfig(embed_dim=inner, num_heads=heads, differential=differential, attention="xla")
        block = {"cross_attn": {"to_q": {"weight": np.eye(q_in.shape[-1], dtype=np.float32)},
                                "to_kv": {"weight": np.eye(kv_in.shape[-1], dtype=np.float32)},
                                "q_norm": {"weight": q_w}, "k_norm": {"weight": k_w},
                                "to_out": {"weight": np.eye(inner, dtype=np.float32)}}}
        hoisted = dit._cross_kv(block, kv_in.astype(np.float32), cfg, f32)
        static = {"cross_k": [hoisted[0]], "cross_v": [hoisted[-1]]}
        if differential:
            static["cross_k_diff"] = [hoisted[1]]
        return dit._cross_attention(q_in.astype(np.float32), static, block, 0, cfg, f32)

    out = run(q2, kv, True)
    qs, kvs = np.split(q2, 2, axis=-1), np.split(kv, 3, axis=-1)
    branch_a = run(qs[0], np.concatenate([kvs[0], kvs[2]], -1), False)
    branch_b = run(qs[1], np.concatenate([kvs[1], kvs[2]], -1), False)
    np.savez_compressed(HERE / f"{name}.npz", q_bits=q_bits, kv_bits=kv_bits, q_weight=q_w, k_weight=k_w, lam=lam,
                        heads=heads, eps=np.float32(1e-6), out_ref=out.astype(np.float32),
                        branch_a=branch_a.astype(np.float32), branch_b=branch_b.astype(np.float32))
    print(f"{name}: out absmax {np.abs(out).max():.4f}")


def band_case(name, *, seed, batch, length, heads, half, window, alpha=0.5, gamma=1.0):
    config, _, dtypes, same_l = _import_reference()
    rng = np.random.default_rng(seed)
    qkv_bits, qkv = _bf16(rng.standard_normal((batch, length, 5 * heads * 64)))

    def norm():
        return {"alpha": np.array(alpha, np.float32),
                "gamma": (gamma + 0.02 * rng.standard_normal(64)).astype(np.float32),
                "beta": (0.02 * rng.standard_normal(64)).astype(np.float32)}

    q_norm, k_norm = norm(), norm()
    lam = rng.uniform(0.2, 0.8, heads // 2).astype(np.float32)
    freqs = _inv_freq(half)
    f32 = dtypes.FP32_PARITY
    inner = heads * 64
    cfg = config.SameConfig(channels=inner, c_mults=(1,), stride=window - 1, attention="xla")
    assert cfg.num_heads == heads and cfg.sub_chunk_size == window and length % window == 0
    mask = same_l._swa_mask(length // window, cfg)
    block = {"self_attn": {"to_qkv": {"weight": np.eye(5 * inner, dtype=np.float32)},
                           "q_norm": q_norm, "k_norm": k_norm,
                           "to_out": {"weight": np.eye(inner, dtype=np.float32)}},
             "rope_inv_freq": freqs}
    out = same_l._attention(qkv.astype(np.float32), block, mask, cfg, f32)
    # the two branches, composed from the same reference functions `_attention` uses (same_l.py:162-168)
    q, k, v, qd, kd = (same_l._heads(t, cfg) for t in np.split(qkv.astype(np.float32), 5, axis=-1))
    cos, sin = same_l._rope_tables(length, freqs, f32)
    rq = lambda t, n: same_l._rope(same_l._dyt(t, n), cos, sin, f32)  # noqa: E731
    branch_a = same_l._merge(same_l._sdpa(rq(q, q_norm), rq(k, k_norm), v, mask, cfg, f32))
    branch_b = same_l._merge(same_l._sdpa(rq(qd, q_norm), rq(kd, k_norm), v, mask, cfg, f32))
    np.savez_compressed(HERE / f"{name}.npz", qkv_bits=qkv_bits, inv_freq=freqs, lam=lam, heads=heads,
                        half=half, window=window,
                        q_alpha=q_norm["alpha"], q_gamma=q_norm["gamma"], q_beta=q_norm["beta"],
                        k_alpha=k_norm["alpha"], k_gamma=k_norm["gamma"], k_beta=k_norm["beta"],
                        out_ref=out.astype(np.float32), branch_a=branch_a.astype(np.float32),
                        branch_b=branch_b.astype(np.float32))
    print(f"{name}: out absmax {np.abs(out).max():.4f}")


def dit_block_case(name, *, seed, batch, latents, memory, context, heads):
    """`sa3jax.dit._block` (dit.py:224-250): one whole block (adaLN, self-attention, gated residuals, cross-attention
    over K/V hoisted by `sa3jax.dit._cross_kv`, `to_local_embed` on the non-memory rows, GLU MLP) with random,
    bf16-representable weights, `attention="xla"`, `differential=True`, under `FP32_PARITY`."""
    config, dit, dtypes, _ = _import_reference()
    rng = np.random.default_rng(seed)
    d = heads * 64
    cfg = config.DiTConfig(embed_dim=d, num_heads=heads, differential=True, attention="xla",
                           num_memory_tokens=memory)
    inner = cfg.ff_inner
    length = memory + latents

    def w(*shape, fan_in=None, scale=1.0):
        fan = fan_in or shape[-1]
        return _bf16(scale * rng.standard_normal(shape) / np.sqrt(fan))[1]

    def near_one(n):
        return _bf16(1.0 + 0.1 * rng.standard_normal(n))[1]

    p = {"to_scale_shift_gate": _bf16(0.3 * rng.standard_normal(6 * d))[1],
         "pre_norm": near_one(d), "cross_attend_norm": near_one(d), "ff_norm": near_one(d),
         "sa_to_qkv": w(5 * d, d), "sa_q_norm": near_one(64), "sa_k_norm": near_one(64), "sa_to_out": w(d, d),
         "ca_to_q": w(2 * d, d), "ca_to_kv": w(3 * d, d), "ca_q_norm": near_one(64), "ca_k_norm": near_one(64),
         "ca_to_out": w(d, d), "local": _bf16(0.2 * rng.standard_normal(d))[1],
         "glu_w": w(2 * inner, d), "glu_b": _bf16(0.05 * rng.standard_normal(2 * inner))[1],
         "proj_w": w(d, inner), "proj_b": _bf16(0.05 * rng.standard_normal(d))[1]}
    h_bits, h = _bf16(rng.standard_normal((batch, length, d)))
    ctx_bits, ctx = _bf16(rng.standard_normal((batch, context, d)))
    gcond_bits, gcond = _bf16(0.3 * rng.standard_normal((batch, 6 * d)))
    freqs = _inv_freq(cfg.rope_dim // 2)
    f32 = dtypes.FP32_PARITY
    block = {"to_scale_shift_gate": p["to_scale_shift_gate"],
             "pre_norm": {"weight": p["pre_norm"]}, "cross_attend_norm": {"weight": p["cross_attend_norm"]},
             "ff_norm": {"weight": p["ff_norm"]},
             "self_attn": {"to_qkv": {"weight": p["sa_to_qkv"]}, "q_norm": {"weight": p["sa_q_norm"]},
                           "k_norm": {"weight": p["sa_k_norm"]}, "to_out": {"weight": p["sa_to_out"]}},
             "cross_attn": {"to_q": {"weight": p["ca_to_q"]}, "to_kv": {"weight": p["ca_to_kv"]},
                            "q_norm": {"weight": p["ca_q_norm"]}, "k_norm": {"weight": p["ca_k_norm"]},
                            "to_out": {"weight": p["ca_to_out"]}},
             "ff": {"glu_proj": {"weight": p["glu_w"], "bias": p["glu_b"]},
                    "proj_out": {"weight": p["proj_w"], "bias": p["proj_b"]}}}
    k, kd, v = dit._cross_kv(block, ctx.astype(np.float32), cfg, f32)
    cos, sin = dit._rope_tables(length, freqs)
    valid = np.ones((batch, length), np.float32)
    static = {"cos": cos, "sin": sin, "v_mask": valid[:, None, :, None], "cross_k": [k], "cross_v": [v],
              "cross_k_diff": [kd], "local": [p["local"]]}
    import jax.numpy as jnp  # the numpy stand-in, on sys.path after _import_reference()
    out = dit._block(jnp.array_at(h.astype(np.float32)), block, static, gcond.astype(np.float32), 0, cfg, f32)
    out = np.asarray(out)
    merge = lambda t: np.asarray(t).transpose(0, 2, 1, 3).reshape(batch, context, d)  # noqa: E731
    kv_normed = np.concatenate([merge(k), merge(kd), merge(v)], -1).astype(np.float32)
    np.savez_compressed(HERE / f"{name}.npz", h_bits=h_bits, ctx_bits=ctx_bits, gcond_bits=gcond_bits,
                        inv_freq=freqs, heads=heads, memory=memory, norm_eps=np.float32(cfg.norm_eps),
                        qk_eps=np.float32(cfg.qk_norm_eps), kv_normed=kv_normed, out_ref=out.astype(np.float32),
                        **{f"p_{key}": _bf16(val)[0] for key, val in p.items()})  # bf16 bit patterns
    print(f"{name}: out absmax {np.abs(out).max():.4f}")


def w8a8_case(name, *, seed, m, k, n):
    """Integer accumulators by a pure-Python dot product (independent of numpy's int matmul)."""
    sys.path.insert(0, str(ROOT))
    from oracle.w8a8 import epilogue, quantize_rows
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k)).astype(np.float32)
    x[1] = 0.0  # an all-zero token: scale 1, q 0
    x[2, :4] = [127.0, 2.5, -3.5, 0.5]  # absmax 127 -> scale exactly 1: exercises round-half-to-even
    x[2, 4:] = 0.0
    x_bits, x = _bf16(x)
    w = (rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float32)
    w_bits, w = _bf16(w)
    bias_bits, _ = _bf16(0.1 * rng.standard_normal(n))
    qx, sx = quantize_rows(x)
    qw, sw = quantize_rows(w)
    assert list(qx[2, :4]) == [127, 2, -4, 0] and np.all(qx[1] == 0) and sx[1] == 1.0
    acc = np.array([[sum(int(a) * int(b) for a, b in zip(qx[i], qw[j])) for j in range(n)] for i in range(m)],
                   dtype=np.int32)
    y_bits = epilogue(acc, sx, sw, bias_bits)
    np.savez_compressed(HERE / f"{name}.npz", x_bits=x_bits, w_bits=w_bits, bias_bits=bias_bits, qx=qx, sx=sx,
                        qw=qw, sw=sw, acc=acc, y_bits=y_bits)
    print(f"{name}: acc absmax {np.abs(acc).max()}")


def main():
    dense_case("dense_h4_l200_full", seed=10, batch=2, length=200, heads=4, half=32, masked_tail=40)
    dense_case("dense_h2_l130_partial", seed=11, batch=1, length=130, heads=2, half=16)
    dense_case("dense_h2_l257_sharp", seed=12, batch=1, length=257, heads=2, half=32, w_scale=3.0)
    cross_case("cross_h4_q200_kv128", seed=40, batch=2, q_len=200, kv_len=128, heads=4)
    cross_case("cross_h2_q130_kv257_sharp", seed=41, batch=1, q_len=130, kv_len=257, heads=2, w_scale=3.0)
    band_case("band_w17_l204_partial", seed=20, batch=1, length=204, heads=4, half=16, window=17)
    band_case("band_w128_l384_full", seed=21, batch=1, length=384, heads=2, half=32, window=128)
    band_case("band_w17_l136_sharp", seed=22, batch=1, length=136, heads=2, half=16, window=17, alpha=1.5,
              gamma=4.0)
    w8a8_case("w8a8_m9_k96_n12", seed=30, m=9, k=96, n=12)
    dit_block_case("dit_block_d256_l136", seed=50, batch=2, latents=128, memory=8, context=16, heads=4)


if __name__ == "__main__":
    main()
