"""Fixed-shape calls of one hot-path kernel each, for profilers (`ncu -k <kernel> -s <skip> -c <count>`).

    python profile_cases.py band    # config 2: SAME-L band attention, B=1, L=82,688, 8 heads
    python profile_cases.py dense   # dense DiT self-attention, B=2, L=2,648, 16 heads
    python profile_cases.py cross   # DiT cross-attention, B=2, 2,648 queries, 128 context, 16 heads
    python profile_cases.py glue    # DiT row kernels: residual + RMSNorm + adaLN, GLU + int8
    python profile_cases.py band_front [--rows R]  # SAME-L front end (block DyT + to_qkv + q/k DyT + RoPE) and
                                                   # the band kernel on its output; config 2 at R = 82,688 rows

Each case builds its seeded synthetic inputs (`hummingbird_b200.workloads`), makes `--calls` calls (default 3)
on the current GPU and prints a checksum of the last output. Nothing is timed here: the bench times.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))


def band(calls: int) -> torch.Tensor:
    from hummingbird_b200.band_attention import band_attention, pack_norm
    from hummingbird_b200.workloads import band_inputs
    w = band_inputs("cuda")
    lam, freqs = torch.from_numpy(w.lam).cuda(), torch.from_numpy(w.inv_freq).cuda()
    qn, kn = pack_norm(w.q_norm, "cuda"), pack_norm(w.k_norm, "cuda")
    for _ in range(calls):
        out = band_attention(w.qkv, qn, kn, freqs, w.heads, 64, w.window, lam=lam)
    return out


def dense(calls: int) -> torch.Tensor:
    from hummingbird_b200 import dense_attention as hb
    from hummingbird_b200.workloads import dense_inputs
    w = dense_inputs("cuda", batch=2, length=2648)
    f = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    cos, sin, mask = hb.tables(2648, f(w.inv_freq), f(w.valid))
    for _ in range(calls):
        out = hb.dense_attention(w.qkv, f(w.q_weight), f(w.k_weight), cos, sin, mask, w.heads, 64, w.half, w.eps,
                                 lam=f(w.lam))
    return out


def cross(calls: int) -> torch.Tensor:
    from hummingbird_b200.cross_attention import cross_attention, cross_kv
    g = torch.Generator(device="cuda").manual_seed(7)
    batch, length, heads, context = 2, 2648, 16, 128
    q2 = torch.randn(batch, length, 2 * heads * 64, generator=g, device="cuda").to(torch.bfloat16)
    kv = cross_kv(torch.randn(batch, context, 3 * heads * 64, generator=g, device="cuda").to(torch.bfloat16),
                  1 + 0.02 * torch.randn(64, generator=g, device="cuda"), heads, 1e-6)
    qw = 1 + 0.02 * torch.randn(64, generator=g, device="cuda")
    for _ in range(calls):
        out = cross_attention(q2, kv, qw, None, heads)
    return out


def glue(calls: int) -> torch.Tensor:
    """One DiT block's row kernels at the 120 s clip's shapes: the residual add + RMSNorm + adaLN before the
    next block (`residual_norm_kernel`, B=2, 2,648 rows, d 1,024) and the GLU + int8 quantiser feeding the MLP's
    second GEMM (`glu_rows_kernel`, 5,296 rows, 2 x 4,096 columns in)."""
    from hummingbird_b200 import dit_glue
    g = torch.Generator(device="cuda").manual_seed(11)
    batch, length, d, f = 2, 2648, 1024, 4096
    bf = lambda *s: torch.randn(*s, generator=g, device="cuda").to(torch.bfloat16)  # noqa: E731
    h, y, cond, weight, proj = bf(batch, length, d), bf(batch, length, d), bf(batch, 6 * d), bf(d), bf(
        batch * length, 2 * f)
    for _ in range(calls):
        x = dit_glue.residual_norm(h, y=y, gate=cond[:, 5 * d:], weight=weight, scale=cond[:, :d],
                                   shift=cond[:, d:2 * d], eps=1e-6)
        q, _ = dit_glue.glu(proj, quantize=True)
    return x.float().mean() + q.float().mean()


def band_front(calls: int, rows: int = 82_688) -> torch.Tensor:
    from hummingbird_b200.band_attention import pack_norm, pack_pre_norm, same_l_attention_x
    from hummingbird_b200.workloads import band_layer_inputs
    w = band_layer_inputs("cuda", length=rows)
    lam, freqs = torch.from_numpy(w.lam).cuda(), torch.from_numpy(w.inv_freq).cuda()
    qn, kn = pack_norm(w.q_norm, "cuda"), pack_norm(w.k_norm, "cuda")
    pre = pack_pre_norm(w.pre_norm, w.x.shape[-1], "cuda")
    for _ in range(calls):
        out = same_l_attention_x(w.x, w.to_qkv, qn, kn, freqs, w.heads, w.window, pre_norm=pre, lam=lam)
    return out


CASES = {"band": band, "dense": dense, "cross": cross, "glue": glue, "band_front": band_front}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--calls", type=int, default=3)
    ap.add_argument("--rows", type=int, default=None, help="sequence rows (band_front only)")
    args = ap.parse_args()
    kw = {"rows": args.rows} if args.rows and args.case == "band_front" else {}
    out = CASES[args.case](args.calls, **kw)
    torch.cuda.synchronize()
    print(args.case, "ok", float(out.float().abs().mean()))


if __name__ == "__main__":
    main()
