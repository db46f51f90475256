"""GPU: the reference's call sites restated around the kernels (`hummingbird_b200.blocks`, `hummingbird_b200.dit`):
`to_qkv` -> fused attention -> `to_out` against the oracle on the same projection, the W8A8 GLU MLP against
its bf16 form, and a DiT denoise step (finite, deterministic, shape-preserving)."""
import numpy as np
import pytest
import torch

from gpu_util import check_attn, to_np
from oracle import band as oband
from oracle import dense as odense

pytestmark = pytest.mark.gpu


def test_dit_self_attention_call_site(cuda_lib):
    from hummingbird_b200 import blocks, dense_attention as hb
    from hummingbird_b200.config import DiTConfig
    cfg = DiTConfig(embed_dim=256, num_heads=4)
    g = torch.Generator(device="cuda").manual_seed(1)
    h = torch.randn(1, 300, 256, generator=g, device="cuda").to(torch.bfloat16)
    attn = {"to_qkv": {"weight": (torch.randn(1280, 256, generator=g, device="cuda") / 16).to(torch.bfloat16)},
            "to_out": {"weight": torch.eye(256, device="cuda", dtype=torch.bfloat16)},
            "q_norm": {"weight": torch.ones(64, device="cuda")}, "k_norm": {"weight": torch.ones(64, device="cuda")}}
    freqs = odense.inv_freq(cfg.rope_dim // 2)
    valid = torch.ones(1, 300, device="cuda")
    cos, sin, mask = hb.tables(300, torch.from_numpy(freqs).cuda(), valid)
    out = blocks.dit_self_attention(h, attn, {"lane_cos": cos, "lane_sin": sin, "lane_mask": mask}, cfg)
    qkv = to_np(h @ attn["to_qkv"]["weight"].T)
    ref = odense.dense_diff_attention(qkv, np.ones(64), np.ones(64), freqs, np.ones((1, 300)), 4, cfg.qk_norm_eps)
    check_attn(to_np(out), ref)  # identity to_out: the call site's output is the attention output (bf16)


def test_same_l_attention_call_site(cuda_lib):
    from hummingbird_b200 import blocks
    from hummingbird_b200.config import SameConfig
    cfg = SameConfig(channels=256, c_mults=(1,), stride=16)
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(1, 17 * 20, 256, generator=g, device="cuda").to(torch.bfloat16)
    norm = {"alpha": np.float32(0.5), "gamma": np.ones(64, np.float32), "beta": np.zeros(64, np.float32)}
    freqs = odense.inv_freq(cfg.rope_half)
    block = {"self_attn": {"to_qkv": {"weight": (torch.randn(1280, 256, generator=g, device="cuda") / 16).to(torch.bfloat16)},
                           "to_out": {"weight": torch.eye(256, device="cuda", dtype=torch.bfloat16)},
                           "q_norm": norm, "k_norm": norm},
             "rope_inv_freq": torch.from_numpy(freqs).cuda()}
    out = blocks.same_l_attention(x, block, cfg)  # d_model 256: the one-GEMM front end
    qkv = to_np(x @ block["self_attn"]["to_qkv"]["weight"].T)
    ref = oband.band_diff_attention(qkv, norm, norm, freqs, 4, cfg.sub_chunk_size)
    check_attn(to_np(out), ref)
    # with the block's DyT pre-norm inside the front end, against `oracle.band.front_end` (same_l.py:191)
    pre = {"alpha": np.float32(0.5), "gamma": np.full(256, 1.1, np.float32), "beta": np.full(256, 0.01, np.float32)}
    out = blocks.same_l_attention(x, block, cfg, pre_norm=pre)
    qkv = oband.front_end(to_np(x), to_np(block["self_attn"]["to_qkv"]["weight"]), pre)
    check_attn(to_np(out), oband.band_diff_attention(qkv, norm, norm, freqs, 4, cfg.sub_chunk_size))


def test_same_l_attention_call_site_wide_model(cuda_lib):
    """d_model 768 (the reference's default SAME-L width, 12 heads): past the front end's 512, so `to_qkv` is a
    bf16 matmul and the band kernel prepares q/k itself."""
    from hummingbird_b200 import blocks
    from hummingbird_b200.config import SameConfig
    cfg = SameConfig(channels=128, c_mults=(6,), stride=16)
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn(1, 17 * 12, 768, generator=g, device="cuda").to(torch.bfloat16)
    norm = {"alpha": np.float32(0.5), "gamma": np.ones(64, np.float32), "beta": np.zeros(64, np.float32)}
    freqs = odense.inv_freq(cfg.rope_half)
    block = {"self_attn": {"to_qkv": {"weight": (torch.randn(3840, 768, generator=g, device="cuda") / 28).to(torch.bfloat16)},
                           "to_out": {"weight": torch.eye(768, device="cuda", dtype=torch.bfloat16)},
                           "q_norm": norm, "k_norm": norm},
             "rope_inv_freq": torch.from_numpy(freqs).cuda()}
    out = blocks.same_l_attention(x, block, cfg)
    qkv = to_np(x @ block["self_attn"]["to_qkv"]["weight"].T)
    check_attn(to_np(out), oband.band_diff_attention(qkv, norm, norm, freqs, 12, cfg.sub_chunk_size))


def test_w8a8_glu_mlp_close_to_bf16(cuda_lib):
    from hummingbird_b200.blocks import DiTFeedForward
    from hummingbird_b200.config import DiTConfig
    g = torch.Generator(device="cuda").manual_seed(3)
    ff = {"glu_proj": {"weight": (torch.randn(8192, 1024, generator=g, device="cuda") / 32).to(torch.bfloat16),
                       "bias": torch.zeros(8192, device="cuda", dtype=torch.bfloat16)},
          "proj_out": {"weight": (torch.randn(1024, 4096, generator=g, device="cuda") / 64).to(torch.bfloat16),
                       "bias": torch.zeros(1024, device="cuda", dtype=torch.bfloat16)}}
    x = torch.randn(512, 1024, generator=g, device="cuda").to(torch.bfloat16)
    y8 = DiTFeedForward(ff, DiTConfig(ff_quant="w8a8"))(x).float()
    yb = DiTFeedForward(ff, DiTConfig(ff_quant="none"))(x).float()
    rel = (y8 - yb).norm() / yb.norm()
    assert rel < 0.05, f"W8A8 MLP relative error {rel:.3f}"


def test_dit_denoise_step_is_finite_and_deterministic(cuda_lib):
    from hummingbird_b200.config import DiTConfig
    from hummingbird_b200.dit import ClipShape, DiT
    shape = ClipShape(batch=2, latents=200, depth=2, steps=2)
    model = DiT(DiTConfig(ff_quant="w8a8"), shape, "cuda")
    g = torch.Generator(device="cuda").manual_seed(5)
    static = model.prepare_static(torch.randn(2, 128, 768, generator=g, device="cuda"),
                                  torch.randn(2, 768, generator=g, device="cuda"))
    x = torch.randn(2, 64, 200, generator=g, device="cuda").to(torch.bfloat16)
    t = torch.full((2,), 0.9, device="cuda", dtype=torch.bfloat16)
    tn = torch.full((2,), 0.5, device="cuda", dtype=torch.bfloat16)
    eps = torch.randn(2, 64, 200, generator=g, device="cuda").to(torch.bfloat16)
    a = model.step(x, t, tn, eps, static)
    b = model.step(x, t, tn, eps, static)
    assert a.shape == x.shape and torch.isfinite(a.float()).all()
    assert torch.equal(a, b)


def test_dit_denoise_loop_graph_matches_eager_steps(cuda_lib):
    """`DiT.denoise_graph`: the whole pingpong loop (sampling.py:81-118) captured as one CUDA graph gives the
    same latents as the steps run one by one with the same schedule, noise and conditioning; a second replay
    from a refilled x0 repeats them."""
    from hummingbird_b200.config import DiTConfig
    from hummingbird_b200.dit import ClipShape, DiT
    shape = ClipShape(batch=2, latents=248, depth=2, steps=3)
    model = DiT(DiTConfig(ff_quant="w8a8"), shape, "cuda")
    g = torch.Generator(device="cuda").manual_seed(6)
    static = model.prepare_static(torch.randn(2, 128, 768, generator=g, device="cuda"),
                                  torch.randn(2, 768, generator=g, device="cuda"))
    x0 = torch.randn(2, 64, 248, generator=g, device="cuda").to(torch.bfloat16)
    eps = torch.randn(3, 2, 64, 248, generator=g, device="cuda").to(torch.bfloat16)
    sched = [float(v) for v in DiT.schedule(3, device="cuda")]
    x = x0
    for s in range(3):
        t = torch.full((2,), sched[s], device="cuda", dtype=torch.bfloat16)
        tn = torch.full((2,), sched[s + 1], device="cuda", dtype=torch.bfloat16)
        x = model.step(x, t, tn, eps[s], static)
    x_in = x0.clone()
    run, graph = model.denoise_graph(x_in, eps, static)
    got = run().clone()
    x_in.copy_(x0)
    again = run().clone()
    torch.cuda.synchronize()
    assert torch.isfinite(got.float()).all()
    rel = ((got.float() - x.float()).norm() / x.float().norm()).item()
    assert rel < 1e-3, f"graph vs eager relative difference {rel:.2e}"
    assert torch.equal(got, again)
    del graph
