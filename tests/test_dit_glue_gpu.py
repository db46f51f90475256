"""GPU: the fused DiT glue kernels (`hummingbird_b200.dit_glue`, through the C ABI) against the torch ops they
replace, and a DiT step with fused glue against the same step with torch glue. The kernels round where the
torch sequence stores bf16, so results agree to within one bf16 rounding on a small fraction of elements
(transcendentals: `__expf` against torch's `expf`; sums: a different reduction order)."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _close_bf16(got, want, frac=0.02):
    """Equal, except a fraction `frac` of elements that may differ by at most 2 bf16 ulps of their value."""
    g, w = got.float(), want.float()
    assert g.shape == w.shape
    assert torch.isfinite(g).all()
    diff = (g - w).abs()
    ulp = torch.clamp(w.abs(), min=2.0 ** -60) * 2.0 ** -7
    assert (diff <= 2 * ulp + 1e-30).all(), f"max diff {diff.max().item():.3e}"
    assert (diff > 0).float().mean().item() <= frac


def _bf(*shape, gen, scale=1.0):
    return (scale * torch.randn(*shape, generator=gen, device="cuda")).to(torch.bfloat16)


@pytest.mark.parametrize("d", [1024, 512])
def test_residual_norm_matches_torch_ops(cuda_lib, d):
    from hummingbird_b200 import dit_glue as glue
    g = torch.Generator(device="cuda").manual_seed(11)
    bsz, t, eps, mem = 2, 300, 1e-5, 64
    h0 = _bf(bsz, t, d, gen=g, scale=3.0)
    y = _bf(bsz, t, d, gen=g)
    cond = _bf(bsz, 3 * d, gen=g, scale=0.5)
    gate, scale, shift = cond[:, :d], cond[:, d:2 * d], cond[:, 2 * d:]
    w = (1 + 0.02 * torch.randn(d, generator=g, device="cuda")).to(torch.bfloat16)
    local = _bf(d, gen=g, scale=0.1)
    # gated residual + norm + modulation (dit.py:235-237 order)
    h = h0.clone()
    x = glue.residual_norm(h, y=y, gate=gate, weight=w, scale=scale, shift=shift, eps=eps)
    h_ref = torch.addcmul(h0, y, torch.sigmoid(1 - gate[:, None, :]))
    x_ref = torch.addcmul(shift[:, None, :], F.rms_norm(h_ref, (d,), w, eps), 1 + scale[:, None, :])
    _close_bf16(h, h_ref)
    _close_bf16(x, x_ref)
    # plain residual + local rows + norm without modulation (dit.py:239-244)
    h = h0.clone()
    x = glue.residual_norm(h, y=y, local=local, local_row0=mem, weight=w, eps=eps)
    h_ref = h0 + y
    h_ref[:, mem:] += local
    _close_bf16(h, h_ref)
    _close_bf16(x, F.rms_norm(h_ref, (d,), w, eps))
    # residual only (the last block)
    h = h0.clone()
    assert glue.residual_norm(h, y=y, gate=gate, eps=eps) is None
    _close_bf16(h, torch.addcmul(h0, y, torch.sigmoid(1 - gate[:, None, :])))


def test_residual_norm_many_batch_elements(cuda_lib):
    """More batch elements than one launch holds column vectors for (d = 2048: two per launch), ragged rows."""
    from hummingbird_b200 import dit_glue as glue
    g = torch.Generator(device="cuda").manual_seed(15)
    bsz, t, d, eps = 5, 37, 2048, 1e-6
    h0 = _bf(bsz, t, d, gen=g, scale=2.0)
    y = _bf(bsz, t, d, gen=g)
    cond = _bf(bsz, 3 * d, gen=g, scale=0.5)
    gate, scale, shift = cond[:, :d], cond[:, d:2 * d], cond[:, 2 * d:]
    w = (1 + 0.02 * torch.randn(d, generator=g, device="cuda")).to(torch.bfloat16)
    h = h0.clone()
    x = glue.residual_norm(h, y=y, gate=gate, weight=w, scale=scale, shift=shift, eps=eps)
    h_ref = torch.addcmul(h0, y, torch.sigmoid(1 - gate[:, None, :]))
    x_ref = torch.addcmul(shift[:, None, :], F.rms_norm(h_ref, (d,), w, eps), 1 + scale[:, None, :])
    _close_bf16(h, h_ref)
    _close_bf16(x, x_ref)


def test_glu_matches_torch_and_quantises_with_the_quantiser_rules(cuda_lib):
    from hummingbird_b200 import dit_glue as glue
    from hummingbird_b200.w8a8 import quantize_rows
    g = torch.Generator(device="cuda").manual_seed(12)
    x = _bf(517, 2 * 4096, gen=g, scale=2.0)
    x[3] = 0  # an all-zero row quantises with scale 1
    value, gate = x.chunk(2, -1)
    z_ref = value * F.silu(gate)
    z = glue.glu(x)
    _close_bf16(z, z_ref)
    q, s = glue.glu(x, quantize=True)
    q_ref, s_ref = quantize_rows(z)  # the quantiser on the kernel's own z: bit-exact
    assert torch.equal(q, q_ref) and torch.equal(s, s_ref)
    assert s[3].item() == 1.0 and (q[3] == 0).all()


def test_head_rms_norm_matches_torch(cuda_lib):
    from hummingbird_b200 import dit_glue as glue
    g = torch.Generator(device="cuda").manual_seed(13)
    x = _bf(2, 300, 2048, gen=g, scale=4.0)
    w = (1 + 0.02 * torch.randn(64, generator=g, device="cuda")).to(torch.bfloat16)
    got = glue.head_rms_norm(x, w, 1e-6)
    want = F.rms_norm(x.view(2, 300, 32, 64), (64,), w, 1e-6).view(2, 300, 2048)
    _close_bf16(got, want)


def test_glue_rejects_bad_shapes(cuda_lib):
    from hummingbird_b200 import dit_glue as glue
    h = torch.zeros(1, 8, 300, dtype=torch.bfloat16, device="cuda")  # d not a multiple of 256
    with pytest.raises(ValueError):
        glue.residual_norm(h, weight=torch.ones(300, dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(ValueError):
        glue.glu(torch.zeros(4, 2 * 8200, dtype=torch.bfloat16, device="cuda"))  # F > 8192


@pytest.mark.parametrize("ff_quant", ["w8a8", "none"])
def test_dit_step_fused_glue_matches_torch_glue(cuda_lib, ff_quant):
    from hummingbird_b200.config import DiTConfig
    from hummingbird_b200.dit import ClipShape, DiT
    shape = ClipShape(batch=2, latents=200, depth=3, steps=2)
    g = torch.Generator(device="cuda").manual_seed(14)
    cross = torch.randn(2, 128, 768, generator=g, device="cuda")
    glob = torch.randn(2, 768, generator=g, device="cuda")
    x = _bf(2, 64, 200, gen=g)
    eps = _bf(2, 64, 200, gen=g)
    t = torch.full((2,), 0.9, device="cuda", dtype=torch.bfloat16)
    tn = torch.full((2,), 0.5, device="cuda", dtype=torch.bfloat16)
    outs = []
    for glue in ("cuda", "torch"):
        model = DiT(DiTConfig(ff_quant=ff_quant), shape, "cuda", glue=glue)
        outs.append(model.step(x, t, tn, eps, model.prepare_static(cross, glob)).float())
    rel = ((outs[0] - outs[1]).norm() / outs[1].norm()).item()
    assert torch.isfinite(outs[0]).all() and rel < 2e-2, f"relative difference {rel:.3e}"


@pytest.mark.parametrize("d,mods", [(1024, "all"), (1024, "none"), (256, "gate_only"), (1536, "all")])
def test_residual_norm_int8_output_matches_quantiser(cuda_lib, d, mods):
    """`hb_dit_residual_norm_int8` writes the normalised, modulated x quantised per row: the same int8 values and
    scales as `quantize_rows` on the bf16 x of `hb_dit_residual_norm`, and the same updated h."""
    from hummingbird_b200 import dit_glue
    from hummingbird_b200.w8a8 import quantize_rows
    g = torch.Generator(device="cuda").manual_seed(d)
    bsz, t = 2, 300
    bf = lambda *s: torch.randn(*s, generator=g, device="cuda").to(torch.bfloat16)  # noqa: E731
    h0, y, cond, w, local = bf(bsz, t, d), bf(bsz, t, d), (0.3 * bf(bsz, 6 * d)).to(torch.bfloat16), bf(d), bf(d)
    kw = dict(y=y, weight=w, eps=1e-6)
    if mods in ("all", "gate_only"):
        kw["gate"] = cond[:, 2 * d:3 * d]
    if mods == "all":
        kw.update(scale=cond[:, :d], shift=cond[:, d:2 * d], local=local, local_row0=8)
    h1, h2 = h0.clone(), h0.clone()
    x = dit_glue.residual_norm(h1, **kw)
    q, s = dit_glue.residual_norm(h2, quantize=True, **kw)
    q_ref, s_ref = quantize_rows(x.reshape(-1, d))
    torch.cuda.synchronize()
    assert torch.equal(h1, h2)
    assert torch.equal(q, q_ref) and torch.equal(s, s_ref)
