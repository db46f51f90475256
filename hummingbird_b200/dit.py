"""The Stable Audio 3 DiT denoiser restated in torch around this library's kernels (random-init weights).

Used to time a whole 120 s clip (the benchmark's config 4): `sa3jax.sampling.pingpong` (sampling.py:81-118)
over `sa3jax.dit.dit_forward` (dit.py:340-361) with its 24 `_block`s (dit.py:224-250). The self-attention is
this library's fused differential kernel (`blocks.dit_self_attention`'s path); the MLP is W8A8 when
`DiTConfig.ff_quant == "w8a8"` (else a bf16 matmul); projections, RMSNorm / adaLN elementwise work and the
differential cross-attention over the 128 hoisted context tokens (dit.py:203-215, 274-284) run as torch ops
(cuBLAS / cuDNN-flash library kernels). No checkpoint is loaded: weights are N(0, 1 / fan_in) bf16 draws.

Cast points follow the reference under the BF16 preset: bf16 activations, RMSNorm in fp32 cast back
(dit.py:45-57), the adaLN gate `sigmoid(1 - gate)` (dit.py:227), cross K/V hoisted once per clip and k-normed
(dit.py:274-284), the constant `to_local_embed` add on the non-memory tokens (dit.py:242-244).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from hummingbird_b200 import dense_attention as hb_dense
from hummingbird_b200.config import DiTConfig
from hummingbird_b200.w8a8 import W8A8Linear


@dataclass(frozen=True)
class ClipShape:
    batch: int = 2            # CFG pair
    latents: int = 2584       # 120 s
    io_channels: int = 64
    context: int = 128        # conditioning tokens
    context_dim: int = 768
    depth: int = 24
    steps: int = 8


def _w(shape, gen, device, fan_in=None):
    fan_in = fan_in or shape[-1]
    return (torch.randn(shape, generator=gen, device=device) / math.sqrt(fan_in)).to(torch.bfloat16)


def _rms(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """`dit._rms`: mean of squares in fp32, scale, cast back to the input dtype."""
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * weight.float()).to(x.dtype)


def _expo_fourier(t: torch.Tensor, dim: int) -> torch.Tensor:
    """`ExpoFourierFeatures(256, 0.5, 10000)` (dit.py:71-79), fp32, cast back."""
    freqs = torch.exp(torch.linspace(0.0, 1.0, dim // 2, device=t.device) * (math.log(10000.0) - math.log(0.5))
                      + math.log(0.5))
    args = t.float()[:, None] * freqs * (2.0 * math.pi)
    return torch.cat([torch.cos(args), torch.sin(args)], -1).to(t.dtype)


class DiT:
    """`dit_forward` with random weights; `static` state is built once per clip (`prepare_static`)."""

    def __init__(self, cfg: DiTConfig, shape: ClipShape, device, seed: int = 4):
        self.cfg, self.shape, self.device = cfg, shape, device
        g = torch.Generator(device=device).manual_seed(seed)
        d, h = cfg.embed_dim, cfg.num_heads
        io, ctx = shape.io_channels, shape.context_dim
        self.p = {
            "preprocess_conv": _w((io, io), g, device), "postprocess_conv": _w((io, io), g, device),
            "project_in": _w((d, io), g, device), "project_out": _w((io, d), g, device),
            "memory_tokens": torch.randn(cfg.num_memory_tokens, d, generator=g, device=device).to(torch.bfloat16),
            "to_cond_embed": [_w((d, ctx), g, device), _w((d, d), g, device)],
            "to_global_embed": [_w((d, ctx), g, device), _w((d, d), g, device)],
            "to_timestep_embed": [_w((d, cfg.fourier_dim), g, device), _w((d, d), g, device)],
            "global_cond_embedder": [_w((d, d), g, device), _w((6 * d, d), g, device)],
            "rope_inv_freq": (1.0 / (cfg.rope_theta ** (torch.arange(0, cfg.rope_dim, 2, device=device).float()
                                                          / cfg.rope_dim))),
        }
        self.blocks = []
        for _ in range(shape.depth):
            b = {
                "to_scale_shift_gate": (0.02 * torch.randn(6 * d, generator=g, device=device)).to(torch.bfloat16),
                "pre_norm": 1 + 0.02 * torch.randn(d, generator=g, device=device),
                "cross_attend_norm": 1 + 0.02 * torch.randn(d, generator=g, device=device),
                "ff_norm": 1 + 0.02 * torch.randn(d, generator=g, device=device),
                "self_attn": {"to_qkv": _w((5 * d, d), g, device), "to_out": _w((d, d), g, device),
                              "q_norm": 1 + 0.02 * torch.randn(cfg.head_dim, generator=g, device=device),
                              "k_norm": 1 + 0.02 * torch.randn(cfg.head_dim, generator=g, device=device)},
                "cross_attn": {"to_q": _w((2 * d, d), g, device), "to_kv": _w((3 * d, d), g, device),
                               "to_out": _w((d, d), g, device),
                               "q_norm": 1 + 0.02 * torch.randn(cfg.head_dim, generator=g, device=device),
                               "k_norm": 1 + 0.02 * torch.randn(cfg.head_dim, generator=g, device=device)},
                "glu": {"w": _w((2 * cfg.ff_inner, d), g, device), "b": torch.zeros(2 * cfg.ff_inner, device=device,
                                                                                    dtype=torch.bfloat16)},
                "proj_out": {"w": _w((d, cfg.ff_inner), g, device), "b": torch.zeros(d, device=device,
                                                                                    dtype=torch.bfloat16)},
                "local": (0.02 * torch.randn(d, generator=g, device=device)).to(torch.bfloat16),
            }
            for name in ("pre_norm", "cross_attend_norm", "ff_norm"):
                b[name + "_bf"] = b[name].to(torch.bfloat16)  # checkpoint norm weights are bf16
            b["cross_attn"]["q_norm_bf"] = b["cross_attn"]["q_norm"].to(torch.bfloat16)
            if cfg.ff_quant == "w8a8":
                b["glu_q"] = W8A8Linear(b["glu"]["w"], b["glu"]["b"])
                b["proj_out_q"] = W8A8Linear(b["proj_out"]["w"], b["proj_out"]["b"])
            self.blocks.append(b)

    # ------------------------------------------------------------------ per clip
    def prepare_static(self, cross_cond: torch.Tensor, global_cond: torch.Tensor) -> dict:
        """`dit.prepare_static` (dit.py:287-337): hoisted, k-normed cross K/V per block, conditioning, tables."""
        cfg, d, h = self.cfg, self.cfg.embed_dim, self.cfg.num_heads
        seq = cfg.num_memory_tokens + self.shape.latents
        valid = torch.ones(self.shape.batch, seq, device=self.device)
        cos, sin, mask = hb_dense.tables(seq, self.p["rope_inv_freq"], valid, cfg.head_dim)
        ctx = self._seq(self.p["to_cond_embed"], cross_cond.to(torch.bfloat16))
        kv = []
        for b in self.blocks:
            x = ctx @ b["cross_attn"]["to_kv"].T
            k, kd, v = (t.unflatten(-1, (h, cfg.head_dim)).transpose(1, 2) for t in x.chunk(3, -1))
            kn = b["cross_attn"]["k_norm"]
            kv.append((_rms(k, kn, cfg.qk_norm_eps), _rms(kd, kn, cfg.qk_norm_eps), v))
        return {"lane_cos": cos, "lane_sin": sin, "lane_mask": mask, "cross_kv": kv,
                "gcond_proj": self._seq(self.p["to_global_embed"], global_cond.to(torch.bfloat16))}

    @staticmethod
    def _seq(layers, x):
        """`nn.Sequential(Linear, SiLU, Linear)` without biases (dit.py:39-42)."""
        return F.silu(x @ layers[0].T) @ layers[1].T

    # ------------------------------------------------------------------ denoiser
    def forward(self, x: torch.Tensor, t: torch.Tensor, static: dict) -> torch.Tensor:
        """`dit_forward`: `(B, io, T)` latents and `(B,)` timesteps -> velocity `(B, io, T)` (dit.py:340-361)."""
        cfg, p = self.cfg, self.p
        h = x.to(torch.bfloat16)
        h = torch.einsum("bct,oc->bot", h, p["preprocess_conv"]) + h
        h = h.transpose(1, 2) @ p["project_in"].T
        mem = p["memory_tokens"].expand(h.shape[0], -1, -1)
        h = torch.cat([mem, h], 1)
        temb = self._seq(p["to_timestep_embed"], _expo_fourier(t.to(torch.bfloat16), cfg.fourier_dim))
        gcond = self._seq(p["global_cond_embedder"], static["gcond_proj"] + temb)
        for i, b in enumerate(self.blocks):
            h = self._block(h, b, static, gcond, i)
        h = h[:, cfg.num_memory_tokens:] @ p["project_out"].T
        v = h.transpose(1, 2)
        return torch.einsum("bct,oc->bot", v, p["postprocess_conv"]) + v

    def _block(self, h, b, static, gcond, index):
        """One block with the elementwise steps fused where torch offers it: RMSNorm (fp32 statistics,
        `rms_norm`), `x * (1 + scale) + shift` and `h + y * sigmoid(1 - gate)` as single `addcmul`s."""
        cfg, d, mem = self.cfg, self.cfg.embed_dim, self.cfg.num_memory_tokens
        ss, sh, gs, sf, shf, gf = (b["to_scale_shift_gate"] + gcond)[:, None, :].chunk(6, -1)
        x = torch.addcmul(sh, F.rms_norm(h, (d,), b["pre_norm_bf"], cfg.norm_eps), 1 + ss)
        sa = b["self_attn"]
        qkv = x @ sa["to_qkv"].T
        att = hb_dense.dense_attention(qkv, sa["q_norm"], sa["k_norm"], static["lane_cos"], static["lane_sin"],
                                       static["lane_mask"], cfg.num_heads, cfg.head_dim, cfg.rope_dim // 2,
                                       cfg.qk_norm_eps)
        h = torch.addcmul(h, att @ sa["to_out"].T, torch.sigmoid(1 - gs))
        x = F.rms_norm(h, (d,), b["cross_attend_norm_bf"], cfg.norm_eps)
        h = h + self._cross(x, b["cross_attn"], static["cross_kv"][index])
        h[:, mem:] += b["local"]
        x = torch.addcmul(shf, F.rms_norm(h, (d,), b["ff_norm_bf"], cfg.norm_eps), 1 + sf)
        return torch.addcmul(h, self._ff(x, b), torch.sigmoid(1 - gf))

    def _cross(self, x, ca, kv):
        """Differential cross-attention, no RoPE, no mask (dit.py:203-215): SDPA(q) - SDPA(q_diff)."""
        cfg = self.cfg
        bsz, length, _ = x.shape
        q2 = (x @ ca["to_q"].T).view(bsz, length, 2, cfg.num_heads, cfg.head_dim)
        q2 = F.rms_norm(q2, (cfg.head_dim,), ca["q_norm_bf"], cfg.qk_norm_eps)
        q, qd = q2[:, :, 0].transpose(1, 2), q2[:, :, 1].transpose(1, 2)
        k, kd, v = kv
        out = F.scaled_dot_product_attention(q, k, v) - F.scaled_dot_product_attention(qd, kd, v)
        return out.transpose(1, 2).reshape(bsz, length, -1) @ ca["to_out"].T

    def _ff(self, x, b):
        """`dit._feed_forward`: GLU `value * silu(gate)` (dit.py:218-221), W8A8 or bf16."""
        if self.cfg.ff_quant == "w8a8":
            value, gate = b["glu_q"](x).chunk(2, -1)
            return b["proj_out_q"](value * F.silu(gate))
        value, gate = (x @ b["glu"]["w"].T + b["glu"]["b"]).chunk(2, -1)
        return (value * F.silu(gate)) @ b["proj_out"]["w"].T + b["proj_out"]["b"]

    # ------------------------------------------------------------------ sampler
    @staticmethod
    def schedule(steps: int, sigma_max: float = 1.0, anchor_logsnr: float = -6.2, logsnr_end: float = 2.0,
                 device=None) -> torch.Tensor:
        """`sampling.build_schedule` (sampling.py:65-78)."""
        t = torch.linspace(sigma_max, 0.0, steps + 1, device=device)
        out = torch.sigmoid(-(logsnr_end - t * (logsnr_end - anchor_logsnr)))
        out = torch.where(t <= 0, torch.zeros_like(out), out)
        out = torch.where(t >= 1, torch.ones_like(out), out)
        out[0] = sigma_max
        return out

    def step(self, x, t_curr, t_next, eps, static):
        """One pingpong step (sampling.py:109-113)."""
        v = self.forward(x, t_curr, static)
        denoised = x - t_curr[:, None, None] * v
        return (1 - t_next[:, None, None]) * denoised + t_next[:, None, None] * eps
