"""The Stable Audio 3 DiT denoiser restated in torch around this library's kernels (random-init weights).

Used to time a whole 120 s clip (the benchmark's config 4): `sa3jax.sampling.pingpong` (sampling.py:81-118)
over `sa3jax.dit.dit_forward` (dit.py:340-361) with its 24 `_block`s (dit.py:224-250). The self-attention is
this library's fused differential kernel (`blocks.dit_self_attention`'s path); the MLP is W8A8 when
`DiTConfig.ff_quant == "w8a8"` (else a bf16 matmul); with `glue="cuda"` the differential cross-attention over
the 128 hoisted context tokens (dit.py:203-215, 274-284) is this library's `hb_cross_diff_attn` kernel and the
residual / RMSNorm / adaLN / GLU steps its row kernels; projections are torch matmuls (cuBLAS). With
`glue="torch"` the cross-attention and the elementwise steps run as torch ops (cuDNN-flash SDPA). No checkpoint
is loaded: weights are N(0, 1 / fan_in) bf16 draws.

With a process group of N ranks (one per GPU) one clip runs on all N. The clip's batch rows are independent
through the whole denoise (the reference runs its CFG pair as a plain batch: guidance is off at
`cfg_scale=1.0`, dit.py:11), so they are split first: with B=2 and N even, ranks [0, N/2) take row 0 and
[N/2, N) row 1, with no collective between the halves. Inside each half of more than one rank, token-wise work
is split by token rows and the self-attention by head pairs, with two all-to-alls per block
(`hummingbird_b200.parallel`). Each rank holds its batch rows (`batch_range`) of the latents of its token rows
(`latent_range`); `local_view` cuts a whole-clip tensor to that part and `gather_latents` rebuilds the clip.

Cast points follow the reference under the BF16 preset: bf16 activations, RMSNorm in fp32 cast back
(dit.py:45-57), the adaLN gate `sigmoid(1 - gate)` (dit.py:227), cross K/V hoisted once per clip and k-normed
(dit.py:274-284), the constant `to_local_embed` add on the non-memory tokens (dit.py:242-244).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, replace

import torch
import torch.distributed as dist
import torch.nn.functional as F

from hummingbird_b200 import cross_attention as hb_cross
from hummingbird_b200 import dense_attention as hb_dense
from hummingbird_b200 import dit_glue as glue
from hummingbird_b200 import parallel as par
from hummingbird_b200.config import DiTConfig
from hummingbird_b200.w8a8 import W8A8GluLinear, W8A8Linear, quantize_rows, w8a8_gemm


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
    """`dit_forward` with random weights; `static` state is built once per clip (`prepare_static`).

    `group`: a process group over which one clip is split (token rows + head pairs); None = this GPU alone.
    `attend`: the differential self-attention (default: this library's kernel, `dense_attention`).
    `glue`: "cuda" runs each block's residual / RMSNorm / adaLN / GLU steps as this library's fused row
    kernels (`hummingbird_b200.dit_glue`); "torch" runs them as separate torch ops (the reference's op order)."""

    def __init__(self, cfg: DiTConfig, shape: ClipShape, device, seed: int = 4, *, group=None, attend=None,
                 glue: str = "cuda", split_batch: bool = True):
        self.cfg, self.full_shape, self.device = cfg, shape, device
        self.attend = attend or hb_dense.dense_attention
        if glue not in ("cuda", "torch"):
            raise ValueError(f"glue must be 'cuda' or 'torch', not {glue!r}")
        self.glue = glue
        # batch rows over groups of ranks first (independent rows, no collective between the groups), then
        # token rows / head pairs inside each group
        self.outer = group
        world_all = dist.get_world_size(group) if group is not None else 1
        rank_all = dist.get_rank(group) if group is not None else 0
        nb = math.gcd(shape.batch, world_all) if split_batch and world_all > 1 else 1
        inner = world_all // nb
        bg = rank_all // inner
        self.batch_groups = nb
        self.batch_range = (shape.batch * bg // nb, shape.batch * (bg + 1) // nb)
        if nb > 1:
            shape = replace(shape, batch=shape.batch // nb)
            # every rank creates every subgroup, in the same order (torch.distributed.new_group is collective)
            subgroups = [dist.new_group(list(range(k * inner, (k + 1) * inner))) if inner > 1 else None
                         for k in range(nb)]
            group = subgroups[bg]
        self.shape = shape
        self.group = group
        self.world = inner if nb > 1 else world_all
        self.rank = rank_all - bg * inner if nb > 1 else rank_all
        self.seq = cfg.num_memory_tokens + shape.latents
        self.t0, self.t1 = par.shard_tokens(self.seq, self.world, self.rank)
        self.mem_rows = max(0, min(self.t1, cfg.num_memory_tokens) - self.t0)
        if cfg.qkv_quant == "w8a8" and (self.world > 1 or glue != "cuda"):
            raise ValueError("qkv_quant='w8a8' needs glue='cuda' and one rank per batch group")
        if cfg.out_quant == "w8a8" and glue != "cuda":
            raise ValueError("out_quant='w8a8' needs glue='cuda'")
        if (cfg.num_heads // 2) % self.world or self.t1 - self.t0 <= self.mem_rows:
            raise ValueError(f"a clip of {self.seq} tokens and {cfg.num_heads // 2} head pairs does not split "
                             f"over {self.world} ranks (equal pair counts, latent rows on every rank)")
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
            b["cross_attn"]["q_norm_f"] = b["cross_attn"]["q_norm_bf"].float()
            if self.world > 1:  # rows grouped by destination rank: one batched GEMM fills the all-to-all buffer
                rows = par.dest_major_qkv_rows(h, self.world).to(device)
                b["self_attn"]["to_qkv_dest"] = b["self_attn"]["to_qkv"][rows].view(self.world, -1, d).transpose(1, 2)
            if cfg.qkv_quant == "w8a8":
                b["self_attn"]["to_qkv_q"] = W8A8Linear(b["self_attn"]["to_qkv"])
            if cfg.out_quant == "w8a8":
                b["self_attn"]["to_out_q"] = W8A8Linear(b["self_attn"]["to_out"])
            if cfg.ff_quant == "w8a8":
                b["glu_q"] = W8A8Linear(b["glu"]["w"], b["glu"]["b"])
                b["glu_fused"] = W8A8GluLinear(b["glu"]["w"], b["glu"]["b"])
                b["proj_out_q"] = W8A8Linear(b["proj_out"]["w"], b["proj_out"]["b"])
            self.blocks.append(b)

    # ------------------------------------------------------------------ per clip
    def prepare_static(self, cross_cond: torch.Tensor, global_cond: torch.Tensor) -> dict:
        """`dit.prepare_static` (dit.py:287-337): hoisted, k-normed cross K/V per block, conditioning, tables.
        The conditioning may hold the whole clip's batch rows; this rank's are taken."""
        cross_cond, global_cond = self._rows(cross_cond), self._rows(global_cond)
        cfg, d, h = self.cfg, self.cfg.embed_dim, self.cfg.num_heads
        seq = cfg.num_memory_tokens + self.shape.latents
        valid = torch.ones(self.shape.batch, seq, device=self.device)
        cos, sin, mask = hb_dense.tables(seq, self.p["rope_inv_freq"], valid, cfg.head_dim)
        ctx = self._seq(self.p["to_cond_embed"], cross_cond.to(torch.bfloat16))
        kv, kv_rows = [], []
        for b in self.blocks:
            x = ctx @ b["cross_attn"]["to_kv"].T
            kn = b["cross_attn"]["k_norm"]
            if self.glue == "cuda":  # the kernel's layout: (B, context, [k | k_diff | v]) rows, keys k-normed
                kv_rows.append(hb_cross.cross_kv(x, kn, h, cfg.qk_norm_eps, cfg.head_dim))
                continue
            k, kd, v = (t.unflatten(-1, (h, cfg.head_dim)).transpose(1, 2) for t in x.chunk(3, -1))
            kv.append((_rms(k, kn, cfg.qk_norm_eps), _rms(kd, kn, cfg.qk_norm_eps), v))
        return {"lane_cos": cos, "lane_sin": sin, "lane_mask": mask, "cross_kv": kv, "cross_kv_rows": kv_rows,
                "gcond_proj": self._seq(self.p["to_global_embed"], global_cond.to(torch.bfloat16))}

    @staticmethod
    def _seq(layers, x):
        """`nn.Sequential(Linear, SiLU, Linear)` without biases (dit.py:39-42)."""
        return F.silu(x @ layers[0].T) @ layers[1].T

    # ------------------------------------------------------------------ sharding
    def latent_range(self) -> tuple[int, int]:
        """Latent indices [a, b) whose rows this rank holds (all of them on one GPU)."""
        mem = self.cfg.num_memory_tokens
        return max(self.t0, mem) - mem, self.t1 - mem

    def _rows(self, t: torch.Tensor) -> torch.Tensor:
        """This rank's batch rows of a tensor that holds the whole clip's batch (others pass through)."""
        if self.batch_groups > 1 and t.shape[0] == self.full_shape.batch:
            return t[self.batch_range[0]:self.batch_range[1]]
        return t

    def local_view(self, x: torch.Tensor) -> torch.Tensor:
        """The whole clip's `(..., B, io, T)` latents -> this rank's `(..., B_r, io, T_r)` part (contiguous)."""
        a, b = self.latent_range()
        b0, b1 = self.batch_range
        return x[..., b0:b1, :, a:b].contiguous()

    def gather_latents(self, x_local: torch.Tensor) -> torch.Tensor:
        """All ranks' `(B_r, io, T_r)` parts -> the whole clip `(B, io, T)`."""
        x = x_local
        if self.world > 1:
            mem = self.cfg.num_memory_tokens
            spans = [par.shard_tokens(self.seq, self.world, r) for r in range(self.world)]
            widths = [t1 - max(t0, mem) for t0, t1 in spans]
            padded = x.new_zeros(*x.shape[:2], max(widths))
            padded[..., :x.shape[-1]] = x
            parts = [torch.empty_like(padded) for _ in range(self.world)]
            dist.all_gather(parts, padded, group=self.group)
            x = torch.cat([part[..., :w] for part, w in zip(parts, widths)], -1)
        if self.batch_groups > 1:  # one copy of each batch group's rows (every rank of a group holds them)
            parts = [torch.empty_like(x) for _ in range(dist.get_world_size(self.outer))]
            dist.all_gather(parts, x.contiguous(), group=self.outer)
            inner = len(parts) // self.batch_groups
            x = torch.cat([parts[k * inner] for k in range(self.batch_groups)], 0)
        return x

    # ------------------------------------------------------------------ denoiser
    def forward(self, x: torch.Tensor, t: torch.Tensor, static: dict) -> torch.Tensor:
        """`dit_forward`: `(B, io, T_r)` latents (this rank's `latent_range`; all T on one GPU) and `(B,)`
        timesteps -> velocity of the same shape (dit.py:340-361)."""
        cfg, p = self.cfg, self.p
        t = self._rows(t)
        h = x.to(torch.bfloat16)
        h = torch.einsum("bct,oc->bot", h, p["preprocess_conv"]) + h
        h = h.transpose(1, 2) @ p["project_in"].T
        if self.mem_rows:
            mem = p["memory_tokens"][self.t0:self.t0 + self.mem_rows].expand(h.shape[0], -1, -1)
            h = torch.cat([mem, h], 1)
        temb = self._seq(p["to_timestep_embed"], _expo_fourier(t.to(torch.bfloat16), cfg.fourier_dim))
        gcond = self._seq(p["global_cond_embedder"], static["gcond_proj"] + temb)
        if self.glue == "cuda":
            h = self._blocks_fused(h.contiguous(), static, gcond)
        else:
            for i, b in enumerate(self.blocks):
                h = self._block(h, b, static, gcond, i)
        h = h[:, self.mem_rows:] @ p["project_out"].T
        v = h.transpose(1, 2)
        return torch.einsum("bct,oc->bot", v, p["postprocess_conv"]) + v

    def _block(self, h, b, static, gcond, index):
        """One block with the elementwise steps fused where torch offers it: RMSNorm (fp32 statistics,
        `rms_norm`), `x * (1 + scale) + shift` and `h + y * sigmoid(1 - gate)` as single `addcmul`s."""
        cfg, d = self.cfg, self.cfg.embed_dim
        ss, sh, gs, sf, shf, gf = (b["to_scale_shift_gate"] + gcond)[:, None, :].chunk(6, -1)
        x = torch.addcmul(sh, F.rms_norm(h, (d,), b["pre_norm_bf"], cfg.norm_eps), 1 + ss)
        h = torch.addcmul(h, self._self_attn(x, b["self_attn"], static) @ b["self_attn"]["to_out"].T,
                          torch.sigmoid(1 - gs))
        x = F.rms_norm(h, (d,), b["cross_attend_norm_bf"], cfg.norm_eps)
        h = h + self._cross(x, b["cross_attn"], static["cross_kv"][index])
        h[:, self.mem_rows:] += b["local"]
        x = torch.addcmul(shf, F.rms_norm(h, (d,), b["ff_norm_bf"], cfg.norm_eps), 1 + sf)
        return torch.addcmul(h, self._ff(x, b), torch.sigmoid(1 - gf))

    def _blocks_fused(self, h, static, gcond):
        """All blocks with the glue in fused kernels: each residual add is fused with the norm (and adaLN
        modulation) that follows it, so `h` is updated in place and read once per residual."""
        cfg, d = self.cfg, self.cfg.embed_dim
        eps = cfg.norm_eps
        conds = [(b["to_scale_shift_gate"] + gcond).contiguous() for b in self.blocks]  # (B, 6d) each

        def part(c, i):  # scale_self, shift_self, gate_self, scale_ff, shift_ff, gate_ff (dit.py:230-232)
            return c[:, i * d:(i + 1) * d]

        qkv_q = cfg.qkv_quant == "w8a8"  # x before the self-attention comes per-token quantised, for to_qkv
        c0 = conds[0]
        x = glue.residual_norm(h, weight=self.blocks[0]["pre_norm_bf"], scale=part(c0, 0), shift=part(c0, 1), eps=eps,
                               quantize=qkv_q)
        for i, b in enumerate(self.blocks):
            c = conds[i]
            y = self._to_out(self._self_attn(x, b["self_attn"], static, lead=h.shape[:-1]), b["self_attn"])
            x = glue.residual_norm(h, y=y, gate=part(c, 2), weight=b["cross_attend_norm_bf"], eps=eps)
            y = self._cross_fused(x, b["cross_attn"], static["cross_kv_rows"][i])
            if self.cfg.ff_quant == "w8a8":  # the MLP's input leaves the norm kernel already quantised per token
                qx, sx = glue.residual_norm(h, y=y, local=b["local"], local_row0=self.mem_rows,
                                            weight=b["ff_norm_bf"], scale=part(c, 3), shift=part(c, 4), eps=eps,
                                            quantize=True)
                y = self._ff_quantized(qx, sx, b, h.shape[:-1])
            else:
                x = glue.residual_norm(h, y=y, local=b["local"], local_row0=self.mem_rows, weight=b["ff_norm_bf"],
                                       scale=part(c, 3), shift=part(c, 4), eps=eps)
                y = self._ff(x, b)
            if i + 1 < len(self.blocks):
                nb, nc = self.blocks[i + 1], conds[i + 1]
                x = glue.residual_norm(h, y=y, gate=part(c, 5), weight=nb["pre_norm_bf"], scale=part(nc, 0),
                                       shift=part(nc, 1), eps=eps, quantize=qkv_q)
            else:
                glue.residual_norm(h, y=y, gate=part(c, 5), eps=eps)
        return h

    def _self_attn(self, x, sa, static, lead=None):
        """`to_qkv` -> fused differential attention (dit.py:185-200), before `to_out`. Over N ranks: this
        rank's rows of every rank's `to_qkv` columns in one batched GEMM, all-to-all to head pairs, the kernel
        on this rank's pairs over all rows, all-to-all back to this rank's rows. `x` may be the per-token int8
        form `(q, scale)` (`qkv_quant="w8a8"`), with `lead` its `(B, T)`."""
        cfg = self.cfg
        args = (sa["q_norm"], sa["k_norm"], static["lane_cos"], static["lane_sin"], static["lane_mask"])
        if isinstance(x, tuple):
            lin = sa["to_qkv_q"]
            qkv = w8a8_gemm(x[0], x[1], lin.qw, lin.sw).view(*lead, -1)
            return self.attend(qkv, *args, cfg.num_heads, cfg.head_dim, cfg.rope_dim // 2, cfg.qk_norm_eps)
        if self.world == 1:
            return self.attend(x @ sa["to_qkv"].T, *args, cfg.num_heads, cfg.head_dim, cfg.rope_dim // 2,
                               cfg.qk_norm_eps)
        bsz, rows, d = x.shape
        send = torch.matmul(x.reshape(1, bsz * rows, d), sa["to_qkv_dest"])  # (N, B * rows, C)
        qkv = par.tokens_to_pairs(send.view(self.world, bsz, rows, -1), self.seq, self.world, self.group)
        att = self.attend(qkv, *args, cfg.num_heads // self.world, cfg.head_dim, cfg.rope_dim // 2, cfg.qk_norm_eps)
        return par.pairs_to_tokens(att, self.seq, self.world, self.rank, self.group)

    def _to_out(self, att, sa):
        """The self-attention's `to_out` (dit.py:199): a bf16 matmul, or with `out_quant="w8a8"` the attention
        output quantised per token and a W8A8 GEMM (`to_out` has no bias)."""
        if self.cfg.out_quant != "w8a8":
            return att @ sa["to_out"].T
        lin = sa["to_out_q"]
        qa, sa_scale = quantize_rows(att.reshape(-1, att.shape[-1]))
        return w8a8_gemm(qa, sa_scale, lin.qw, lin.sw).view(*att.shape[:-1], -1)

    def _cross_fused(self, x, ca, kv_rows):
        """Differential cross-attention (dit.py:203-215) as this library's kernel: `to_q`, then q RMSNorm and
        both softmax branches over the hoisted keys in one launch (`hb_cross_diff_attn`), then `to_out`."""
        cfg = self.cfg
        att = hb_cross.cross_attention(x @ ca["to_q"].T, kv_rows, ca["q_norm_f"], None, cfg.num_heads,
                                       cfg.head_dim, cfg.qk_norm_eps)
        return att @ ca["to_out"].T

    def _cross(self, x, ca, kv):
        """Differential cross-attention, no RoPE, no mask (dit.py:203-215): SDPA(q) - SDPA(q_diff), torch ops."""
        cfg = self.cfg
        bsz, length, _ = x.shape
        q2 = (x @ ca["to_q"].T).view(bsz, length, 2, cfg.num_heads, cfg.head_dim)
        q2 = F.rms_norm(q2, (cfg.head_dim,), ca["q_norm_bf"], cfg.qk_norm_eps)
        q, qd = q2[:, :, 0].transpose(1, 2), q2[:, :, 1].transpose(1, 2)
        k, kd, v = kv
        out = F.scaled_dot_product_attention(q, k, v) - F.scaled_dot_product_attention(qd, kd, v)
        return out.transpose(1, 2).reshape(bsz, length, -1) @ ca["to_out"].T

    def _ff_quantized(self, qx, sx, b, lead):
        """The W8A8 MLP from its per-token quantised input: GEMM1 with the GLU in its epilogue, the quantiser,
        GEMM2."""
        z = b["glu_fused"].quantized(qx, sx)
        q, s = quantize_rows(z)
        po = b["proj_out_q"]
        return w8a8_gemm(q, s, po.qw, po.sw, po.bias).view(*lead, -1)

    def _ff(self, x, b):
        """`dit._feed_forward`: GLU `value * silu(gate)` (dit.py:218-221), W8A8 or bf16."""
        if self.cfg.ff_quant == "w8a8":
            if self.glue == "cuda":  # value * silu(gate) in the first GEMM's epilogue, then the per-token quantiser
                z = b["glu_fused"](x)
                q, s = quantize_rows(z.reshape(-1, z.shape[-1]))
                po = b["proj_out_q"]
                return w8a8_gemm(q, s, po.qw, po.sw, po.bias).view(*x.shape[:-1], -1)
            g = b["glu_q"](x)
            value, gate = g.chunk(2, -1)
            return b["proj_out_q"](value * F.silu(gate))
        g = x @ b["glu"]["w"].T + b["glu"]["b"]
        if self.glue == "cuda":
            return glue.glu(g) @ b["proj_out"]["w"].T + b["proj_out"]["b"]
        value, gate = g.chunk(2, -1)
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

    def denoise_graph(self, x0: torch.Tensor, eps: torch.Tensor, static: dict, steps: int | None = None):
        """`sampling.pingpong` (sampling.py:81-118, one `lax.scan` over the steps) as one CUDA graph: every step
        of the denoise loop, the schedule's timesteps baked in as constants, replayed with one launch per clip.

        `x0` is this rank's `(B_r, io, T_r)` initial latents and `eps` its `(steps, B_r, io, T_r)` noise, both
        read by the graph (refill `x0` in place between replays). Returns `run`, which replays the graph and
        returns the final latents (a tensor the graph owns, overwritten by the next replay), and the graph:
        keep it alive while replaying, and release it before the process group when the loop holds
        collectives. Capture needs a CUDA device."""
        steps = self.shape.steps if steps is None else steps
        sched = [float(v) for v in self.schedule(steps, device=x0.device)]
        bsz, dev = x0.shape[0], x0.device
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):  # warm-up outside the capture: library handles and workspaces
            t = torch.full((bsz,), sched[0], device=dev, dtype=torch.bfloat16)
            for _ in range(2):
                self.step(x0, t, t, eps[0], static)
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            x = x0
            for s in range(steps):
                t_cur = torch.full((bsz,), sched[s], device=dev, dtype=torch.bfloat16)
                t_nxt = torch.full((bsz,), sched[s + 1], device=dev, dtype=torch.bfloat16)
                x = self.step(x, t_cur, t_nxt, eps[s], static)
        x_out = x

        def run():
            graph.replay()
            return x_out

        return run, graph

    def step(self, x, t_curr, t_next, eps, static):
        """One pingpong step (sampling.py:109-113)."""
        t_curr, t_next = self._rows(t_curr), self._rows(t_next)
        v = self.forward(x, t_curr, static)
        denoised = x - t_curr[:, None, None] * v
        return (1 - t_next[:, None, None]) * denoised + t_next[:, None, None] * eps
