"""CPU (gloo, world sizes 2 to 8): the host-side partitioning of the multi-GPU paths — row / pair / clip
shards, the halo exchange that feeds sequence-sharded band attention, and the head-pair all-gather."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hummingbird_b200 import parallel as par


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(fn, world, *args):
    port = _free_port()
    mp.spawn(_entry, args=(fn, world, port, args), nprocs=world, join=True)


def _entry(rank, fn, world, port, args):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        fn(rank, world, *args)
    finally:
        dist.destroy_process_group()


def test_row_shards_cover_sequence_with_aligned_boundaries():
    for length in (82_688, 1000, 261_888):
        for world in (1, 2, 3, 8):
            bounds = [par.shard_rows(length, world, r) for r in range(world)]
            assert bounds[0][0] == 0 and bounds[-1][1] == length
            for (a0, a1), (b0, b1) in zip(bounds, bounds[1:]):
                assert a1 == b0 and a1 % 128 == 0


def test_pair_shards_cover_pairs_including_uneven_split():
    for pairs, world in ((8, 2), (8, 8), (12, 8), (4, 4)):
        sh = [par.shard_pairs(pairs, world, r) for r in range(world)]
        assert sh[0][0] == 0 and sh[-1][1] == pairs
        sizes = [b - a for a, b in sh]
        assert max(sizes) - min(sizes) <= 1


def test_qkv_columns_select_pair_lanes_of_every_section():
    cols = par.qkv_columns_for_pairs(heads=16, p0=2, p1=4)
    assert cols.numel() == 5 * 2 * 128
    assert cols[0].item() == 256 and cols[256].item() == 1024 + 256


def _halo_worker(rank, world, length, window):
    lay = par.band_layout(length, world, rank, window)
    rows = torch.arange(length, dtype=torch.float32)[None, :, None].repeat(1, 1, 4)  # row index as value
    buf = torch.full((1, lay["rows"], 4), -1.0)
    buf[:, lay["before"]:lay["before"] + lay["q_count"]] = rows[:, lay["s0"]:lay["s1"]]
    par.halo_exchange(buf, lay, rank)
    expect = rows[:, lay["pos0"]:lay["pos0"] + lay["rows"]]
    assert torch.equal(buf, expect), f"rank {rank}: halo rows differ"


@pytest.mark.parametrize("world", [2, 3])
def test_halo_exchange_gloo(world):
    _run(_halo_worker, world, 1000, 128)


def _gather_worker(rank, world, pairs):
    p0, p1 = par.shard_pairs(pairs, world, rank)
    local = torch.arange(p0 * 128, p1 * 128, dtype=torch.float32).repeat(2, 3, 1)
    full = par.gather_pairs(local, pairs, world)
    assert torch.equal(full, torch.arange(pairs * 128, dtype=torch.float32).repeat(2, 3, 1))


@pytest.mark.parametrize("world,pairs", [(2, 8), (3, 8)])
def test_gather_pairs_gloo(world, pairs):
    _run(_gather_worker, world, pairs)


def test_shard_shorter_than_window_is_rejected():
    with pytest.raises(ValueError):
        par.band_layout(300, 3, 2, 128)  # the last shard holds rows 256..300


def _stand_in_attention(qkv, q_w, k_w, cos, sin, mask, num_heads, head_dim, half, eps):
    """A torch fp32 form of the kernel's contract (RMSNorm -> bf16 -> RoPE from the lane tables -> bf16, masked
    v, two softmax branches, A - B), so the DiT's sharding can be checked on the CPU."""
    b, length, _ = qkv.shape
    q, k, v, qd, kd = qkv.float().view(b, length, 5, num_heads, head_dim).permute(2, 0, 3, 1, 4)
    d = torch.arange(head_dim)
    partner = torch.where(d < half, d + half, torch.where(d < 2 * half, d - half, d))

    def prep(t, w):
        t = (t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps) * w.float()).bfloat16().float()
        return (t * cos[:length, :head_dim] + t[..., partner] * sin[:length, :head_dim]).bfloat16().float()

    v = v * mask[:, None, :length, :1].float()

    def branch(a, c):
        return torch.softmax(prep(a, q_w) @ prep(c, k_w).transpose(-1, -2) / 8, -1) @ v

    out = branch(q, k) - branch(qd, kd)
    return out.permute(0, 2, 1, 3).reshape(b, length, num_heads * head_dim).bfloat16()


def _tiny_dit(group, split_batch=True):
    from hummingbird_b200.config import DiTConfig
    from hummingbird_b200.dit import ClipShape, DiT
    cfg = DiTConfig(embed_dim=512, num_heads=8, num_memory_tokens=8)
    shape = ClipShape(batch=2, latents=88, io_channels=16, context=8, context_dim=32, depth=2, steps=2)
    return DiT(cfg, shape, "cpu", group=group, attend=_stand_in_attention, glue="torch",
               split_batch=split_batch), shape


def _dit_inputs(shape):
    g = torch.Generator().manual_seed(7)
    cross = torch.randn(shape.batch, shape.context, shape.context_dim, generator=g)
    glob = torch.randn(shape.batch, shape.context_dim, generator=g)
    x = torch.randn(shape.batch, shape.io_channels, shape.latents, generator=g).bfloat16()
    return cross, glob, x


def _dit_worker(rank, world, split_batch):
    full, shape = _tiny_dit(None)
    cross, glob, x = _dit_inputs(shape)
    t = torch.tensor([0.7, 0.4]).bfloat16()  # a different timestep per batch row: the rows must not mix
    expect = full.forward(x, t, full.prepare_static(cross, glob)).float()
    model, _ = _tiny_dit(dist.group.WORLD, split_batch)
    got = model.gather_latents(model.forward(model.local_view(x), t, model.prepare_static(cross, glob))).float()
    assert got.shape == expect.shape
    rel = ((got - expect).norm() / expect.norm()).item()
    assert rel < 1e-2, f"rank {rank}: sharded DiT differs from the single-rank one (relative {rel:.2e})"
    if split_batch and world == 2:  # one batch row per rank, nothing split inside it: the same bits
        assert model.world == 1 and model.batch_range == (rank, rank + 1)
        assert torch.equal(got, expect)


@pytest.mark.parametrize("world,split_batch", [(2, True), (4, True), (8, True), (2, False), (4, False)])
def test_dit_sharding_gloo(world, split_batch):
    """One clip over 2 / 4 / 8 ranks equals one rank: batch rows over rank groups (no collective between them),
    then token rows + head pairs inside each group (two all-to-alls per block; at 8 ranks four per batch row, one
    head pair each); or token rows + head pairs over all ranks when the batch is not split."""
    _run(_dit_worker, world, split_batch)


def test_dit_sharding_rejects_uneven_pairs():
    from hummingbird_b200.config import DiTConfig
    from hummingbird_b200.dit import ClipShape, DiT

    class _Group:  # stands in for a 3-rank group; construction must fail before any collective
        pass

    import unittest.mock as mock
    with mock.patch.object(dist, "get_world_size", return_value=3), mock.patch.object(dist, "get_rank", return_value=0):
        with pytest.raises(ValueError):
            DiT(DiTConfig(embed_dim=512, num_heads=8), ClipShape(latents=88, depth=1), "cpu", group=_Group())
