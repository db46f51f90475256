"""Partitioning of the hot paths over the GPUs of one node (one process per GPU, torch.distributed).

* band attention — sequence sharding: rank r owns rows `shard_rows(L, N, r)` (128-aligned boundaries) and
  receives `window` halo rows from each neighbour before its kernel runs (`halo_exchange`: NCCL send/recv
  over NVLink; gloo on CPU in tests). The kernel then sees a buffer [halo_before | own | halo_after] with
  `q_begin = halo_before` and `pos0 = s0 - halo_before` (global RoPE positions).
* dense attention — head-pair sharding: rank r owns pairs `shard_pairs(P, N, r)` (uneven splits allowed,
  e.g. the reference's 12 pairs on 8 GPUs), computes them from its column slice of `to_qkv`, and
  `gather_pairs` all-gathers the (B, L, pairs * 128) pieces into the full (B, L, H * 64) output.
* clips — data parallel: rank r renders clips `shard_clips(n, N, r)`; no collective.
* the DiT denoiser of one clip — token rows `shard_tokens(L, N, r)` for every token-wise op (projections,
  adaLN, cross-attention, MLP) and head pairs `shard_pairs(P, N, r)` for the self-attention, switched by two
  all-to-alls per block (`tokens_to_pairs`, `pairs_to_tokens`): rank r sends each rank s the `to_qkv`
  columns of s's pairs for its own rows, and gets back its rows of every rank's attention output.

The reference has no parallelism at all (it runs one TPU chip); these follow the partitions its kernels
admit: head pairs are independent (dense_attention.py:126-127), band rows depend only on +-window rows
(band_attention.py:15-19).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_rows(length: int, world: int, rank: int, align: int = 128) -> tuple[int, int]:
    """Contiguous row range of `rank`: boundaries rounded to multiples of `align`, the last rank takes the rest."""
    tiles = -(-length // align)
    t0 = tiles * rank // world
    t1 = tiles * (rank + 1) // world
    return min(length, t0 * align), min(length, t1 * align)


def shard_pairs(pairs: int, world: int, rank: int) -> tuple[int, int]:
    """Head-pair range [begin, end) of `rank` (contiguous, sizes differ by at most one)."""
    return pairs * rank // world, pairs * (rank + 1) // world


def shard_tokens(length: int, world: int, rank: int) -> tuple[int, int]:
    """Token range [t0, t1) of `rank` for the DiT's token-wise ops (sizes differ by at most one)."""
    return length * rank // world, length * (rank + 1) // world


def dest_major_qkv_rows(heads: int, world: int) -> torch.Tensor:
    """Row order of `to_qkv` whose output columns are grouped by destination rank: rank s's block holds the
    q, k, v, q_diff, k_diff columns of its pairs (each block in the kernel's section order)."""
    pairs = heads // 2
    return torch.cat([qkv_columns_for_pairs(heads, *shard_pairs(pairs, world, s)) for s in range(world)])


def tokens_to_pairs(send: torch.Tensor, length: int, world: int, group=None) -> torch.Tensor:
    """All-to-all from token shards to head-pair shards.

    `send` is `(world, B, rows_r, C)`: block s holds this rank's rows of the `C` `to_qkv` columns of rank s's
    pairs (equal pair counts on every rank). Returns `(B, length, C)`: every row of this rank's pairs."""
    n, b, rows, c = send.shape
    lens = [t1 - t0 for t0, t1 in (shard_tokens(length, world, s) for s in range(world))]
    recv = send.new_empty(b * length * c)
    dist.all_to_all_single(recv, send.reshape(-1), [b * l * c for l in lens], [b * rows * c] * world, group=group)
    return torch.cat([blk.view(b, l, c) for blk, l in zip(recv.split([b * l * c for l in lens]), lens)], 1)


def pairs_to_tokens(att: torch.Tensor, length: int, world: int, rank: int, group=None) -> torch.Tensor:
    """All-to-all back: `att` `(B, length, W)` is this rank's pairs for every row; returns `(B, rows_r, world * W)`,
    this rank's rows of every rank's pairs in pair order (the full attention output of its rows)."""
    b, _, w = att.shape
    bounds = [shard_tokens(length, world, s) for s in range(world)]
    r0, r1 = bounds[rank]
    send = torch.cat([att[:, t0:t1].reshape(-1) for t0, t1 in bounds])
    recv = att.new_empty(world * b * (r1 - r0) * w)
    dist.all_to_all_single(recv, send, [b * (r1 - r0) * w] * world, [b * (t1 - t0) * w for t0, t1 in bounds],
                           group=group)
    return recv.view(world, b, r1 - r0, w).permute(1, 2, 0, 3).reshape(b, r1 - r0, world * w)


def shard_clips(n_clips: int, world: int, rank: int) -> range:
    return range(n_clips * rank // world, n_clips * (rank + 1) // world)


def band_layout(length: int, world: int, rank: int, window: int) -> dict:
    """Buffer layout of `rank`'s band-attention input: its own rows plus up to `window` halo rows each side.
    Every shard must be at least `window` rows long (a halo never spans more than one neighbour)."""
    s0, s1 = shard_rows(length, world, rank)
    if world > 1 and s1 - s0 < window:
        raise ValueError(f"shard of {s1 - s0} rows is shorter than the window ({window})")
    before = min(window, s0)
    after = min(window, length - s1)
    return {"s0": s0, "s1": s1, "before": before, "after": after, "rows": before + (s1 - s0) + after,
            "q_begin": before, "q_count": s1 - s0, "pos0": s0 - before, "length": length, "world": world,
            "window": window}


def halo_exchange(buf: torch.Tensor, layout: dict, rank: int, group=None, comm=None) -> None:
    """Fill the halo rows of `buf` (dim 1 = buffer rows, laid out as `band_layout`) from the neighbours.

    Rank r sends its first rows to r - 1 (that rank's trailing halo) and its last rows to r + 1 (that rank's
    leading halo), and receives its own halos the same way; all sends and receives of a rank are issued as
    one batched group. With `comm` (a `hummingbird_b200.comm.HbComm`) the exchange runs through the library's
    NCCL C ABI; otherwise through torch.distributed (NCCL on GPUs, gloo in the CPU tests)."""
    if comm is not None:
        comm.halo_exchange(buf, layout)
        return
    world, length, window = layout["world"], layout["length"], layout["window"]
    before, after = layout["before"], layout["after"]
    own0, own1 = before, layout["rows"] - after
    ops = []
    if rank > 0:
        left = band_layout(length, world, rank - 1, window)
        ops.append(dist.P2POp(dist.isend, buf[:, own0:own0 + left["after"]].contiguous(), rank - 1, group))
        ops.append(dist.P2POp(dist.irecv, buf[:, :before], rank - 1, group))
    if rank < world - 1:
        right = band_layout(length, world, rank + 1, window)
        ops.append(dist.P2POp(dist.isend, buf[:, own1 - right["before"]:own1].contiguous(), rank + 1, group))
        ops.append(dist.P2POp(dist.irecv, buf[:, own1:], rank + 1, group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()


def band_attention_sharded(qkv_own: torch.Tensor, q_norm, k_norm, inv_freq: torch.Tensor, num_heads: int,
                           window: int, length: int, rank: int, world: int, *, lam=None, group=None,
                           buf: torch.Tensor | None = None) -> torch.Tensor:
    """Band attention of this rank's rows `(B, s1 - s0, 5 H 64)` of a sequence sharded over `world` ranks."""
    from hummingbird_b200.band_attention import band_attention_shard
    lay = band_layout(length, world, rank, window)
    b, own, width = qkv_own.shape
    if own != lay["q_count"]:
        raise ValueError(f"rank {rank} holds {own} rows, its shard is {lay['q_count']}")
    if buf is None:
        buf = qkv_own.new_empty(b, lay["rows"], width)
    buf[:, lay["before"]:lay["before"] + own] = qkv_own
    halo_exchange(buf, lay, rank, group)
    return band_attention_shard(buf, q_norm, k_norm, inv_freq, num_heads, 64, window, q_begin=lay["q_begin"],
                                q_count=lay["q_count"], pos0=lay["pos0"], lam=lam)


def gather_pairs(local: torch.Tensor, pairs: int, world: int, group=None) -> torch.Tensor:
    """All-gather head-pair pieces `(B, L, (p1 - p0) * 128)` of every rank into `(B, L, pairs * 128)`."""
    sizes = [shard_pairs(pairs, world, r) for r in range(world)]
    counts = [(p1 - p0) for p0, p1 in sizes]
    b, length, _ = local.shape
    widest = max(counts) * 128
    padded = local.new_zeros(b, length, widest)
    padded[..., :local.shape[-1]] = local
    gathered = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(gathered, padded.contiguous(), group=group)
    return torch.cat([g[..., :c * 128] for g, c in zip(gathered, counts)], dim=-1)


def qkv_columns_for_pairs(heads: int, p0: int, p1: int, device=None) -> torch.Tensor:
    """Column indices of `to_qkv`'s output (sections q, k, v, q_diff, k_diff) that head pairs [p0, p1) use;
    index the `to_qkv` weight rows with them to compute only this rank's slice."""
    cols = [torch.arange(s * heads * 64 + p0 * 128, s * heads * 64 + p1 * 128) for s in range(5)]
    return torch.cat(cols).to(device)
