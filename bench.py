#!/usr/bin/env python
"""Benchmark of hummingbird-b200's hot paths on B200 (one JSON line on rank 0).

Headline (`value`): SAME-L differential band attention, BASELINE config 2 (B=1, L=82,688 rows per GPU,
d_model 512 = 8 heads, window +-128, bf16), in algorithmic TFLOP/s summed over ranks. A step is one pass of
the hot path over one batch: [halo exchange over NCCL when N > 1] + DyT/RoPE preparation + attention. At
N > 1 each rank owns an 82,688-row shard of one long sequence (weak scaling) and receives +-128 halo rows
from its neighbours with NCCL send/recv before its kernels run.

The SAME-L attention layer itself (`e2e_layer`): x -> block DyT pre-norm + to_qkv + q/k DyT + RoPE in one GEMM
-> the band kernel on the prepared projection -> to_out, device-resident and from pinned host memory, with its
own CPU baseline (the layer's oracle) and parity check.

Secondary paths (N = 1 only, reported under `paths`): dense DiT differential attention (config 1, and the
120 s clip's per-block call B=2, L=2,648, 16 heads) and the W8A8 GEMM pair (config 3).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl hb|reference]

`--impl reference` times the reference's path on the host cores instead: JAX (the reference's runtime) is
not installed, so it runs the fp32 CPU restatement in `oracle/` on a spawn pool over every core.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
METRIC = "diff-attn TFLOP/s & W8A8 int8 TOPS (% peak), ms per 120 s clip at 1/2/4/8 B200"
WINDOW = 128
L_PER_GPU = 82_688
HEADS = 8
# DRAM bytes per launch of band_fused_kernel on this workload, from the committed ncu capture (None until taken)
BAND_NCU_TRAFFIC = 506_192_128
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ----------------------------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (200 ms) while the timed loops run."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = None

    def start(self):
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
            time.sleep(1.0)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.file.seek(0)
        rows = [r.split(",") for r in self.file.read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.file.name)
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ----------------------------------------------------------------------------------------------- dist
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def init_dist(world: int, local: int):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return torch.device("cuda", local)


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t)
    return float(t.item())


def barrier(world: int):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


# ----------------------------------------------------------------------------------------------- band
def band_rank_inputs(device, rank: int):
    """Rank r's 82,688 rows of a long sequence: shared weights / norms / lambda (seed 1), rank 0's rows are
    exactly config 2, other ranks draw their rows from seed (1, r)."""
    from hummingbird_b200.workloads import band_inputs
    return band_inputs(device, seed=1, length=L_PER_GPU, d_model=512, heads=HEADS, window=WINDOW,
                       x_seed=None if rank == 0 else (1, rank))


class BandStep:
    """One step of the band hot path on this rank: halo exchange (N > 1), preparation, attention."""

    def __init__(self, device, rank: int, world: int, comm=None):
        import torch
        from hummingbird_b200 import band_attention as hb
        from hummingbird_b200 import parallel as par
        from hummingbird_b200._tensors import workspace
        self.torch, self.hb, self.par = torch, hb, par
        self.rank, self.world, self.comm = rank, world, comm
        self.w = band_rank_inputs(device, rank)
        self.lay = par.band_layout(L_PER_GPU * world, world, rank, WINDOW)
        assert self.lay["q_count"] == L_PER_GPU
        self.before = self.lay["before"]
        rows = self.lay["rows"]
        self.buf = torch.zeros(1, rows, 5 * HEADS * 64, dtype=torch.bfloat16, device=device)
        self.buf[:, self.before:self.before + L_PER_GPU] = self.w.qkv
        self.out = torch.empty(1, L_PER_GPU, HEADS * 64, dtype=torch.bfloat16, device=device)
        self.qn = hb.pack_norm(self.w.q_norm, device)
        self.kn = hb.pack_norm(self.w.k_norm, device)
        self.freqs = torch.from_numpy(self.w.inv_freq).to(device)
        self.lam = torch.from_numpy(self.w.lam).to(device)
        self.ws = workspace(hb.workspace_bytes(1, rows, HEADS // 2, WINDOW, len(self.w.inv_freq)), device)
        self.pos0 = self.lay["pos0"]
        self.flops = band_flops(L_PER_GPU * world, rank * L_PER_GPU, (rank + 1) * L_PER_GPU)
        self.launches = 1  # the fused band kernel (its prepare stage launches nothing for window <= 128)

    def exchange(self):
        if self.world > 1:
            self.par.halo_exchange(self.buf, self.lay, self.rank, comm=self.comm)

    def run(self, stages: int, out=None):
        self.hb.band_attention_shard(self.buf, self.qn, self.kn, self.freqs, HEADS, 64, WINDOW, q_begin=self.before,
                                     q_count=L_PER_GPU, pos0=self.pos0, lam=self.lam, out=self.out if out is None else out,
                                     ws=self.ws, stages=stages)


def band_flops(length: int, q0: int, q1: int) -> float:
    q = np.arange(q0, q1, dtype=np.int64)
    keys = np.minimum(length - 1, q + WINDOW) - np.maximum(0, q - WINDOW) + 1
    return float(2 * 2 * 2 * 64 * HEADS * keys.sum())


def time_band(step: BandStep, steps: int, warmup: int, world: int) -> dict:
    import torch
    from hummingbird_b200._lib import HB_STAGE_ATTEND, HB_STAGE_PREPARE
    stream = torch.cuda.current_stream()
    n_ev = steps + 1
    ev_start = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ev_mid = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ev_end = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for _ in range(warmup):
        step.exchange()
        step.run(HB_STAGE_PREPARE)
        step.run(HB_STAGE_ATTEND)
    barrier(world)
    t_begin = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_begin.record(stream)
    for i in range(steps):
        step.exchange()
        ev_start[i].record(stream)
        step.run(HB_STAGE_PREPARE)
        ev_mid[i].record(stream)
        step.run(HB_STAGE_ATTEND)
        ev_end[i].record(stream)
    t_end.record(stream)
    barrier(world)
    del n_ev
    total_ms = t_begin.elapsed_time(t_end)
    prep = [a.elapsed_time(b) for a, b in zip(ev_start, ev_mid)]
    attn = [a.elapsed_time(b) for a, b in zip(ev_mid, ev_end)]
    return {"ms_per_step": max_over_ranks(total_ms / steps, world),
            "prep_ms": statistics.mean(prep), "attn_ms": statistics.mean(attn)}


def time_band_e2e(step: BandStep, steps: int, warmup: int, world: int) -> dict:
    """Through the public API with host buffers (`band_attention_from_host`): the step's rows stream from
    pinned host memory in chunks, each chunk's queries run once their rows (and the window after them) have
    landed, the halo exchange runs on the device at N > 1, and finished rows stream back to pinned host
    memory, all inside the timed region."""
    import torch
    h_in = step.w.qkv.cpu().pin_memory()
    h_out = torch.empty(step.out.shape, dtype=torch.bfloat16).pin_memory()
    stream = torch.cuda.current_stream()

    def one():
        step.hb.band_attention_from_host(h_in, step.qn, step.kn, step.freqs, HEADS, 64, WINDOW, lam=step.lam,
                                         out_host=h_out, dev_in=step.buf, dev_out=step.out,
                                         layout=step.lay if world > 1 else None, comm=step.comm)

    for _ in range(warmup):
        one()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        one()
    b.record(stream)
    barrier(world)
    ms = max_over_ranks(a.elapsed_time(b) / steps, world)
    return {"ms_per_step": ms, "h2d": h_in.numel() * 2, "d2h": h_out.numel() * 2}


def _gather_rows(vals: list, world: int) -> list:
    """Every rank's list of floats, on every rank (rank order)."""
    if world == 1:
        return [vals]
    import torch
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t)
    return [p.tolist() for p in parts]


def band_parity(step: BandStep, world: int, edge: int = 384) -> dict:
    """Output check of the headline step on every rank, outside the timed region: the first and the last `edge`
    query rows this rank owns (at N > 1 these border the neighbouring shards, where the halo rows matter) against
    the fp32 oracle (`oracle/band.py`) evaluated on the rank's buffer slice holding those rows and +-window keys,
    at their global RoPE positions. Tolerance max-abs 2e-2, mean-abs 2e-3 (the north star's)."""
    import torch
    from hummingbird_b200._lib import HB_STAGE_ALL
    from oracle import band as oband
    step.exchange()
    step.run(HB_STAGE_ALL)
    torch.cuda.synchronize()
    before, own, rows = step.before, L_PER_GPU, step.buf.shape[1]
    w = step.w
    worst, means = 0.0, []
    for q0 in (0, own - edge):
        s0 = max(0, before + q0 - WINDOW)
        s1 = min(rows, before + q0 + edge + WINDOW)
        qkv = step.buf[:, s0:s1].float().cpu().numpy()
        ref = oband.band_diff_attention(qkv, w.q_norm, w.k_norm, w.inv_freq, HEADS, WINDOW, lam=w.lam,
                                        offset=step.pos0 + s0)
        a = before + q0 - s0
        got = step.out[:, q0:q0 + edge].float().cpu().numpy()
        diff = np.abs(got - ref[:, a:a + edge])
        worst = max(worst, float(diff.max()))
        means.append(float(diff.mean()))
    mine = [worst, float(np.mean(means)), float(worst <= 2e-2 and np.mean(means) <= 2e-3)]
    allr = _gather_rows(mine, world)
    return {"ok": all(r[2] == 1.0 for r in allr), "max_abs": max(r[0] for r in allr),
            "mean_abs": max(r[1] for r in allr), "per_rank": [[round(r[0], 5), round(r[1], 6)] for r in allr],
            "rows": f"first and last {edge} own rows per rank vs the fp32 oracle"}


# ----------------------------------------------------------------------------------------------- band layer
LAYER_SEED = 1


def band_layer_rank_inputs(device, rank: int):
    """The SAME-L attention layer's inputs at config 2 (x ~ N(0,1), to_qkv / to_out ~ N(0, 1/512), block DyT
    pre-norm and q/k DyT alpha 0.5, gamma 1 + N(0, 0.02), beta N(0, 0.02)); ranks > 0 draw other rows of the
    same sequence with the same weights."""
    from hummingbird_b200.workloads import band_layer_inputs
    return band_layer_inputs(device, seed=LAYER_SEED, length=L_PER_GPU, d_model=512, heads=HEADS, window=WINDOW,
                             x_seed=None if rank == 0 else (LAYER_SEED, rank))


class BandLayerStep:
    """`same_l._attention` of `_block` (same_l.py:151-161, 191) on this rank's 82,688 rows: the one-GEMM front
    end (block DyT pre-norm + to_qkv + q/k DyT + RoPE, `band_proj_kernel`) on the own rows, [the halo exchange of
    the prepared rows over NCCL at N > 1], the band kernel on the prepared projection, to_out (cuBLAS)."""

    def __init__(self, device, rank: int, world: int, comm=None):
        import torch
        from hummingbird_b200 import band_attention as hb
        from hummingbird_b200 import parallel as par
        self.torch, self.hb, self.par = torch, hb, par
        self.rank, self.world, self.comm = rank, world, comm
        self.w = band_layer_rank_inputs(device, rank)
        self.lay = par.band_layout(L_PER_GPU * world, world, rank, WINDOW)
        self.before = self.lay["before"]
        self.qkv = torch.zeros(1, self.lay["rows"], 5 * HEADS * 64, dtype=torch.bfloat16, device=device)
        self.att = torch.empty(1, L_PER_GPU, HEADS * 64, dtype=torch.bfloat16, device=device)
        self.out = torch.empty_like(self.att)
        self.qn, self.kn = hb.pack_norm(self.w.q_norm, device), hb.pack_norm(self.w.k_norm, device)
        self.pre = hb.pack_pre_norm(self.w.pre_norm, 512, device)
        self.freqs = torch.from_numpy(self.w.inv_freq).to(device)
        self.lam = torch.from_numpy(self.w.lam).to(device)
        self.flops = band_flops(L_PER_GPU * world, rank * L_PER_GPU, (rank + 1) * L_PER_GPU)
        self.proj_flops = 2.0 * L_PER_GPU * 512 * 5 * HEADS * 64

    def project(self):
        self.hb.qkv_project(self.w.x, self.w.to_qkv, self.qn, self.kn, self.freqs, HEADS, pre_norm=self.pre,
                            pos0=self.lay["pos0"] + self.before,
                            out=self.qkv[:, self.before:self.before + L_PER_GPU])

    def exchange(self):
        if self.world > 1:
            self.par.halo_exchange(self.qkv, self.lay, self.rank, comm=self.comm)

    def attend(self):
        self.hb.band_attention_prepared(self.qkv, HEADS, WINDOW, q_begin=self.before, q_count=L_PER_GPU,
                                        lam=self.lam, out=self.att)

    def to_out(self):
        self.torch.matmul(self.att[0], self.w.to_out.t(), out=self.out[0])


def time_band_layer(step: BandLayerStep, steps: int, warmup: int, world: int) -> dict:
    """Device-resident layer step (x in HBM): per-stage CUDA events on the launching stream, max over ranks."""
    import torch
    stream = torch.cuda.current_stream()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]
    for _ in range(warmup):
        step.project()
        step.exchange()
        step.attend()
        step.to_out()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(steps):
        ev[i][0].record(stream)
        step.project()
        ev[i][1].record(stream)
        step.exchange()
        step.attend()
        ev[i][2].record(stream)
        step.to_out()
        ev[i][3].record(stream)
    b.record(stream)
    barrier(world)
    proj = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    attn = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
    out = statistics.mean(e[2].elapsed_time(e[3]) for e in ev)
    return {"ms_per_step": max_over_ranks(a.elapsed_time(b) / steps, world), "proj_ms": proj,
            "attn_ms": attn, "to_out_ms": out}


def time_band_layer_e2e(step: BandLayerStep, steps: int, warmup: int, world: int) -> dict:
    """Through the public API with host buffers (`same_l_attention_from_host`): the layer input x streams from
    pinned host memory in chunks, is projected on the device (front end), the band kernel and to_out run per
    chunk, the output streams back to pinned host memory, all inside the timed region. Only x (85 MB) and the
    output (85 MB) cross PCIe."""
    import torch
    x_host = step.w.x.cpu().pin_memory()
    h_out = torch.empty(step.out.shape, dtype=torch.bfloat16).pin_memory()
    stream = torch.cuda.current_stream()
    dev_x = torch.empty_like(step.w.x)

    def one():
        step.hb.same_l_attention_from_host(x_host, step.w.to_qkv, step.qn, step.kn, step.freqs, HEADS, WINDOW,
                                           to_out=step.w.to_out, pre_norm=step.pre, lam=step.lam, out_host=h_out,
                                           dev_x=dev_x, dev_qkv=step.qkv, dev_att=step.att, dev_out=step.out,
                                           layout=step.lay if world > 1 else None, comm=step.comm)

    for _ in range(warmup):
        one()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        one()
    b.record(stream)
    barrier(world)
    ms = max_over_ranks(a.elapsed_time(b) / steps, world)
    return {"ms_per_step": ms, "h2d": x_host.numel() * 2, "d2h": h_out.numel() * 2}


def layer_parity(step: BandLayerStep, world: int, edge: int = 384) -> dict:
    """Output check of the layer step on every rank, outside the timed region: the band output (before to_out)
    of the first and last `edge` own rows against the oracle run from x (`oracle.band.front_end`: pre-norm +
    to_qkv; then the band attention), the neighbours' x rows at shard edges regenerated from their seeds.
    Tolerance max-abs 2e-2, mean-abs 2e-3."""
    import torch
    from oracle import band as oband
    step.project()
    step.exchange()
    step.attend()
    torch.cuda.synchronize()
    own_x = step.w.x[0].float().cpu().numpy()
    glob = L_PER_GPU * world
    g_own = step.rank * L_PER_GPU
    neighbours = {}

    def x_rows(g0: int, g1: int) -> np.ndarray:
        parts = []
        for r in range(g0 // L_PER_GPU, (g1 - 1) // L_PER_GPU + 1):
            lo, hi = max(g0, r * L_PER_GPU) - r * L_PER_GPU, min(g1, (r + 1) * L_PER_GPU) - r * L_PER_GPU
            if r == step.rank:
                parts.append(own_x[lo:hi])
            else:
                if r not in neighbours:
                    neighbours[r] = band_layer_rank_inputs("cpu", r).x[0].float().numpy()
                parts.append(neighbours[r][lo:hi])
        return np.concatenate(parts)[None]

    worst, means = 0.0, []
    for q0 in (0, L_PER_GPU - edge):
        g0, g1 = max(0, g_own + q0 - WINDOW), min(glob, g_own + q0 + edge + WINDOW)
        qkv = oband.front_end(x_rows(g0, g1), step.w.to_qkv.float().cpu().numpy(), step.w.pre_norm)
        ref = oband.band_diff_attention(qkv, step.w.q_norm, step.w.k_norm, step.w.inv_freq, HEADS, WINDOW,
                                        lam=step.w.lam, offset=g0)
        a = g_own + q0 - g0
        got = step.att[:, q0:q0 + edge].float().cpu().numpy()
        diff = np.abs(got - ref[:, a:a + edge])
        worst = max(worst, float(diff.max()))
        means.append(float(diff.mean()))
    mine = [worst, float(np.mean(means)), float(worst <= 2e-2 and np.mean(means) <= 2e-3)]
    allr = _gather_rows(mine, world)
    return {"ok": all(r[2] == 1.0 for r in allr), "max_abs": max(r[0] for r in allr),
            "mean_abs": max(r[1] for r in allr), "per_rank": [[round(r[0], 5), round(r[1], 6)] for r in allr],
            "rows": f"first and last {edge} own rows per rank, band output vs the oracle from x"}


def cpu_layer_baseline(w, q_rows: int, min_seconds: float = 10.0) -> dict:
    """The layer's oracle (front end + band + to_out) on the host cores over queries [0, q_rows) of the rank-0
    workload, repeated until at least `min_seconds` of wall time have been measured."""
    sys.path.insert(0, str(ROOT))
    from oracle.cpu_baseline import time_layer_sample
    rows = min(L_PER_GPU, q_rows + WINDOW)
    x = w.x[:, :rows].float().cpu().numpy()
    r = time_layer_sample(x, w.to_qkv.float().cpu().numpy(), w.to_out.float().cpu().numpy(), w.pre_norm, w.q_norm,
                          w.k_norm, w.inv_freq, HEADS, WINDOW, w.lam, q_rows, min_seconds=min_seconds)
    return {"value": r["flops"] / r["seconds"] / 1e12, "unit": "TFLOP/s", "cores": r["cores"], "kind": "port",
            "sample": f"layer (pre-norm + to_qkv, band attention, to_out) over queries 0..{q_rows} of config 2 x "
                      f"{r['passes']} passes, fp32 numpy oracle, {r['cores']}-process spawn pool, "
                      f"{r['seconds']:.1f} s; attention FLOPs counted"}


# ----------------------------------------------------------------------------------------------- dense
def _flush_l2(flush) -> None:
    """Evict L2 by reading a buffer twice its size: a read leaves the lines clean, so the timed call that follows
    does not pay for writing back the flush (a zero-fill would leave 126 MB of dirty lines behind)."""
    flush.sum()


def _event_median(fn, steps: int, warmup: int, flush) -> float:
    """Median CUDA-event time of `fn` on the current stream, L2 flushed before each call. A ~0.5 ms GPU sleep
    between the flush and the start event keeps the GPU busy while the host enqueues the call, so the
    interval holds the device work of `fn` and not the host's launch latency."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    stream = torch.cuda.current_stream()
    for _ in range(steps):
        _flush_l2(flush)
        torch.cuda._sleep(1_000_000)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        times.append((a, b))
    torch.cuda.synchronize()
    return statistics.median(a.elapsed_time(b) for a, b in times)


def time_dense(device, steps: int, warmup: int, batch: int, length: int, heads: int, d_model: int) -> dict:
    import torch
    from hummingbird_b200 import dense_attention as hb
    from hummingbird_b200.workloads import dense_inputs
    w = dense_inputs(device, batch=batch, length=length, d_model=d_model, heads=heads)
    cos, sin, mask = hb.tables(length, torch.from_numpy(w.inv_freq).to(device), torch.from_numpy(w.valid).to(device))
    qw, kw = torch.from_numpy(w.q_weight).to(device), torch.from_numpy(w.k_weight).to(device)
    lam = torch.from_numpy(w.lam).to(device)
    out = torch.empty(batch, length, heads * 64, dtype=torch.bfloat16, device=device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)  # > L2 (126 MB)

    def one():
        hb.dense_attention(w.qkv, qw, kw, cos, sin, mask, heads, 64, w.half, w.eps, lam=lam, out=out)

    ms = _event_median(one, steps, warmup, flush)
    flops = 8.0 * batch * heads * length * length * 64
    return {"config": {"batch": batch, "length": length, "heads": heads}, "ms": ms,
            "tflops": flops / (ms * 1e-3) / 1e12, "launches_per_call": 2, "l2": "flushed (256 MB read) before each call"}


def time_cross(device, steps: int, warmup: int, hbm_peak: float, batch: int = 2, length: int = 2648,
               heads: int = 16, context: int = 128) -> dict:
    """The DiT's differential cross-attention per block call (120 s clip shape): this library's kernel against
    the torch ops it replaces in the DiT (q RMSNorm, two cuDNN/flash SDPA calls, subtraction, head merge)."""
    import torch
    import torch.nn.functional as F
    from hummingbird_b200.cross_attention import cross_attention, cross_kv
    g = torch.Generator(device=device).manual_seed(7)
    width = heads * 64
    q2 = torch.randn(batch, length, 2 * width, generator=g, device=device).to(torch.bfloat16)
    kv = cross_kv(torch.randn(batch, context, 3 * width, generator=g, device=device).to(torch.bfloat16),
                  1 + 0.02 * torch.randn(64, generator=g, device=device), heads, 1e-6)
    qw = (1 + 0.02 * torch.randn(64, generator=g, device=device)).to(torch.bfloat16)
    out = torch.empty(batch, length, width, dtype=torch.bfloat16, device=device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)  # > L2 (126 MB)
    qwf = qw.float()
    ms = _event_median(lambda: cross_attention(q2, kv, qwf, None, heads, 64, 1e-6, out=out), steps, warmup, flush)
    k, kd, v = (t.unflatten(-1, (heads, 64)).transpose(1, 2) for t in kv.chunk(3, -1))

    def torch_ops():
        q = F.rms_norm(q2.view(batch, length, 2, heads, 64), (64,), qw, 1e-6)
        a, b = q[:, :, 0].transpose(1, 2), q[:, :, 1].transpose(1, 2)
        o = F.scaled_dot_product_attention(a, k, v) - F.scaled_dot_product_attention(b, kd, v)
        return o.transpose(1, 2).reshape(batch, length, width)

    ms_torch = _event_median(torch_ops, steps, warmup, flush)
    nbytes = 2 * (batch * length * 2 * width + batch * context * 3 * width + batch * length * width)
    flops = 8.0 * batch * heads * length * context * 64
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"config": {"batch": batch, "q_len": length, "kv_len": context, "heads": heads}, "ms": ms,
            "gbs": gbs, "hbm_frac": gbs / hbm_peak, "tflops": flops / (ms * 1e-3) / 1e12,
            "algorithmic_bytes": nbytes, "launches_per_call": 1, "torch_ops_ms": ms_torch,
            "l2": "flushed (256 MB read) before each call"}


# ----------------------------------------------------------------------------------------------- w8a8
def int8_peak(device) -> float:
    import torch
    a = torch.randint(-127, 127, (8192, 8192), dtype=torch.int8, device=device)
    b = torch.randint(-127, 127, (8192, 8192), dtype=torch.int8, device=device).T
    for _ in range(3):
        torch._int_mm(a, b)
    torch.cuda.synchronize()
    best = 1e9
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch._int_mm(a, b)
        e.record()
        torch.cuda.synchronize()
        best = min(best, s.elapsed_time(e))
    return 2 * 8192 ** 3 / (best * 1e-3) / 1e12


def time_w8a8(device, steps: int, warmup: int) -> dict:
    import torch
    from hummingbird_b200.w8a8 import W8A8Linear, quantize_rows, w8a8_gemm
    from hummingbird_b200.workloads import w8a8_inputs
    w = w8a8_inputs(device)
    l1, l2 = W8A8Linear(w.w1, w.b1), W8A8Linear(w.w2, w.b2)
    m = w.x.shape[0]
    q1 = torch.empty(m, 1024, dtype=torch.int8, device=device)
    s1 = torch.empty(m, dtype=torch.float32, device=device)
    h = torch.empty(m, 4096, dtype=torch.bfloat16, device=device)
    q2 = torch.empty(m, 4096, dtype=torch.int8, device=device)
    s2 = torch.empty(m, dtype=torch.float32, device=device)
    y = torch.empty(m, 1024, dtype=torch.bfloat16, device=device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(steps)]

    def one(e=None):
        if e: e[0].record(stream)
        quantize_rows(w.x, q1, s1)
        if e: e[1].record(stream)
        w8a8_gemm(q1, s1, l1.qw, l1.sw, l1.bias, out=h)
        if e: e[2].record(stream)
        quantize_rows(h, q2, s2)
        if e: e[3].record(stream)
        w8a8_gemm(q2, s2, l2.qw, l2.sw, l2.bias, out=y)
        if e: e[4].record(stream)

    for _ in range(warmup):
        one()
    torch.cuda.synchronize()
    for i in range(steps):
        _flush_l2(flush)
        torch.cuda._sleep(1_000_000)  # the GPU waits ~0.5 ms while the host enqueues the four launches
        one(ev[i])
    torch.cuda.synchronize()
    med = lambda j, k: statistics.median(e[j].elapsed_time(e[k]) for e in ev)  # noqa: E731
    g1, g2, total = med(1, 2), med(3, 4), med(0, 4)
    ops = 2.0 * m * 1024 * 4096
    peak = int8_peak(device)
    return {"config": {"M": m, "gemm1": "1024->4096", "gemm2": "4096->1024"}, "ms_pair_with_quant": total,
            "gemm1_ms": g1, "gemm2_ms": g2, "gemm1_tops": ops / (g1 * 1e-3) / 1e12,
            "gemm2_tops": ops / (g2 * 1e-3) / 1e12, "pair_tops": 2 * ops / (total * 1e-3) / 1e12,
            "int8_peak_tops_measured": peak, "gemm1_frac_of_int8_peak": ops / (g1 * 1e-3) / 1e12 / peak,
            "int8_peak_how": "torch._int_mm 8192^3, best of 10 (burst)", "launches_per_pair": 4,
            "l2": "flushed (256 MB read) before each pair"}


def time_w8a8_glu_mlp(device, steps: int, warmup: int) -> dict:
    """The DiT's W8A8 MLP at the 120 s clip's shape (M = 5,296 tokens, 1,024 -> 2 x 4,096 GLU -> 1,024): the GLU in
    the first GEMM's epilogue (`hb_w8a8_gemm_glu`, then the row quantiser) against the separate GLU + quantise
    kernel after a plain GEMM. Same bits out (tested); L2 flushed before each MLP call."""
    import torch
    from hummingbird_b200 import dit_glue
    from hummingbird_b200.w8a8 import W8A8GluLinear, W8A8Linear, quantize_rows, w8a8_gemm
    g = torch.Generator(device=device).manual_seed(12)
    m, d, f = 5296, 1024, 4096
    x = torch.randn(m, d, generator=g, device=device).to(torch.bfloat16)
    w1 = (torch.randn(2 * f, d, generator=g, device=device) / d ** 0.5).to(torch.bfloat16)
    w2 = (torch.randn(d, f, generator=g, device=device) / f ** 0.5).to(torch.bfloat16)
    plain, fused, l2 = W8A8Linear(w1), W8A8GluLinear(w1), W8A8Linear(w2)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)

    def unfused():
        q, s = dit_glue.glu(plain(x), quantize=True)
        return w8a8_gemm(q, s, l2.qw, l2.sw)

    def with_epilogue():
        q, s = quantize_rows(fused(x))
        return w8a8_gemm(q, s, l2.qw, l2.sw)

    ms_u = _event_median(unfused, steps, warmup, flush)
    ms_f = _event_median(with_epilogue, steps, warmup, flush)
    ops = 2.0 * m * d * 2 * f + 2.0 * m * f * d
    return {"config": {"M": m, "d": d, "F": f}, "ms_glu_in_epilogue": ms_f, "ms_separate_glu": ms_u,
            "tops_glu_in_epilogue": ops / (ms_f * 1e-3) / 1e12, "launches": "4 (quantise x, GEMM1+GLU, quantise z, "
            "GEMM2) vs 4 (quantise x, GEMM1, GLU+quantise, GEMM2)", "l2": "flushed (256 MB read) before each call"}


# ----------------------------------------------------------------------------------------------- DiT clip
def _dit_clip_runner(model, shape, device, seed: int = 44):
    """Inputs of one clip and a `clip()` that denoises it: the whole 8-step denoise loop captured in one CUDA graph
    (`DiT.denoise_graph`; NCCL all-to-alls included when the clip is split over ranks inside a batch group),
    replayed once per clip. Returns `clip` and the objects the graph reads (the graph itself, the per-clip static
    tensors): the caller keeps them alive while it replays and releases them together."""
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    static = model.prepare_static(torch.randn(shape.batch, shape.context, shape.context_dim, generator=g, device=device),
                                  torch.randn(shape.batch, shape.context_dim, generator=g, device=device))
    x_full = torch.randn(shape.batch, shape.io_channels, shape.latents, generator=g, device=device).to(torch.bfloat16)
    eps = model.local_view(torch.randn(shape.steps, shape.batch, shape.io_channels, shape.latents, generator=g,
                                       device=device).to(torch.bfloat16))
    x0 = model.local_view(x_full)
    x_in = x0.clone()
    run, graph = model.denoise_graph(x_in, eps, static, shape.steps)

    def clip():
        x_in.copy_(x0)
        return run()

    return clip, (graph, static, eps, x_in)


def time_dit_clip(device, ff_quant: str, world: int = 1, clips: int = 3, qkv_quant: str = "none",
                  out_quant: str = "none") -> dict:
    """Config 4: a whole 120 s clip (B=2 CFG pair, 2,584 latents + 64 memory tokens, 24 blocks, 8 pingpong
    steps, random weights) through `hummingbird_b200.dit`, split over `world` GPUs when world > 1: the batch
    rows over two rank groups, then token rows + head pairs inside a group (two NCCL all-to-alls per block).
    Returns ms per clip (max over ranks)."""
    import torch
    import torch.distributed as dist
    from hummingbird_b200.config import DiTConfig
    from hummingbird_b200.dit import DiT, ClipShape
    shape = ClipShape()
    model = DiT(DiTConfig(ff_quant=ff_quant, qkv_quant=qkv_quant, out_quant=out_quant), shape, device,
                group=dist.group.WORLD if world > 1 else None)
    clip, held = _dit_clip_runner(model, shape, device)
    clip()
    barrier(world)
    torch.cuda.synchronize()
    times = []
    for _ in range(clips):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(world)
        a.record()
        x = clip()
        b.record()
        torch.cuda.synchronize()
        times.append(max_over_ranks(a.elapsed_time(b), world))
    finite = bool(torch.isfinite(x.float()).all())
    del clip, held
    torch.cuda.synchronize()
    parity = dit_split_parity(model, shape, device, world, ff_quant) if world > 1 else None
    return {"ms_per_clip": statistics.median(times), "n_gpus": world, "parity": parity,
            "config": "120 s clip: B=2 (CFG), 2,584 latents + 64 memory, 24 blocks, d 1024, 16 heads, 8 pingpong "
                      "steps, 128 context tokens, random weights",
            "mlp": "W8A8" if ff_quant == "w8a8" else "bf16 cuBLAS", "finite": finite,
            "to_qkv": "W8A8 (input quantised by the pre-norm kernel)" if qkv_quant == "w8a8" else "bf16 cuBLAS",
            "to_out": "W8A8 (attention output quantised per token)" if out_quant == "w8a8" else "bf16 cuBLAS",
            "glue": "fused row kernels (residual + RMSNorm + adaLN, GLU + quantise) and the fused "
                    "differential cross-attention kernel",
            "parallelism": (f"one clip over {world} GPUs: the 2 batch rows over 2 groups of {world // 2} "
                            "(no collective between them)" + (f"; inside each group token rows x{world // 2}, "
                            f"self-attention head pairs x{world // 2}, 2 NCCL all-to-alls per block"
                            if world > 2 else "")) if world > 1 else "single GPU",
            "how": "the whole 8-step denoise loop captured in one CUDA graph, one replay per clip; CUDA events, max "
                   "over ranks"}


def dit_split_parity(model, shape, device, world: int, ff_quant: str) -> dict:
    """The split clip's result checked outside the timed region: one denoise step of the model split over the
    ranks (all ranks, gathered) against the same step of the unsplit model (same seed, so the same weights) on
    rank 0 alone, on seeded inputs. Relative L2 difference < 2e-2 and max-abs reported (bf16 activations through
    24 blocks; the two runs use different GEMM shapes, so they agree to rounding, not bit for bit)."""
    import torch
    import torch.distributed as dist
    from hummingbird_b200.config import DiTConfig
    from hummingbird_b200.dit import DiT
    g = torch.Generator(device=device).manual_seed(77)
    cross = torch.randn(shape.batch, shape.context, shape.context_dim, generator=g, device=device)
    glob = torch.randn(shape.batch, shape.context_dim, generator=g, device=device)
    x = torch.randn(shape.batch, shape.io_channels, shape.latents, generator=g, device=device).to(torch.bfloat16)
    eps = torch.randn(shape.batch, shape.io_channels, shape.latents, generator=g, device=device).to(torch.bfloat16)
    t = torch.full((shape.batch,), 0.9, device=device, dtype=torch.bfloat16)
    tn = torch.full((shape.batch,), 0.5, device=device, dtype=torch.bfloat16)
    got = model.gather_latents(model.step(model.local_view(x), t, tn, model.local_view(eps),
                                          model.prepare_static(cross, glob))).float()
    res = torch.zeros(3, dtype=torch.float64, device=device)
    if dist.get_rank() == 0:
        single = DiT(DiTConfig(ff_quant=ff_quant), shape, device)
        expect = single.step(x, t, tn, eps, single.prepare_static(cross, glob)).float()
        rel = ((got - expect).norm() / expect.norm()).item()
        res[0], res[1] = rel, (got - expect).abs().max().item()
        res[2] = float(bool(torch.isfinite(got).all()) and rel < 2e-2)
        del single
    dist.broadcast(res, 0)
    torch.cuda.synchronize()
    return {"ok": bool(res[2].item() == 1.0), "rel_l2": res[0].item(), "max_abs": res[1].item(),
            "check": "one denoise step split over the ranks vs the unsplit model on one GPU"}


SONG_LATENTS = 8184           # 380 s of audio
SONG_BAND_ROWS = 261_888      # SAME-L decoder rows of a 380 s clip
SONG_CLIPS = 8
SONG_DECODER_LAYERS = 12


def _song_band_layers(device, n_layers: int):
    """`n_layers` SAME-L attention layers (d_model 512, 8 heads, window +-128) with random weights."""
    import torch
    from hummingbird_b200.workloads import inv_freq
    g = torch.Generator(device=device).manual_seed(9)
    layers = []
    for _ in range(n_layers):
        def norm():
            return {"alpha": torch.tensor(0.5), "gamma": 1 + 0.02 * torch.randn(64, generator=g, device=device),
                    "beta": 0.02 * torch.randn(64, generator=g, device=device)}
        layers.append({"self_attn": {"to_qkv": {"weight": (torch.randn(5 * 512, 512, generator=g, device=device)
                                                           / 512 ** 0.5).to(torch.bfloat16)},
                                     "to_out": {"weight": (torch.randn(512, 512, generator=g, device=device)
                                                           / 512 ** 0.5).to(torch.bfloat16)},
                                     "q_norm": norm(), "k_norm": norm()},
                       "rope_inv_freq": torch.from_numpy(inv_freq(16)).to(device)})
    return layers


def time_song(device, world: int, rank: int) -> dict:
    """Config 5: a batch of 8 independent 380 s clips, clip-parallel over `world` GPUs (rank r renders clips
    `shard_clips(8, world, r)`, no collective). Per clip: the DiT denoise at 8,184 latents (+64 memory
    tokens, 24 blocks, 8 steps, W8A8 MLP, CUDA graph) and the 12 SAME-L attention layers of the decoder at
    261,888 rows (to_qkv -> fused band kernel -> to_out). Returns ms for the batch (max over ranks)."""
    import torch
    from hummingbird_b200 import blocks, parallel as par
    from hummingbird_b200.config import DiTConfig, SameConfig
    from hummingbird_b200.dit import DiT, ClipShape
    shape = ClipShape(latents=SONG_LATENTS)
    model = DiT(DiTConfig(ff_quant="w8a8"), shape, device)
    clip, held = _dit_clip_runner(model, shape, device, seed=45)
    layers = _song_band_layers(device, SONG_DECODER_LAYERS)
    scfg = SameConfig(channels=512, c_mults=(1,), stride=127)  # d 512, 8 heads, window (sub_chunk_size) 128
    x = torch.randn(1, SONG_BAND_ROWS, 512, generator=torch.Generator(device=device).manual_seed(46),
                    device=device).to(torch.bfloat16)

    def decoder():
        y = x
        for layer in layers:
            y = blocks.same_l_attention(y, layer, scfg)
        return y

    mine = par.shard_clips(SONG_CLIPS, world, rank)
    clip()
    decoder()  # warm-up
    barrier(world)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    dit_ms = dec_ms = 0.0
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in mine:
        ev[0].record()
        lat = clip()
        ev[1].record()
        y = decoder()
        ev[2].record()
        torch.cuda.synchronize()
        dit_ms += ev[0].elapsed_time(ev[1])
        dec_ms += ev[1].elapsed_time(ev[2])
    b.record()
    torch.cuda.synchronize()
    total = max_over_ranks(a.elapsed_time(b), world)
    finite = {"dit": bool(torch.isfinite(lat.float()).all()), "decoder": bool(torch.isfinite(y.float()).all())}
    del clip, held
    torch.cuda.synchronize()
    n = max(1, len(mine))
    return {"ms_per_batch_of_8": total, "clips_per_s": SONG_CLIPS / (total * 1e-3), "n_gpus": world,
            "dit_ms_per_clip": dit_ms / n, "decoder_attention_ms_per_clip": dec_ms / n, "finite": finite,
            "config": "380 s song: 8 clips; per clip DiT B=2 (CFG), 8,184 latents + 64 memory, 24 blocks, d 1024, "
                      "16 heads, 8 pingpong steps, W8A8 MLP; 12 SAME-L attention layers at 261,888 rows, d 512, "
                      "8 heads, window +-128 (pre-normed input, to_qkv + band kernel + to_out); random weights",
            "parallelism": f"clips data-parallel over {world} GPUs" if world > 1 else "single GPU, clips in sequence"}


def time_band_song_layer(device, world: int, rank: int, steps: int = 20, warmup: int = 3, comm=None) -> dict:
    """Config 5's band attention, one layer at L = 261,888 (window +-128, 8 heads) sequence-sharded over
    `world` GPUs (strong scaling): each rank's rows plus a 128-row halo per side by NCCL send/recv, then the
    fused kernel. Returns ms per layer (halo exchange included; max over ranks) and TFLOP/s of all ranks."""
    import torch
    from hummingbird_b200 import band_attention as hb
    from hummingbird_b200 import parallel as par
    from hummingbird_b200.workloads import band_inputs
    lay = par.band_layout(SONG_BAND_ROWS, world, rank, WINDOW)
    w = band_inputs(device, seed=1, length=lay["q_count"], d_model=512, heads=HEADS, window=WINDOW,
                    x_seed=(2, rank))
    buf = torch.zeros(1, lay["rows"], 5 * HEADS * 64, dtype=torch.bfloat16, device=device)
    buf[:, lay["before"]:lay["before"] + lay["q_count"]] = w.qkv
    out = torch.empty(1, lay["q_count"], HEADS * 64, dtype=torch.bfloat16, device=device)
    qn, kn = hb.pack_norm(w.q_norm, device), hb.pack_norm(w.k_norm, device)
    freqs, lam = torch.from_numpy(w.inv_freq).to(device), torch.from_numpy(w.lam).to(device)

    def one():
        if world > 1:
            par.halo_exchange(buf, lay, rank, comm=comm)
        hb.band_attention_shard(buf, qn, kn, freqs, HEADS, 64, WINDOW, q_begin=lay["q_begin"], q_count=lay["q_count"],
                                pos0=lay["pos0"], lam=lam, out=out)

    for _ in range(warmup):
        one()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        one()
    b.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(a.elapsed_time(b) / steps, world)
    flops = band_flops(SONG_BAND_ROWS, 0, SONG_BAND_ROWS)
    return {"ms_per_layer": ms, "tflops": flops / (ms * 1e-3) / 1e12, "n_gpus": world,
            "rows_per_gpu": lay["q_count"], "scaling": "strong",
            "config": "SAME-L band differential attention at L=261,888 (380 s), d_model 512 (8 heads), window +-128",
            "parallelism": f"sequence-sharded x{world}, NCCL halo send/recv" if world > 1 else "single GPU"}


# ----------------------------------------------------------------------------------------------- CPU baseline
def cpu_band_baseline(qkv_dev, w, q_rows: int, min_seconds: float = 10.0) -> dict:
    """The oracle port on the host cores over queries [0, q_rows) of the rank-0 workload, repeated until at
    least `min_seconds` of wall time have been measured."""
    sys.path.insert(0, str(ROOT))
    from oracle.cpu_baseline import time_band_sample
    q_rows = min(q_rows, qkv_dev.shape[1])
    rows = min(qkv_dev.shape[1], q_rows + WINDOW)
    qkv = qkv_dev[:, :rows].float().cpu().numpy()
    r = time_band_sample(qkv, w.q_norm, w.k_norm, w.inv_freq, HEADS, WINDOW, w.lam, q_rows, min_seconds=min_seconds)
    return {"value": r["flops"] / r["seconds"] / 1e12, "unit": "TFLOP/s", "cores": r["cores"], "kind": "port",
            "sample": f"queries 0..{q_rows} of config 2 (8 heads, window 128) x {r['passes']} passes, fp32 numpy "
                      f"oracle, {r['cores']}-process spawn pool, {r['seconds']:.1f} s"}


# The workload both arms time (the reference arm on the host cores in fp32, this library in bf16 on the GPU).
WORKLOAD = ("SAME-L band differential attention, config 2 per GPU: B=1, L=82,688 rows/GPU, d_model 512 (8 heads x "
            "64), window +-128, DyT + RoPE(half 16), bf16")


def run_reference(args, result_out):
    """`--impl reference`: the reference's path (its fp32 restatement; JAX is absent) on the host cores."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT))
    import torch
    from hummingbird_b200.workloads import band_inputs
    from oracle.cpu_baseline import shutdown, time_band_sample
    w = band_inputs("cpu", seed=1, length=L_PER_GPU, d_model=512, heads=HEADS, window=WINDOW)
    q_rows = L_PER_GPU  # each step: the whole config-2 call
    qkv = w.qkv[:, :q_rows + WINDOW].float().numpy()
    for _ in range(args.warmup):
        time_band_sample(qkv, w.q_norm, w.k_norm, w.inv_freq, HEADS, WINDOW, w.lam, q_rows)
    secs, cores = 0.0, 0
    for _ in range(args.steps):
        r = time_band_sample(qkv, w.q_norm, w.k_norm, w.inv_freq, HEADS, WINDOW, w.lam, q_rows)
        secs += r["seconds"]
        cores = r["cores"]
    shutdown()
    flops = band_flops(L_PER_GPU, 0, q_rows)
    value = flops * args.steps / secs / 1e12
    line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": secs / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                             "sample": f"{q_rows} queries per step; JAX absent, fp32 numpy restatement of the "
                                       "reference XLA path (oracle/band.py)"},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    del torch, world
    print(json.dumps(line), file=result_out, flush=True)


def paths_summary(paths: dict, peaks: dict) -> dict:
    """One short string per secondary path: time, rate and fraction of the measured peak."""
    bf16 = peaks["bf16_tflops"]
    out = {}
    for key, name in (("dense_config1", "dense_c1"), ("dense_120s_block_call", "dense_120s_block")):
        if key in paths:
            d = paths[key]
            out[name] = f"{d['ms']:.4f} ms {d['tflops']:.0f} TFLOP/s {d['tflops'] / bf16:.1%} bf16"
    if "cross_120s_block_call" in paths:
        d = paths["cross_120s_block_call"]
        out["cross_120s_block"] = f"{d['ms']:.4f} ms {d['gbs']:.0f} GB/s {d['hbm_frac']:.1%} HBM"
    if "w8a8_config3" in paths:
        d = paths["w8a8_config3"]
        pk = d["int8_peak_tops_measured"]
        out["w8a8_c3"] = (f"g1 {d['gemm1_ms'] * 1e3:.1f} us {d['gemm1_tops']:.0f} TOPS {d['gemm1_tops'] / pk:.0%}; "
                          f"g2 {d['gemm2_ms'] * 1e3:.1f} us {d['gemm2_tops']:.0f} TOPS {d['gemm2_tops'] / pk:.0%}")
    if "w8a8_dit_mlp" in paths:
        d = paths["w8a8_dit_mlp"]
        out["w8a8_mlp_120s"] = f"GLU in epilogue {d['ms_glu_in_epilogue'] * 1e3:.1f} us vs {d['ms_separate_glu'] * 1e3:.1f} us"
    for key, name in (("dit_120s_clip_bf16_mlp", "dit_120s_bf16"), ("dit_120s_clip_w8a8_mlp", "dit_120s_w8a8"),
                      ("dit_120s_clip_w8a8_mlp_qkv", "dit_120s_w8a8_qkv"),
                      ("dit_120s_clip_w8a8_mlp_qkv_out", "dit_120s_w8a8_qkv_out")):
        if key in paths:
            out[name] = f"{paths[key]['ms_per_clip']:.1f} ms/clip"
    if "band_380s_layer" in paths:
        d = paths["band_380s_layer"]
        out["band_380s"] = f"{d['ms_per_layer']:.3f} ms {d['tflops']:.0f} TFLOP/s"
    if "song_380s_8_clips" in paths:
        out["song_380s_x8"] = f"{paths['song_380s_8_clips']['ms_per_batch_of_8']:.0f} ms"
    return out


# ----------------------------------------------------------------------------------------------- main
def _stdout_for_result():
    """Route everything written to fd 1 (library banners, NCCL) to stderr; return a stream on the original
    stdout that carries only the result line."""
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    return os.fdopen(saved, "w")


def main():
    result_out = _stdout_for_result()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="hb", choices=["hb", "reference"])
    ap.add_argument("--no-secondary", action="store_true", help="skip the dense / W8A8 lines (N = 1)")
    ap.add_argument("--cpu-rows", type=int, default=L_PER_GPU, help="queries in the CPU-baseline sample")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        run_reference(args, result_out)
        return

    rank, world, local = dist_env()
    import torch
    sys.path.insert(0, str(ROOT))
    from hummingbird_b200 import _lib
    _lib.lib()
    device = init_dist(world, local)
    peaks, peak_kind = load_peaks()

    comm = None
    if world > 1:  # the halo exchanges run through the library's own NCCL C ABI (libhb_comm.so)
        from hummingbird_b200.comm import HbComm
        comm = HbComm(rank, world, timeout_ms=120_000)
    step = BandStep(device, rank, world, comm)
    layer = BandLayerStep(device, rank, world, comm)
    clocks = ClockSampler(local)
    clocks.start()
    t = time_band(step, args.steps, args.warmup, world)
    e2e = time_band_e2e(step, max(10, args.steps // 4), args.warmup, world)
    tl = time_band_layer(layer, max(10, args.steps // 2), args.warmup, world)
    e2e_l = time_band_layer_e2e(layer, max(10, args.steps // 4), args.warmup, world)
    clk = clocks.stop()
    total_flops = sum_over_ranks(step.flops, world)
    value = total_flops / (t["ms_per_step"] * 1e-3) / 1e12

    # the step's one kernel (band_fused_kernel) and its roofline: HBM-bound (AI 171 FLOP/B < ridge 257)
    qkv_bytes = L_PER_GPU * 5 * HEADS * 64 * 2
    out_bytes = L_PER_GPU * HEADS * 64 * 2
    k_bytes = qkv_bytes + out_bytes  # algorithmic: read the projection once, write the output once
    k_ms = t["attn_ms"]
    achieved = k_bytes / (k_ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD,
                   "global_rows": L_PER_GPU * world, "parallelism": f"sequence-sharded x{world}, NCCL halo "
                   "send/recv of 128 rows per side through hb_comm_halo_exchange" if world > 1 else "single GPU",
                   "l2": "inputs 423 MB per GPU > 126 MB L2 (no flush needed)"},
        "clocks": clk,
        "e2e": {"value": total_flops / (e2e["ms_per_step"] * 1e-3) / 1e12, "unit": "TFLOP/s",
                "ms_per_step": e2e["ms_per_step"], "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                "how": "band_attention_from_host: pinned host qkv streamed to the device in 8,192-row chunks, "
                       "halo exchange on the device (N > 1), each chunk's queries as soon as their rows landed, "
                       "output streamed back to pinned host memory"},
        "e2e_layer": {
            "value": total_flops / (e2e_l["ms_per_step"] * 1e-3) / 1e12, "unit": "TFLOP/s",
            "ms_per_step": e2e_l["ms_per_step"], "h2d_bytes_per_step": e2e_l["h2d"],
            "d2h_bytes_per_step": e2e_l["d2h"],
            "how": "same_l_attention_from_host: the SAME-L attention layer (same_l._attention of _block: block DyT "
                   "pre-norm, to_qkv, band attention, to_out) with its input x in pinned host memory, streamed in "
                   "16,384-row chunks through the one-GEMM front end and the band kernel; attention FLOPs counted",
            "device_ms_per_step": tl["ms_per_step"],
            "device_stages_ms": {"front_end": tl["proj_ms"], "band": tl["attn_ms"], "to_out": tl["to_out_ms"]},
            "front_end_roofline": {"bound": "tensor", "kernel": "band_proj_kernel",
                                   "achieved": layer.proj_flops / (tl["proj_ms"] * 1e-3) / 1e12,
                                   "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                                   "frac": layer.proj_flops / (tl["proj_ms"] * 1e-3) / 1e12 / peaks["bf16_tflops"],
                                   "flops_per_launch": layer.proj_flops}},
        "gpu_launches": step.launches * args.steps,
        "roofline": {"bound": "hbm", "kernel": "band_fused_kernel", "achieved": achieved, "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "traffic": BAND_NCU_TRAFFIC,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch of "
                                       "this workload (committed summary under profiles/)",
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, burst copy)" if peak_kind == "measured"
                     else "fallback 6650 GB/s", "algorithmic_bytes_per_launch": k_bytes, "kernel_ms": k_ms,
                     "tensor_frac_of_bf16": value / world / peaks["bf16_tflops"],
                     "tensor_peak_tflops": peaks["bf16_tflops"]},
    }
    if not args.no_secondary:
        paths = {}
        if world == 1:
            paths["dense_config1"] = time_dense(device, 50, 5, 1, 646, 16, 1024)
            paths["dense_120s_block_call"] = time_dense(device, 20, 3, 2, 2648, 16, 1024)
            paths["cross_120s_block_call"] = time_cross(device, 50, 5, peaks["hbm_gbs"])
            paths["w8a8_config3"] = time_w8a8(device, 50, 5)
            paths["w8a8_dit_mlp"] = time_w8a8_glu_mlp(device, 30, 5)
            paths["dit_120s_clip_bf16_mlp"] = time_dit_clip(device, "none")
            paths["dit_120s_clip_w8a8_mlp_qkv"] = time_dit_clip(device, "w8a8", qkv_quant="w8a8")
            paths["dit_120s_clip_w8a8_mlp_qkv_out"] = time_dit_clip(device, "w8a8", qkv_quant="w8a8",
                                                                    out_quant="w8a8")
        paths["dit_120s_clip_w8a8_mlp"] = time_dit_clip(device, "w8a8", world)
        paths["band_380s_layer"] = time_band_song_layer(device, world, rank, comm=comm)
        paths["song_380s_8_clips"] = time_song(device, world, rank)
        line["paths"] = paths
    if world == 1 and rank == 0:
        line["cpu_baseline"] = cpu_band_baseline(step.w.qkv, step.w, args.cpu_rows)
        line["e2e_layer"]["cpu_baseline"] = cpu_layer_baseline(layer.w, args.cpu_rows)
        from oracle.cpu_baseline import shutdown
        shutdown()
    parity = {"band_headline": band_parity(step, world), "band_layer": layer_parity(layer, world)}
    if "paths" in line and line["paths"]["dit_120s_clip_w8a8_mlp"].get("parity"):
        parity["dit_split_step"] = line["paths"]["dit_120s_clip_w8a8_mlp"]["parity"]
    line["parity"] = parity
    if "paths" in line:  # the secondary paths in one short entry, last on the line
        line["paths_summary"] = paths_summary(line["paths"], peaks)
    if rank == 0:
        print(json.dumps(line), file=result_out, flush=True)
    if world > 1:
        import torch.distributed as dist
        torch.cuda.synchronize()
        dist.barrier()
        comm.close()
        dist.destroy_process_group()
    del torch


if __name__ == "__main__":
    main()
