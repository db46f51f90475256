"""Timed CPU baselines: the oracle port run on the host's cores — test / benchmark infrastructure only.

Used by `bench.py` (`cpu_baseline` and `--impl reference`): the reference's own XLA CPU path cannot run here
(JAX is not installed), so its fp32 restatement in `oracle.band` / `oracle.dense` / `oracle.w8a8` stands in
for it, computed in float32 (the reference's FP32 XLA precision) and spread over the host's cores with a
`spawn` process pool (one BLAS thread per worker), on a bounded sample of the benchmark's workload.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import time

import numpy as np

_POOL = None
_WORKERS = 0


def _init_worker():
    """One BLAS thread per worker process (the pool supplies the parallelism)."""
    from threadpoolctl import threadpool_limits
    threadpool_limits(1)


def pool(workers: int | None = None):
    """A spawn-context pool (safe to create after CUDA initialisation in the parent)."""
    global _POOL, _WORKERS
    workers = workers or os.cpu_count() or 1
    if _POOL is None or _WORKERS != workers:
        ctx = mp.get_context("spawn")
        saved = {k: os.environ.get(k) for k in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")}
        os.environ.update({k: "1" for k in saved})  # inherited by the spawned workers before numpy loads
        try:
            _POOL = ctx.Pool(workers, initializer=_init_worker)
        finally:
            for k, v in saved.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v
        _WORKERS = workers
    return _POOL


def shutdown():
    global _POOL
    if _POOL is not None:
        _POOL.terminate()
        _POOL = None


def band_flops(length: int, heads: int, window: int, q0: int = 0, q1: int | None = None) -> float:
    """Algorithmic FLOPs of band differential attention over queries [q0, q1): 2 branches x (QK^T + PV) x
    2 FLOP x 64 dims x heads x sum_q |{k : |k - q| <= window, 0 <= k < length}|."""
    q1 = length if q1 is None else q1
    q = np.arange(q0, q1, dtype=np.int64)
    keys = np.minimum(length - 1, q + window) - np.maximum(0, q - window) + 1
    return float(2 * 2 * 2 * 64 * heads * keys.sum())


def dense_flops(batch: int, length: int, heads: int) -> float:
    """2 branches x (QK^T + PV) x 2 FLOP x 64 x L^2 per head: 8 * B * H * L^2 * 64."""
    return 8.0 * batch * heads * length * length * 64


_SHM_CACHE: dict = {}


def _attach(name: str, shape: tuple) -> np.ndarray:
    from multiprocessing import shared_memory
    if name not in _SHM_CACHE:
        _SHM_CACHE.clear()
        shm = shared_memory.SharedMemory(name=name)
        _SHM_CACHE[name] = (shm, np.ndarray(shape, np.float32, buffer=shm.buf))
    return _SHM_CACHE[name][1]


def _band_task(args):
    from oracle.band import band_diff_attention
    name, shape, qn, kn, freqs, heads, window, lam, lo, hi, q0, q1 = args
    qkv = _attach(name, shape)[:, lo:hi]
    out = band_diff_attention(qkv, qn, kn, freqs, heads, window, lam=lam, offset=lo, dtype=np.float32)
    return float(out[:, q0 - lo:q1 - lo].sum())


def time_band_sample(qkv: np.ndarray, q_norm: dict, k_norm: dict, freqs: np.ndarray, heads: int, window: int,
                     lam: np.ndarray, q_rows: int, workers: int | None = None, chunk: int = 256,
                     min_seconds: float = 0.0) -> dict:
    """Time the oracle on queries [0, q_rows) of `qkv` (float32 `(1, L, 5 H 64)`, placed in shared memory),
    split into `chunk`-row tasks (each reading its +-window halo) over a spawn pool, repeating the whole sample
    until `min_seconds` have passed (at least once). Returns seconds, FLOPs of all passes, the pass count and
    the worker count."""
    from multiprocessing import shared_memory
    length = qkv.shape[1]
    p = pool(workers)
    shm = shared_memory.SharedMemory(create=True, size=qkv.nbytes)
    try:
        np.ndarray(qkv.shape, np.float32, buffer=shm.buf)[...] = qkv
        tasks = []
        for q0 in range(0, q_rows, chunk):
            q1 = min(q_rows, q0 + chunk)
            lo, hi = max(0, q0 - window), min(length, q1 + window)
            tasks.append((shm.name, qkv.shape, q_norm, k_norm, freqs, heads, window, lam, lo, hi, q0, q1))
        p.map(_band_task, tasks[: min(len(tasks), _WORKERS)])  # warm the workers (imports, BLAS, mapping)
        t0 = time.perf_counter()
        passes = 0
        while True:
            p.map(_band_task, tasks)
            passes += 1
            if time.perf_counter() - t0 >= min_seconds:
                break
        seconds = time.perf_counter() - t0
    finally:
        shm.close()
        shm.unlink()
    return {"seconds": seconds, "flops": passes * band_flops(length, heads, window, 0, q_rows), "passes": passes,
            "cores": _WORKERS}


def _front_task(args):
    from oracle.band import front_end
    xname, xshape, qname, qshape, w_qkv, pre, r0, r1 = args
    x = _attach_many(xname, xshape)
    qkv = _attach_many(qname, qshape)
    qkv[:, r0:r1] = front_end(x[:, r0:r1], w_qkv, pre)
    return r1 - r0


def _layer_task(args):
    from oracle.band import band_diff_attention
    qname, qshape, qn, kn, freqs, heads, window, lam, w_out, lo, hi, q0, q1 = args
    qkv = _attach_many(qname, qshape)[:, lo:hi]
    out = band_diff_attention(qkv, qn, kn, freqs, heads, window, lam=lam, offset=lo, dtype=np.float32)
    y = out[:, q0 - lo:q1 - lo] @ w_out.T
    return float(y.sum())


_SHM_MANY: dict = {}


def _attach_many(name: str, shape: tuple) -> np.ndarray:
    from multiprocessing import shared_memory
    if name not in _SHM_MANY:
        if len(_SHM_MANY) > 8:
            _SHM_MANY.clear()
        shm = shared_memory.SharedMemory(name=name)
        _SHM_MANY[name] = (shm, np.ndarray(shape, np.float32, buffer=shm.buf))
    return _SHM_MANY[name][1]


def time_layer_sample(x: np.ndarray, w_qkv: np.ndarray, w_out: np.ndarray, pre_norm: dict | None, q_norm: dict,
                      k_norm: dict, freqs: np.ndarray, heads: int, window: int, lam: np.ndarray, q_rows: int,
                      workers: int | None = None, chunk: int = 256, min_seconds: float = 0.0) -> dict:
    """Time the SAME-L attention layer's oracle (`oracle.band.front_end`: block DyT pre-norm + `to_qkv`; the
    band attention; `to_out`) on queries [0, q_rows) of x (float32 `(1, L, d)` holding bf16 values) over a spawn
    pool: phase 1 projects the rows the sample needs once, in `chunk`-row tasks, into a shared array; phase 2
    runs the band attention and `to_out` per `chunk` of queries. Repeats the whole sample until `min_seconds`
    have passed (at least once). FLOPs counted: the attention's only (as for `time_band_sample`)."""
    from multiprocessing import shared_memory
    length = x.shape[1]
    rows = min(length, q_rows + window)
    n = w_qkv.shape[0]
    p = pool(workers)
    xs = shared_memory.SharedMemory(create=True, size=x[:, :rows].nbytes)
    qs = shared_memory.SharedMemory(create=True, size=rows * n * 4)
    try:
        xshape, qshape = (1, rows, x.shape[2]), (1, rows, n)
        np.ndarray(xshape, np.float32, buffer=xs.buf)[...] = x[:, :rows]
        front = [(xs.name, xshape, qs.name, qshape, w_qkv, pre_norm, r0, min(rows, r0 + chunk))
                 for r0 in range(0, rows, chunk)]
        layer = []
        for q0 in range(0, q_rows, chunk):
            q1 = min(q_rows, q0 + chunk)
            lo, hi = max(0, q0 - window), min(rows, q1 + window)
            layer.append((qs.name, qshape, q_norm, k_norm, freqs, heads, window, lam, w_out, lo, hi, q0, q1))
        p.map(_front_task, front[: min(len(front), _WORKERS)])  # warm the workers
        t0 = time.perf_counter()
        passes = 0
        while True:
            p.map(_front_task, front)
            p.map(_layer_task, layer)
            passes += 1
            if time.perf_counter() - t0 >= min_seconds:
                break
        seconds = time.perf_counter() - t0
    finally:
        for shm in (xs, qs):
            shm.close()
            shm.unlink()
    return {"seconds": seconds, "flops": passes * band_flops(length, heads, window, 0, q_rows), "passes": passes,
            "cores": _WORKERS}


def _dense_task(args):
    from oracle.dense import dense_branches
    qkv, q_w, k_w, freqs, valid, heads, eps = args
    a, b = dense_branches(qkv.astype(np.float32), q_w, k_w, freqs, valid, heads, eps)
    return a.shape


def time_dense_sample(qkv: np.ndarray, q_w, k_w, freqs, valid, heads: int, eps: float,
                      workers: int | None = None) -> dict:
    """Time the dense oracle over all heads of `qkv`, one task per head."""
    p = pool(workers)
    b, length, _ = qkv.shape
    sec = np.split(qkv, 5, axis=-1)
    tasks = []
    for h in range(heads):
        cols = [s[..., h * 64:(h + 1) * 64] for s in sec]
        tasks.append((np.concatenate(cols, -1), q_w, k_w, freqs, valid, 1, eps))
    p.map(_dense_task, tasks[: min(len(tasks), _WORKERS)])
    t0 = time.perf_counter()
    p.map(_dense_task, tasks)
    seconds = time.perf_counter() - t0
    return {"seconds": seconds, "flops": dense_flops(b, length, heads), "cores": _WORKERS}
