"""CPU: the algorithmic work units `bench.py` reports against. Band FLOPs count every (query, key) pair inside
the window once per branch (`2 branches x (QK^T + PV) x 2 x 64` per pair and head, keys clipped at the
sequence ends); a sharded sequence's per-rank counts add up to the whole; the band kernel's minimum bytes are
one read of `qkv` and one write of the output."""
import numpy as np
import pytest

import bench


def _pairs(length, window, q0=0, q1=None):
    q1 = length if q1 is None else q1
    q = np.arange(q0, q1, dtype=np.int64)
    return int((np.minimum(length - 1, q + window) - np.maximum(0, q - window) + 1).sum())


def test_band_flops_at_the_benchmark_configs():
    # config 2: L = 82,688, 8 heads, window 128 -> 21,234,304 (query, key) pairs per head, 86.98 GFLOP
    assert _pairs(82_688, 128) == 21_234_304
    assert bench.band_flops(82_688, 0, 82_688) == 8 * 64 * 8 * 21_234_304
    assert round(bench.band_flops(82_688, 0, 82_688) / 1e9, 2) == 86.98
    # config 5's decoder layer: L = 261,888 -> 67,288,704 pairs per head, 275.6 GFLOP
    assert _pairs(261_888, 128) == 67_288_704
    assert round(bench.band_flops(261_888, 0, 261_888) / 1e9, 1) == 275.6


@pytest.mark.parametrize("world", [2, 4, 8])
def test_band_flops_of_shards_add_up(world):
    total = world * bench.L_PER_GPU
    parts = [bench.band_flops(total, r * bench.L_PER_GPU, (r + 1) * bench.L_PER_GPU) for r in range(world)]
    assert sum(parts) == bench.band_flops(total, 0, total)
    # interior shards see full windows on both sides, the two end shards lose half a window each
    assert parts[0] == parts[-1] < parts[len(parts) // 2] if world > 2 else parts[0] == parts[1]


def test_band_minimum_bytes_and_arithmetic_intensity():
    qkv = bench.L_PER_GPU * 5 * bench.HEADS * 64 * 2
    out = bench.L_PER_GPU * bench.HEADS * 64 * 2
    assert round((qkv + out) / 1e6, 1) == 508.0
    ai = bench.band_flops(bench.L_PER_GPU, 0, bench.L_PER_GPU) / (qkv + out)
    assert 170 < ai < 172  # below the B200 ridge point (~257 FLOP/B), so HBM is the roofline


def test_peaks_come_from_the_measured_file_when_present():
    peaks, source = bench.load_peaks()
    if (bench.ROOT / "MEASURED_PEAKS.json").exists():
        assert source == "measured" and peaks["hbm_gbs"] > 1000
    else:
        assert source == "fallback" and peaks == bench.FALLBACK_PEAKS
