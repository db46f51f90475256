"""CPU: the division-free rounding of the int8 quantisers (`hummingbird_b200/csrc/quant_common.cuh`, used by
`hb_quant_rows_int8` and the GLU's fused quantisation), restated step by step in numpy fp32, equals the
quantisation rule of the oracle: clamp(rint(x / s), -127, 127) with a correctly rounded fp32 division and
round-half-to-even. The cases include exact ties, near-ties, all-zero rows, scales across the bf16 range and
scales so small that 1 / s overflows to infinity."""
import numpy as np

from oracle import w8a8
from oracle.common import bf16_bits_to_f32, f32_to_bf16_bits

MAGIC = np.float32(12582912.0)          # 1.5 * 2^23
NEAR_HALF = np.float32(0.5 - 2.0 ** -14)


def _bf16(x):
    return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(x, np.float32)))


def fast_quantize(x: np.ndarray):
    """The device steps: s = absmax / 127 (1 for a zero row), rs = fl(1 / s), q0 = fl(x * rs),
    n = fl(fl(q0 + MAGIC) - MAGIC); n unless |q0 - n| is not below NEAR_HALF (or not finite), else
    rint(fl(x / s)); clamp to +-127; the int8 is the low byte of fl(v + MAGIC). Also returns the fraction of
    elements that took the division."""
    x = np.asarray(x, np.float32)
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        amax = np.abs(x).max(axis=1).astype(np.float32)
        s = np.where(amax == 0, np.float32(1), (amax / np.float32(127)).astype(np.float32)).astype(np.float32)
        rs = (np.float32(1) / s).astype(np.float32)
        q0 = (x * rs[:, None]).astype(np.float32)
        n = ((q0 + MAGIC).astype(np.float32) - MAGIC).astype(np.float32)
        fast = np.abs(q0 - n) < NEAR_HALF          # False for NaN / inf, as the device's !(a < b)
        exact = np.rint((x / s[:, None]).astype(np.float32))
        v = np.where(fast, n, exact)
        v = np.fmin(np.fmax(v, np.float32(-127)), np.float32(127)).astype(np.float32)  # NaN-ignoring, as fminf / fmaxf
        q = ((v + MAGIC).astype(np.float32).view(np.uint32) & 0xFF).astype(np.uint8).view(np.int8)
    return q, s, float((~fast).mean())


def _check(x):
    q, s, frac = fast_quantize(x)
    q_ref, s_ref = w8a8.quantize_rows(x)
    assert np.array_equal(s, s_ref)
    assert np.array_equal(q, q_ref), np.argwhere(q != q_ref)[:5]
    return frac


def test_random_rows_across_the_bf16_range():
    rng = np.random.default_rng(5)
    rows = [_bf16(rng.standard_normal(4096) * np.float32(10.0 ** e)) for e in rng.uniform(-35, 35, 96)]
    frac = _check(np.stack(rows))
    assert frac < 0.01  # the division is the rare path


def test_exact_and_near_ties():
    ties = np.concatenate([np.arange(-127, 127) + np.float32(0.5), [np.float32(127)]]).astype(np.float32)
    rows = [ties, ties * np.float32(2.0 ** -100), ties * np.float32(2.0 ** 100), -ties]
    # near-ties: bf16 values whose quotient by a non-power-of-two scale lands close to k + 1/2
    rng = np.random.default_rng(6)
    for _ in range(64):
        amax = np.float32(_bf16([rng.uniform(1, 2) * 2.0 ** rng.integers(-60, 60)]).reshape(-1)[0])
        s = np.float32(amax / np.float32(127))
        k = rng.integers(-126, 126, 254) + 0.5
        row = _bf16((k * s).astype(np.float32))
        row = np.concatenate([row, [amax]]).astype(np.float32)
        rows.append(row)
    _check(np.stack(rows))


def test_zero_and_tiny_rows():
    zero = np.zeros(256, np.float32)
    tiny = _bf16(np.linspace(-1e-39, 1e-39, 256, dtype=np.float32))  # subnormal scale: 1 / s overflows
    tiny_zero = tiny.copy()
    tiny_zero[::7] = 0                                                  # x = 0 with rs = inf gives q0 = NaN
    small = _bf16(np.linspace(-3e-37, 3e-37, 256, dtype=np.float32))  # scale near the subnormal boundary
    x = np.stack([zero, tiny, tiny_zero, small])
    with np.errstate(over="ignore"):
        assert not np.isfinite(np.float32(1) / np.float32(np.abs(tiny).max() / np.float32(127)))
    _check(x)
    q, s, _ = fast_quantize(zero[None])
    assert s[0] == 1 and not q.any()
