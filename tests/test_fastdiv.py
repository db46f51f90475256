"""CPU: the multiply-high division of the dense prologue's task decode (`FastDiv` in csrc/dense_attn.cu).

For a divisor d > 1 the host precomputes l = ceil(log2 d), p = 31 + l, mul = ceil(2^p / d) and shift = p - 32;
the kernel then takes n / d as umulhi(n, mul) >> shift (umulhi = the high 32 bits of the 64-bit product), and
d = 1 passes n through. The kernel relies on this being exact integer division for 0 <= n < 2^31 (the host
refuses problems with 2^31 or more tasks). This restates the arithmetic bit for bit and checks it against `//`
for the divisors the decode uses (head groups, padded rows per batch element) and beyond."""
import numpy as np


def _fastdiv_init(d: int) -> tuple[int, int]:
    if d == 1:
        return 0, 0
    l = 0
    while (1 << l) < d:
        l += 1
    p = 31 + l
    mul = ((1 << p) + d - 1) // d
    assert mul < (1 << 32), "the multiplier must fit the kernel's 32-bit register"
    return mul, p - 32


def _fastdiv(n: np.ndarray, d: int, mul: int, shift: int) -> np.ndarray:
    if d == 1:
        return n
    return ((n.astype(np.uint64) * np.uint64(mul)) >> np.uint64(32 + shift)).astype(np.int64)


def _divisors() -> list[int]:
    ds = list(range(1, 300))
    ds += [t * 128 for t in (1, 2, 6, 21, 65, 646, 2046, 4096, 65535)]  # padded rows per batch element
    ds += [2 ** k for k in range(1, 31)] + [2 ** k - 1 for k in range(2, 31)] + [2 ** k + 1 for k in range(2, 31)]
    rng = np.random.default_rng(0)
    ds += rng.integers(2, 2 ** 31 - 1, 200).tolist()
    return sorted(set(ds))


def test_fastdiv_is_exact_below_2_31():
    rng = np.random.default_rng(1)
    top = 2 ** 31 - 1
    for d in _divisors():
        mul, shift = _fastdiv_init(d)
        q = np.arange(0, top // d + 1, max(1, (top // d) // 4096), dtype=np.int64)
        edges = np.concatenate([q * d, q * d - 1, q * d + d - 1])  # both sides of every sampled quotient step
        n = np.concatenate([edges, rng.integers(0, top, 20_000), [0, 1, d - 1, d, top, top - 1]])
        n = n[(n >= 0) & (n <= top)].astype(np.int64)
        got = _fastdiv(n, d, mul, shift)
        assert np.array_equal(got, n // d), d
