"""CPU oracle for hummingbird's three hot paths — TEST INFRASTRUCTURE, not product code.

Only `tests/`, `__graft_entry__.smoke()` and `bench.py` (its `cpu_baseline` leg and `--impl reference`)
may import this package, and only as the checker or as the timed CPU baseline. The product path
(`hummingbird_b200`) never imports it and has no CPU fallback.

What it restates (the reference is kelechi-c/hummingbird, package `sa3jax`):

* `oracle.dense` — the DiT differential self-attention on the XLA path: `dit._rms` (dit.py:45-57),
  `dit._rope_tables`/`_rope` (dit.py:82-98), `dit._sdpa` (dit.py:113-119), `dit._attend`/`_attend_out`
  (dit.py:131-176) and the 5-way split of `dit._self_attention` (dit.py:185-200), in fp32
  (`dtypes.FP32_PARITY`, dtypes.py:41-49), with the per-pair `lambda` that the benchmark configs add
  (`out = A - lambda * B`; lambda = 1 is the reference).
* `oracle.band` — the SAME-L differential band attention on the XLA path: `same_l._dyt` (same_l.py:58-69),
  `same_l._rope_tables`/`_rope` (same_l.py:84-100), `same_l._sdpa` over `_windows`/`_swa_mask`
  (same_l.py:103-148) and `same_l._attention` (same_l.py:151-169), written as a direct band
  `|k - q| <= window, 0 <= k < L` (the same function as the grouped form, same_l.py:14-20).
* `oracle.w8a8` — the W8A8 GEMM that the benchmark configs specify but the reference lacks (its call
  site would be `dit._feed_forward`/`_linear`, dit.py:33-36, 218-221): per-row symmetric int8
  quantisation, exact integer accumulation and a fixed-order fp32 epilogue.

Pinning. The two attention restatements are pinned to golden vectors produced by running the
reference's own `sa3jax` XLA-path functions (dit.py, same_l.py) with a numpy stand-in for `jax`
(`tests/golden/make_golden.py`; JAX itself is absent from this image). The W8A8 path has no
reference implementation: its parity is UNPINNED against the reference; it is pinned instead to
exact integer arithmetic (an independent pure-Python integer matmul in `tests/golden`).
"""
from oracle.common import bf16_round, bf16_bits_to_f32, f32_to_bf16_bits, check_close  # noqa: F401
