"""hummingbird-b200: B200-native (sm_100a) hot paths of kelechi-c/hummingbird (`sa3jax`).

* `hummingbird_b200.dense_attention` — drop-in for `sa3jax.dense_attention` (DiT differential self-attention)
* `hummingbird_b200.band_attention`  — drop-in for `sa3jax.band_attention` (SAME-L differential band attention)
* `hummingbird_b200.w8a8`            — W8A8 int8 linear for the DiT MLP
* `hummingbird_b200.config`          — `DiTConfig` / `SameConfig` mirrors with the `"cuda"` switch values
* `hummingbird_b200.parallel`        — head-pair, sequence-shard (halo exchange) and clip sharding over NCCL

All compute runs in `libhb_b200.so` (C ABI in `include/hb_b200.h`); there is no CPU fallback.
"""
__version__ = "0.1.0"
