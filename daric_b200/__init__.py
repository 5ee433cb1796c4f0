"""daric_b200 — B200-native (sm_100a) reused-KV hot path of DARIC.

Drop-in modules:
  daric_b200.cache_ops  <- daric.cache_ops  (CacheCopier, batched_memcpy_*)
  daric_b200.adaption   <- daric.adaption   (Adapter, DARICPolicy)
New:
  daric_b200.reuse      fused store -> re-rotated paged KV loader
  daric_b200.select     GPU recompute selection (top-k / threshold / policy ranges)
The compute runs in libdaric_b200.so (C ABI: include/daric_b200.h).
"""
__version__ = "0.1.0"
