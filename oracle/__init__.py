"""TEST INFRASTRUCTURE ONLY — CPU restatement of the reference's reused-KV path.

This package is the checker for the sm_100a kernels of ``daric_b200``. Only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import it; the product never calls it and has no CPU path.

Modules (each function cites the reference code it restates):
  numerics  bf16 / fp16 / fp8-e4m3 rounding (round-to-nearest-even)
  pages     page-copy shape + byte-exact gather/scatter (csrc/cache_ops)
  rerotate  RoPE re-rotation of K in paged caches (daric/adaption/adapter.py)
  select    top-k / threshold selection + slot mapping, deviation scores

Pinning: the policy and the re-rotation are checked against golden vectors
produced by the reference itself (tests/golden/make_golden.py: the
reference's DARICPolicy, and its Triton kernel run by Triton's CPU
interpreter); the page copies against the reference's compiled CUDA module on
the GPU box (oracle/build_ref.py -> oracle/_ref/). Deviation scores and the
score-driven selection have no counterpart in the reference: their parity is
against this restatement only (unpinned).
"""
