"""TEST INFRASTRUCTURE ONLY — recompute selection restatement.

The reference has no score-driven selection (its policy is positional,
daric/adaption/policy.py:45-103); this is the specification the GPU select
kernel is checked against:
  * top-k: order by score descending, ties to the lower token index; every
    NaN ranks above +inf; output positions ascending.
  * threshold: every token with score >= threshold (NaN never).
  * slot of position p: block_ids[p // bs] * bs + p % bs, the mapping vLLM
    derives for the recompute sub-requests (integration/vllm/worker.py:310-346).
"""
from __future__ import annotations

import numpy as np


def score_key(scores: np.ndarray) -> np.ndarray:
    f = np.ascontiguousarray(scores, np.float32)
    u = f.view(np.uint32)
    key = np.where(u & 0x80000000, ~u, u | 0x80000000).astype(np.uint32)
    return np.where(np.isnan(f), np.uint32(0xFFFFFFFF), key)


def topk_positions(scores_row: np.ndarray, k: int) -> np.ndarray:
    n = len(scores_row)
    k = max(0, min(k, n))
    key = score_key(scores_row)
    idx = np.arange(n, dtype=np.int64)
    order = np.lexsort((idx, ~key))  # primary: key descending, secondary: index ascending
    return np.sort(order[:k])


def threshold_positions(scores_row: np.ndarray, threshold: float) -> np.ndarray:
    return np.nonzero(np.asarray(scores_row, np.float32) >= np.float32(threshold))[0].astype(np.int64)


def slots(block_ids, positions, block_size: int) -> np.ndarray:
    bl = np.asarray(block_ids, np.int64)
    p = np.asarray(positions, np.int64)
    return bl[p // block_size] * block_size + p % block_size


def ranges_to_positions(ranges) -> np.ndarray:
    parts = [np.arange(s, e, dtype=np.int64) for s, e in ranges if e > s]
    return np.concatenate(parts) if parts else np.zeros(0, np.int64)
