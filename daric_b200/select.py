"""Recompute selection on the GPU: score-driven top-k / threshold select and
DARIC-policy range expansion, both emitting the recompute index list and the
slot mapping ``block_ids[p // bs] * bs + p % bs`` (the formula vLLM applies to
the recompute sub-requests, integration/vllm/worker.py:310-346,
utils.py:406-465).
"""
from __future__ import annotations

import ctypes as C
import functools
from collections.abc import Sequence
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import _lib
from ._lib import check, i64

__all__ = ["Selection", "score_select", "ptrs_to_slots", "topk_count"]


def topk_count(num_tokens: int, ratio: float) -> int:
    """Tokens recomputed for a ratio: floor(ratio * num_tokens)."""
    return int(np.floor(ratio * num_tokens + 1e-9)) if num_tokens > 0 else 0


@dataclass
class Selection:
    """Per (layer, request) selection. ``idx``/``slot`` are [L, out_ld]
    device tensors; row l holds request s's entries at
    [out_off[s], out_off[s] + count[l, s])."""
    idx: torch.Tensor
    slot: torch.Tensor
    count: torch.Tensor
    out_off: np.ndarray

    def get(self, layer: int, seg: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
        n = int(self.count[layer, seg])
        o = int(self.out_off[seg])
        return self.idx[layer, o:o + n], self.slot[layer, o:o + n]


@functools.lru_cache(maxsize=256)
def _select_args(L: int, T: int, seg_len, seg_col_off, seg_pos0, seg_blk_off, k, ratio, threshold):
    """Host arrays of one selection shape (cached: serving repeats shapes)."""
    lens = np.asarray(seg_len if seg_len is not None else (T,), np.int64)
    nseg = len(lens)
    cols = np.asarray(seg_col_off, np.int64) if seg_col_off is not None else \
        np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    if len(cols) != nseg or (nseg and (cols.min() < 0 or (cols + lens).max() > T)):
        raise RuntimeError("score segments must lie inside the score rows")
    pos0 = np.asarray(seg_pos0 if seg_pos0 is not None else (0,) * nseg, np.int64)
    blk = np.asarray(seg_blk_off if seg_blk_off is not None else (0,) * nseg, np.int64)
    if threshold is not None:
        mode, kk = _lib.SELECT_THRESHOLD, np.zeros(nseg, np.int64)
        caps = lens.copy()
    else:
        mode = _lib.SELECT_TOPK
        if k is None:
            if ratio is None:
                raise ValueError("score_select needs k, ratio or threshold")
            kk = np.array([topk_count(int(n), ratio) for n in lens], np.int64)
        else:
            kk = np.broadcast_to(np.asarray(k, np.int64), (nseg,)).copy()
        caps = np.minimum(kk, lens)
    out_off = np.concatenate([[0], np.cumsum(caps)[:-1]]).astype(np.int64)
    out_ld = max(int(caps.sum()), 1)
    arrs = tuple(np.ascontiguousarray(a) for a in (lens, cols, pos0, blk, kk, out_off))
    for a in arrs:
        a.setflags(write=False)
    return mode, nseg, out_ld, arrs


def _tup(x):
    if x is None:
        return None
    if isinstance(x, (int, np.integer)):
        return int(x)
    return tuple(int(v) for v in x)


def score_select(scores: torch.Tensor, block_table: torch.Tensor, block_size: int, *,
                 seg_len: Optional[Sequence[int]] = None, seg_col_off: Optional[Sequence[int]] = None,
                 seg_pos0: Optional[Sequence[int]] = None, seg_blk_off: Optional[Sequence[int]] = None,
                 k: Optional[Sequence[int] | int] = None, ratio: Optional[float] = None,
                 threshold: Optional[float] = None, stream: int = 0,
                 out: Optional[Selection] = None) -> Selection:
    """Selects recompute tokens per layer and request from fp32 ``scores``
    [L, T_total] (CUDA). Requests are column segments (default: one segment
    covering the row). Top-k (``k`` or ``ratio``) keeps the k highest scores,
    ties to the lower token index; ``threshold`` keeps every score >= it.
    Output positions are ascending per (layer, request)."""
    if not scores.is_cuda or scores.dtype != torch.float32 or scores.dim() != 2 or scores.stride(1) != 1:
        raise RuntimeError("scores must be a CUDA float32 [layers, tokens] matrix with unit column stride")
    if not block_table.is_cuda or block_table.dtype != torch.int32 or not block_table.is_contiguous():
        raise RuntimeError("block_table must be a contiguous CUDA int32 tensor")
    L, T = scores.shape
    mode, nseg, out_ld, (lens, cols, pos0, blk, kk, out_off) = _select_args(
        L, T, _tup(seg_len), _tup(seg_col_off), _tup(seg_pos0), _tup(seg_blk_off), _tup(k),
        None if ratio is None else float(ratio), None if threshold is None else float(threshold))
    dev = scores.device.index
    if out is None:
        out = Selection(
            idx=torch.empty((L, out_ld), dtype=torch.int32, device=scores.device),
            slot=torch.empty((L, out_ld), dtype=torch.int64, device=scores.device),
            count=torch.empty((L, nseg), dtype=torch.int32, device=scores.device),
            out_off=out_off)
    else:
        if out.idx.shape[1] < out_ld or out.idx.shape[0] < L or out.count.shape != (L, nseg):
            raise RuntimeError("preallocated selection output is too small")
        out.out_off = out_off
    p64 = lambda a: a.ctypes.data
    s = stream or torch.cuda.current_stream(dev).cuda_stream
    check(_lib.load().daric_score_select(
        C.c_void_p(scores.data_ptr()), L, scores.stride(0), nseg, p64(cols), p64(lens), p64(pos0), p64(kk),
        mode, C.c_float(threshold if threshold is not None else 0.0), C.c_void_p(block_table.data_ptr()),
        block_table.numel(), p64(blk), int(block_size), C.c_void_p(out.idx.data_ptr()),
        C.c_void_p(out.slot.data_ptr()), C.c_void_p(out.count.data_ptr()), out.idx.stride(0), p64(out_off), dev,
        C.c_void_p(s)))
    return out


def ptrs_to_slots(ranges: Sequence[Sequence[int]], block_table: torch.Tensor, block_size: int, *,
                  range_blk_off: Optional[Sequence[int]] = None,
                  stream: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Expands [start, end) ranges (DARICPolicy.get_recompute_ptrs) into the
    recompute positions and their slots, in range order."""
    if not block_table.is_cuda or block_table.dtype != torch.int32 or not block_table.is_contiguous():
        raise RuntimeError("block_table must be a contiguous CUDA int32 tensor")
    n = len(ranges)
    starts = [int(r[0]) for r in ranges]
    ends = [int(r[1]) for r in ranges]
    total = sum(max(0, e - s) for s, e in zip(starts, ends))
    idx = torch.empty(total, dtype=torch.int32, device=block_table.device)
    slot = torch.empty(total, dtype=torch.int64, device=block_table.device)
    if total == 0:
        return idx, slot
    a, ap = i64(starts)
    b, bp = i64(ends)
    c, cp = i64(range_blk_off if range_blk_off is not None else [0] * n)
    dev = block_table.device.index
    s = stream or torch.cuda.current_stream(dev).cuda_stream
    check(_lib.load().daric_ptrs_to_slots(
        n, ap, bp, cp, C.c_void_p(block_table.data_ptr()), block_table.numel(), int(block_size),
        C.c_void_p(idx.data_ptr()), C.c_void_p(slot.data_ptr()), dev, C.c_void_p(s)))
    return idx, slot
