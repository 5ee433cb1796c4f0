"""Drop-in for the reference's native module ``daric.cache_ops``.

Same names, argument meanings and error behaviour as the pybind11 module of
the reference (csrc/cache_ops/bindings.cpp:7-31, daric/cache_ops.pyi:6-53):
``CacheCopier`` with ``register_layer / register_store / gather_pages /
scatter_pages`` and the module functions ``batched_memcpy_d2h / _h2d``. All
work runs in ``libdaric_b200.so`` (sm_100a kernels); this file only converts
torch tensors and Python sequences to the C ABI.

Added operations of the reused-KV path (not in the reference module):
``register_rotary``, ``rerotate_scatter_pages`` (fused gather-rotate-scatter)
and ``rerotate_inplace`` (all-layer in-place re-rotation).
"""
from __future__ import annotations

import ctypes as C
from collections.abc import Sequence
from typing import Optional

import numpy as np
import torch

from . import _lib
from ._lib import check, i64, names_array

__all__ = ["CacheCopier", "batched_memcpy_d2h", "batched_memcpy_h2d", "kv_dtype_code", "table_dtype_code"]

_KV_CODES = {
    torch.bfloat16: _lib.DTYPE_BF16,
    torch.float16: _lib.DTYPE_F16,
    torch.float32: _lib.DTYPE_F32,
    torch.uint8: _lib.DTYPE_FP8_E4M3,  # uint8 caches are viewed as e4m3 (adapter.py:370-371)
}
if hasattr(torch, "float8_e4m3fn"):
    _KV_CODES[torch.float8_e4m3fn] = _lib.DTYPE_FP8_E4M3

_TAB_CODES = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16, torch.float32: _lib.DTYPE_F32}

_MODES = {"none": _lib.ROPE_NONE, "flexible": _lib.ROPE_FLEXIBLE, "delta": _lib.ROPE_DELTA,
          "strict": _lib.ROPE_DELTA}


def kv_dtype_code(dtype: torch.dtype) -> int:
    if dtype not in _KV_CODES:
        raise ValueError(f"unsupported KV cache dtype for rerotate: {dtype}")
    return _KV_CODES[dtype]


def table_dtype_code(dtype: torch.dtype) -> int:
    if dtype not in _TAB_CODES:
        raise ValueError(f"unsupported cos_sin_cache dtype: {dtype}")
    return _TAB_CODES[dtype]


def mode_code(mode) -> int:
    if isinstance(mode, str):
        return _MODES[mode.lower()]
    return int(mode)


def _stream_ptr(stream: int, device: int) -> int:
    # 0 means the current torch stream of the device (copier.cpp:27-30).
    if stream:
        return int(stream)
    return torch.cuda.current_stream(device).cuda_stream


def _record(t: torch.Tensor, stream: int) -> None:
    # The caching allocator must not reuse `t` before `stream` is done with it
    # (record_tensor_on_external_stream, helpers.cu:182-185).
    if stream and t.is_cuda:
        t.record_stream(torch.cuda.ExternalStream(stream, device=t.device))


def _check_indices(indices_flat: torch.Tensor) -> None:
    # validate_common_job_inputs (helpers.cu:160-163)
    if not indices_flat.is_cuda:
        raise RuntimeError("indices_flat must be on CUDA")
    if indices_flat.dim() != 1:
        raise RuntimeError("indices_flat must be 1D")
    if indices_flat.dtype != torch.int32:
        raise RuntimeError("indices_flat must be int32")
    if not indices_flat.is_contiguous():
        raise RuntimeError("indices_flat must be contiguous")


def _check_lengths(num_jobs: int, offsets, byte_sizes, indices_offsets) -> None:
    if len(offsets) != num_jobs:
        raise RuntimeError("offsets length mismatch")
    if len(byte_sizes) != num_jobs:
        raise RuntimeError("byte_sizes length mismatch")
    if len(indices_offsets) != num_jobs + 1:
        raise RuntimeError("indices_offsets size must be num_jobs + 1")


class CacheCopier:
    """Paged KV <-> flat store copier (reference: class CacheCopier,
    csrc/cache_ops/cache_ops.h:91-126, copier.cpp:7-111).

    Holds references to every registered layer and to the store buffer so
    that imported (e.g. CUDA-IPC) tensors stay alive (copier.cpp:10, 21-24).
    Not internally locked, like the reference."""

    def __init__(self) -> None:
        self._lib = _lib.load()
        h = C.c_void_p()
        check(self._lib.daric_copier_create(C.byref(h)))
        self._h = h
        self._layers: dict[str, torch.Tensor] = {}
        self._tables: dict[str, torch.Tensor] = {}
        self._store: Optional[torch.Tensor] = None

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            self._lib.daric_copier_destroy(h)
            self._h = None

    # ---------------------------------------------------------- registry --
    def register_layer(self, name: str, tensor: torch.Tensor, is_page_first: bool) -> None:
        if not tensor.is_cuda:
            raise RuntimeError(f"kvcache tensor must be on GPU: {name}")
        sizes, sp = i64(tensor.shape)
        strides, tp = i64(tensor.stride())
        check(self._lib.daric_copier_register_layer(
            self._h, name.encode(), C.c_void_p(tensor.data_ptr()), tensor.device.index, tensor.dim(), sp, tp,
            tensor.element_size(), int(bool(is_page_first))))
        self._layers[name] = tensor
        self._tables.pop(name, None)

    def register_store(self, buffer: torch.Tensor) -> None:
        # copier.cpp:16-19
        if not buffer.is_cuda:
            raise RuntimeError("staging buffer must be on CUDA")
        if buffer.dim() != 1:
            raise RuntimeError("store buffer must be 1D")
        if buffer.dtype != torch.uint8:
            raise RuntimeError("store buffer must be uint8")
        if not buffer.is_contiguous():
            raise RuntimeError("store buffer must be contiguous")
        check(self._lib.daric_copier_register_store(
            self._h, C.c_void_p(buffer.data_ptr()), buffer.numel(), buffer.device.index))
        self._store = buffer

    def register_rotary(self, layer_name: str, cos_sin_cache: torch.Tensor, rotary_dim: int,
                        is_neox_style: bool) -> None:
        """Attaches a layer's rotary table (vLLM ``rotary_emb.cos_sin_cache``:
        [max_position, rotary_dim] in the model dtype). The table is used as
        is (its bf16 values are what the reference kernel consumes)."""
        if layer_name not in self._layers:
            raise RuntimeError(f"layer not registered: {layer_name}")
        kv = self._layers[layer_name]
        if cos_sin_cache.device != kv.device:
            cos_sin_cache = cos_sin_cache.to(kv.device)
        cos_sin_cache = cos_sin_cache.contiguous()
        if cos_sin_cache.dim() != 2 or cos_sin_cache.shape[1] != rotary_dim:
            raise ValueError(
                f"cos_sin_cache must be [max_position, rotary_dim={rotary_dim}], got {tuple(cos_sin_cache.shape)}")
        check(self._lib.daric_copier_register_rotary(
            self._h, layer_name.encode(), kv_dtype_code(kv.dtype), C.c_void_p(cos_sin_cache.data_ptr()),
            table_dtype_code(cos_sin_cache.dtype), cos_sin_cache.shape[0], int(rotary_dim),
            int(bool(is_neox_style))))
        self._tables[layer_name] = cos_sin_cache

    def has_rotary(self, layer_name: str) -> bool:
        return layer_name in self._tables

    def rotary_table(self, layer_name: str) -> Optional[torch.Tensor]:
        return self._tables.get(layer_name)

    # ------------------------------------------------------------- copies --
    def _jobs(self, layer_names, offsets, byte_sizes, indices_flat, indices_offsets):
        if self._store is None:
            raise RuntimeError("store buffer not registered; call register_store() first")
        n = len(layer_names)
        if n == 0:
            return None
        _check_lengths(n, offsets, byte_sizes, indices_offsets)
        _check_indices(indices_flat)
        return (n, names_array(layer_names), i64(offsets), i64(byte_sizes), i64(indices_offsets))

    def gather_pages(self, layer_names: Sequence[str], offsets: Sequence[int], byte_sizes: Sequence[int],
                     indices_flat: torch.Tensor, indices_offsets: Sequence[int], stream: int = 0) -> None:
        """Paged KV -> store (reference: CacheCopier.gather_pages, copier.cpp:41-76)."""
        j = self._jobs(layer_names, offsets, byte_sizes, indices_flat, indices_offsets)
        if j is None:
            return
        n, names, (_, op), (_, bp), (_, iop) = j
        dev = indices_flat.device.index
        s = _stream_ptr(stream, dev)
        _record(indices_flat, stream)
        check(self._lib.daric_copier_gather_pages(
            self._h, n, names, op, bp, C.c_void_p(indices_flat.data_ptr()), indices_flat.numel(), dev, iop,
            C.c_void_p(s)))

    def scatter_pages(self, layer_names: Sequence[str], offsets: Sequence[int], byte_sizes: Sequence[int],
                      indices_flat: torch.Tensor, indices_offsets: Sequence[int], stream: int = 0) -> None:
        """Store -> paged KV (reference: CacheCopier.scatter_pages, copier.cpp:78-111)."""
        j = self._jobs(layer_names, offsets, byte_sizes, indices_flat, indices_offsets)
        if j is None:
            return
        n, names, (_, op), (_, bp), (_, iop) = j
        dev = indices_flat.device.index
        s = _stream_ptr(stream, dev)
        _record(indices_flat, stream)
        check(self._lib.daric_copier_scatter_pages(
            self._h, n, names, op, bp, C.c_void_p(indices_flat.data_ptr()), indices_flat.numel(), dev, iop,
            C.c_void_p(s)))

    def rerotate_scatter_pages(self, layer_names: Sequence[str], offsets: Sequence[int],
                               byte_sizes: Sequence[int], indices_flat: torch.Tensor,
                               indices_offsets: Sequence[int], job_meta: Sequence[int], mode,
                               meta_pos_a: Sequence[int], meta_pos_b: Optional[Sequence[int]],
                               meta_len: Sequence[int], scores: Optional[torch.Tensor] = None,
                               job_score_row: Optional[Sequence[int]] = None,
                               meta_score_col: Optional[Sequence[int]] = None, stream: int = 0) -> None:
        """Fused store -> paged KV scatter with K re-rotated in fp32.

        Equivalent to ``scatter_pages`` followed by the reference's re-rotation
        of the scattered chunks (adapter.py:196-295 for mode "flexible" with
        meta_pos_a = saved positions and meta_pos_b = new positions;
        adapter.py:118-194 for mode "delta" with meta_pos_a = deltas), except
        that pages with block id 0 are neither written nor rotated.
        ``scores`` (fp32 CUDA [rows, score_ld]) optionally receives each rotated
        token's deviation sum_heads sum_d (K' - K)^2 at
        [job_score_row[i], meta_score_col[meta] + token]."""
        j = self._jobs(layer_names, offsets, byte_sizes, indices_flat, indices_offsets)
        if j is None:
            return
        n, names, (_, op), (_, bp), (_, iop) = j
        code = mode_code(mode)
        jm, jmp = i64(job_meta)
        if len(jm) != n:
            raise RuntimeError("job_meta length mismatch")
        pa, pap = i64(meta_pos_a)
        ln, lnp = i64(meta_len)
        if len(ln) != len(pa):
            raise RuntimeError("meta_len length mismatch")
        pb, pbp = i64(meta_pos_b if meta_pos_b is not None else [0] * len(pa))
        if len(pb) != len(pa):
            raise RuntimeError("meta_pos_b length mismatch")
        sptr, ld, rows_p, cols_p, keep = None, 0, None, None, []
        if scores is not None:
            if not scores.is_cuda or scores.dtype != torch.float32 or scores.dim() != 2 or scores.stride(1) != 1:
                raise RuntimeError("scores must be a CUDA float32 matrix with unit column stride")
            if job_score_row is None or meta_score_col is None:
                raise RuntimeError("scores need job_score_row and meta_score_col")
            rows, rows_p = i64(job_score_row)
            cols, cols_p = i64(meta_score_col)
            if len(rows) != n or len(cols) != len(pa):
                raise RuntimeError("job_score_row / meta_score_col length mismatch")
            if len(rows) and (rows.min() < 0 or rows.max() >= scores.shape[0]):
                raise RuntimeError("job_score_row out of range")
            # every scored token column must fit in the row
            span = max((int(c) + int(l) for c, l in zip(cols, ln)), default=0)
            if span > scores.shape[1]:
                raise RuntimeError("meta_score_col + meta_len exceeds the score row")
            keep = [rows, cols]
            sptr, ld = C.c_void_p(scores.data_ptr()), scores.stride(0)
        dev = indices_flat.device.index
        s = _stream_ptr(stream, dev)
        _record(indices_flat, stream)
        check(self._lib.daric_copier_rerotate_scatter_pages(
            self._h, n, names, op, bp, C.c_void_p(indices_flat.data_ptr()), indices_flat.numel(), dev, iop,
            jmp, code, len(pa), pap, pbp, lnp, sptr, ld, rows_p, cols_p, C.c_void_p(s)))
        del keep

    def load_chunks(self, layer_names, chunk_stg_off: Sequence[int], chunk_blk_off: Sequence[int],
                    chunk_pages: Sequence[int], block_ids: torch.Tensor, mode="flexible",
                    pos_a: Optional[Sequence[int]] = None, pos_b: Optional[Sequence[int]] = None,
                    chunk_len: Optional[Sequence[int]] = None, scores: Optional[torch.Tensor] = None,
                    score_col: Optional[Sequence[int]] = None, layer_range: Optional[tuple] = None,
                    stream: int = 0) -> None:
        """Chunk-level fused load: the copy plan of KVIOManager._build_copy_plan
        (gpu_kv_io.py:334-379) expanded on the device from one descriptor per
        chunk. ``layer_names`` = every layer of a chunk in store order; chunk m
        starts at ``chunk_stg_off[m]`` and all its layers use the block ids
        ``block_ids[chunk_blk_off[m]:][:chunk_pages[m]]``. ``layer_range``
        (begin, end) loads a subset of the layers. mode "flexible" / "delta" /
        "none" with pos_a / pos_b / chunk_len per chunk as in
        rerotate_scatter_pages; ``scores`` row j is layer j's deviations at
        column score_col[m] + token."""
        _check_indices(block_ids)
        names = names_array(layer_names)
        nl = len(names)
        l0, l1 = layer_range if layer_range is not None else (0, nl)
        so, sop = i64(chunk_stg_off)
        bo, bop = i64(chunk_blk_off)
        pg, pgp = i64(chunk_pages)
        M = len(so)
        if not (len(bo) == len(pg) == M):
            raise RuntimeError("chunk arrays must have the same length")
        code = mode_code(mode)
        keep = []
        pap = pbp = lnp = None
        if code != _lib.ROPE_NONE:
            pa, pap = i64(pos_a)
            ln, lnp = i64(chunk_len)
            pb, pbp = i64(pos_b if pos_b is not None else [0] * M)
            if not (len(pa) == len(ln) == len(pb) == M):
                raise RuntimeError("chunk position arrays must have one entry per chunk")
            keep += [pa, ln, pb]
        sptr, ld, colp = None, 0, None
        if scores is not None:
            if not scores.is_cuda or scores.dtype != torch.float32 or scores.dim() != 2 or scores.stride(1) != 1:
                raise RuntimeError("scores must be a CUDA float32 matrix with unit column stride")
            if score_col is None or scores.shape[0] < l1:
                raise RuntimeError("scores need score_col and one row per layer")
            col, colp = i64(score_col)
            if len(col) != M:
                raise RuntimeError("score_col must have one entry per chunk")
            if code != _lib.ROPE_NONE and M and int((col + keep[1]).max()) > scores.shape[1]:
                raise RuntimeError("score_col + chunk_len exceeds the score row")
            keep.append(col)
            sptr, ld = C.c_void_p(scores.data_ptr()), scores.stride(0)
        dev = block_ids.device.index
        s = _stream_ptr(stream, dev)
        _record(block_ids, stream)
        check(self._lib.daric_copier_load_chunks(
            self._h, nl, names, int(l0), int(l1), M, sop, bop, pgp, C.c_void_p(block_ids.data_ptr()),
            block_ids.numel(), dev, code, pap, pbp, lnp, sptr, ld, colp, C.c_void_p(s)))
        del keep

    def rerotate_inplace(self, layer_names: Sequence[str], mode, block_table: torch.Tensor,
                         seg_blk_off: Sequence[int], seg_tok_start: Sequence[int], seg_tok_len: Sequence[int],
                         seg_pos_a: Sequence[int], seg_pos_b: Optional[Sequence[int]] = None,
                         stream: int = 0) -> None:
        """Re-rotates K of every listed layer in place, one launch for all
        layers (replaces the per-layer Triton launches, adapter.py:174-194,
        268-295). Segment s rotates request positions
        [tok_start, tok_start + tok_len) whose slots come from
        block_table[seg_blk_off[s]:]; its token t uses positions
        (pos_a + t, pos_b + t) in "flexible" mode and pos_a in "delta" mode."""
        if len(layer_names) == 0 or len(seg_tok_len) == 0:
            return
        if not block_table.is_cuda or block_table.dtype != torch.int32 or not block_table.is_contiguous():
            raise RuntimeError("block_table must be a contiguous CUDA int32 tensor")
        code = mode_code(mode)
        bo, bop = i64(seg_blk_off)
        ts, tsp = i64(seg_tok_start)
        tl, tlp = i64(seg_tok_len)
        pa, pap = i64(seg_pos_a)
        pb, pbp = i64(seg_pos_b if seg_pos_b is not None else [0] * len(pa))
        if not (len(bo) == len(ts) == len(tl) == len(pa) == len(pb)):
            raise RuntimeError("segment arrays must have the same length")
        dev = block_table.device.index
        s = _stream_ptr(stream, dev)
        _record(block_table, stream)
        check(self._lib.daric_copier_rerotate_inplace(
            self._h, len(layer_names), names_array(layer_names), code, len(tl),
            C.c_void_p(block_table.data_ptr()), block_table.numel(), bop, tsp, tlp, pap, pbp, C.c_void_p(s)))


def _as_uint8_ptr(t: torch.Tensor, what: str) -> int:
    if t.dtype != torch.uint8:
        raise RuntimeError(f"expected scalar type Byte for {what} but found {t.dtype}")
    return t.data_ptr()


def _check_regions(a: torch.Tensor, a_off, b: torch.Tensor, b_off, sizes) -> None:
    # The reference does not bound-check these regions; a bad region here
    # raises instead of letting the copy engine touch foreign memory.
    z = np.asarray(sizes, np.int64)
    for t, off, what in ((a, a_off, "source"), (b, b_off, "destination")):
        o = np.asarray(off, np.int64)
        if len(o) != len(z):
            raise RuntimeError("offsets and sizes must have the same length")
        if len(z) and ((o < 0).any() or (z < 0).any() or (o + z).max() > t.numel()):
            raise RuntimeError(f"copy region outside the {what} buffer")


def batched_memcpy_d2h(staging: torch.Tensor, shm: torch.Tensor, stg_offsets: Sequence[int],
                       shm_offsets: Sequence[int], sizes: Sequence[int], stream: int = 0) -> None:
    """One copy-engine cudaMemcpyAsync (D2H) per region (helpers.cu:187-217).
    ``shm`` must be page-locked for the copy to be asynchronous."""
    n = len(sizes)
    if n == 0:
        return
    _check_regions(staging, stg_offsets, shm, shm_offsets, sizes)
    src = _as_uint8_ptr(staging, "staging")
    dst = _as_uint8_ptr(shm, "shm")
    dev = staging.device.index if staging.is_cuda else torch.cuda.current_device()
    s = _stream_ptr(stream, torch.cuda.current_device())
    a, ap = i64(stg_offsets)
    b, bp = i64(shm_offsets)
    z, zp = i64(sizes)
    check(_lib.load().daric_batched_memcpy_d2h(C.c_void_p(src), C.c_void_p(dst), n, ap, bp, zp, dev, C.c_void_p(s)))


def batched_memcpy_h2d(shm: torch.Tensor, staging: torch.Tensor, shm_offsets: Sequence[int],
                       stg_offsets: Sequence[int], sizes: Sequence[int], stream: int = 0) -> None:
    """One copy-engine cudaMemcpyAsync (H2D) per region (helpers.cu:219-248).
    ``shm`` must be page-locked for the copy to be asynchronous."""
    n = len(sizes)
    if n == 0:
        return
    _check_regions(shm, shm_offsets, staging, stg_offsets, sizes)
    src = _as_uint8_ptr(shm, "shm")
    dst = _as_uint8_ptr(staging, "staging")
    dev = staging.device.index if staging.is_cuda else torch.cuda.current_device()
    s = _stream_ptr(stream, torch.cuda.current_device())
    a, ap = i64(shm_offsets)
    b, bp = i64(stg_offsets)
    z, zp = i64(sizes)
    check(_lib.load().daric_batched_memcpy_h2d(C.c_void_p(src), C.c_void_p(dst), n, ap, bp, zp, dev, C.c_void_p(s)))
