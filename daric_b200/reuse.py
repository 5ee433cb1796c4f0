"""Reused-KV load path: store staging -> re-rotated paged KV in one launch.

The reference splits this across two processes: the KV store scatters the
staged chunk bytes into the paged cache (management/service/gpu_kv_io.py:
518-584 -> CacheCopier.scatter_pages) and the vLLM worker later re-rotates K
in place (integration/vllm/worker.py:208-217 -> Adapter.apply_rerotate_load).
``ReusedKVLoader`` runs both as the fused ``rerotate_scatter_pages`` kernel
wherever the staging buffer and the rotary tables are visible together
(worker-owned staging).

The staging layout is the store's wire format (gpu_kv_io.py:320-379): per
chunk, for each layer in sorted name order, ``[prefix][n_sel pages][page
bytes]``, chunks back to back.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np
import torch

from .cache_ops import CacheCopier
from .topo import CacheTopo

__all__ = ["ChunkPlan", "LayerwiseLoad", "LoadPlan", "ReusedKVLoader", "build_chunk_plan", "build_load_plan",
           "layer_block_bytes"]


def layer_block_bytes(kv: torch.Tensor, page_first: bool) -> int:
    """Bytes one page (block) of a layer occupies in the store: prefix x page
    span (the ``block_byte_size`` the store multiplies by len(block_ids))."""
    if page_first:
        return int(np.prod(kv.shape[1:])) * kv.element_size()
    return int(kv.shape[0]) * int(np.prod(kv.shape[2:])) * kv.element_size()


@dataclass
class LoadPlan:
    """Host-side job arrays of one load (one job per chunk x layer)."""
    layer_names: list[str]
    offsets: np.ndarray          # staging byte offset of each job
    byte_sizes: np.ndarray       # bytes of each job
    indices_offsets: np.ndarray  # num_jobs + 1
    indices_flat: torch.Tensor   # device int32 block ids
    job_meta: np.ndarray         # chunk of each job
    job_layer: np.ndarray        # layer index (sorted order) of each job
    chunk_offsets: np.ndarray    # staging offset of each chunk
    chunk_sizes: np.ndarray      # staging bytes of each chunk
    total_bytes: int = 0
    extra: dict = field(default_factory=dict)

    @property
    def c_names(self):
        """Layer-name array in C form, built once per plan."""
        if "c_names" not in self.extra:
            from ._lib import names_array
            self.extra["c_names"] = names_array(self.layer_names)
        return self.extra["c_names"]


@dataclass
class ChunkPlan:
    """One descriptor per chunk (the device derives each (chunk, layer) job):
    chunk m starts at ``chunk_offsets[m]`` in staging, has ``chunk_pages[m]``
    pages and its block ids at ``block_ids[chunk_blk_off[m]:]``; layer j's
    bytes of the chunk start ``chunk_pages[m] * page_off[j]`` into it."""
    layer_names: list[str]       # every layer, store (sorted) order
    c_names: object              # the same as a C array
    page_off: np.ndarray         # bytes per chunk page of the layers before j (num_layers + 1)
    chunk_offsets: np.ndarray
    chunk_pages: np.ndarray
    chunk_blk_off: np.ndarray
    block_ids: torch.Tensor      # device int32, the chunks' block lists back to back
    chunk_sizes: np.ndarray
    total_bytes: int = 0

    def layer_regions(self, l0: int, l1: int, base: Optional[np.ndarray] = None):
        """(offsets, sizes) of every chunk's bytes of layers [l0, l1), which
        are contiguous inside a chunk; ``base`` replaces the chunk offsets
        (e.g. the chunks' offsets in host memory)."""
        b = self.chunk_offsets if base is None else np.asarray(base, np.int64)
        return b + self.chunk_pages * self.page_off[l0], self.chunk_pages * (self.page_off[l1] - self.page_off[l0])


class LayerwiseLoad:
    """Completion events of a layer-wise load: layer j of the store order is
    in the paged cache once ``wait_layer(j)`` has been honoured by a stream."""

    def __init__(self):
        self.events: list[tuple[int, torch.cuda.Event]] = []  # (end layer of a step, its event)

    def wait_layer(self, layer: int, stream: Optional[torch.cuda.Stream] = None) -> None:
        s = stream if stream is not None else torch.cuda.current_stream()
        for end, ev in self.events:
            if layer < end:
                s.wait_event(ev)
                return
        raise IndexError(f"layer {layer} is not part of this load")


def build_load_plan(topo: CacheTopo, bpb: dict[str, int], block_ids_list: Sequence[Sequence[Sequence[int]]],
                    device, layer_name: Optional[str] = None, base_offset: int = 0) -> LoadPlan:
    """Job arrays for chunks ``block_ids_list[m][group] -> block ids``,
    following ``KVIOManager._build_copy_plan`` (gpu_kv_io.py:334-379) with the
    chunks packed from ``base_offset``. ``bpb[name]`` = bytes per block."""
    names = [layer_name] if layer_name is not None else topo.get_all_layer_names()
    L = len(names)
    groups = np.array([topo.get_group_idx(n) for n in names], np.int64)
    bpbs = np.array([bpb[n] for n in names], np.int64)
    M = len(block_ids_list)
    counts = np.array([[len(block_ids_list[m][g]) for g in groups] for m in range(M)], np.int64).reshape(M, L)
    sizes = counts * bpbs[None, :]
    chunk_sizes = sizes.sum(axis=1)
    chunk_offsets = base_offset + np.concatenate([[0], np.cumsum(chunk_sizes)[:-1]]).astype(np.int64)
    intra = np.concatenate([np.zeros((M, 1), np.int64), np.cumsum(sizes, axis=1)[:, :-1]], axis=1)
    offsets = (chunk_offsets[:, None] + intra).reshape(-1)
    flat_counts = counts.reshape(-1)
    indices_offsets = np.concatenate([[0], np.cumsum(flat_counts)]).astype(np.int64)
    flat = np.empty(int(indices_offsets[-1]), np.int32)
    k = 0
    for m in range(M):
        for g in groups:
            ids = block_ids_list[m][g]
            flat[k:k + len(ids)] = np.asarray(ids, np.int32)
            k += len(ids)
    if not flat.size:
        idx = torch.zeros(0, dtype=torch.int32, device=device)
    elif torch.device(device).type == "cuda":
        # pinned source: the upload is queued on the stream instead of
        # blocking the host (the caching host allocator keeps the buffer
        # until the copy has run)
        idx = torch.from_numpy(flat).pin_memory().to(device, non_blocking=True)
    else:
        idx = torch.from_numpy(flat).to(device)
    return LoadPlan(
        layer_names=names * M, offsets=offsets, byte_sizes=sizes.reshape(-1), indices_offsets=indices_offsets,
        indices_flat=idx, job_meta=np.repeat(np.arange(M, dtype=np.int64), L),
        job_layer=np.tile(np.arange(L, dtype=np.int64), M), chunk_offsets=chunk_offsets,
        chunk_sizes=chunk_sizes, total_bytes=int(chunk_sizes.sum()))


def build_chunk_plan(topo: CacheTopo, bpb: dict[str, int], block_ids_list, device, base_offset: int = 0,
                     group: int = 0) -> ChunkPlan:
    """Chunk plan of chunks ``block_ids_list[m]`` (a block-id list, or a
    tuple of lists per KV group, of which ``group`` is used): the store's
    layout (gpu_kv_io.py:355-373) packed from ``base_offset``, in O(chunks)
    host work and one block-id list per chunk. Every layer must belong to KV
    group ``group``."""
    names = topo.get_all_layer_names()
    if any(topo.get_group_idx(n) != group for n in names):
        raise RuntimeError("a chunk plan needs every layer in one KV group; use build_load_plan instead")
    per_page = np.array([bpb[n] for n in names], np.int64)
    page_off = np.concatenate([[0], np.cumsum(per_page)]).astype(np.int64)
    lists = [np.asarray(b[group] if isinstance(b, tuple) else b, np.int32).reshape(-1) for b in block_ids_list]
    pages = np.array([len(x) for x in lists], np.int64)
    sizes = pages * page_off[-1]
    offs = base_offset + np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.int64)
    blk_off = np.concatenate([[0], np.cumsum(pages)[:-1]]).astype(np.int64)
    flat = np.concatenate(lists) if lists else np.zeros(0, np.int32)
    if not flat.size:
        ids = torch.zeros(0, dtype=torch.int32, device=device)
    elif torch.device(device).type == "cuda":
        ids = torch.from_numpy(flat).pin_memory().to(device, non_blocking=True)
    else:
        ids = torch.from_numpy(flat).to(device)
    try:
        from ._lib import names_array
        c_names = names_array(names)
    except Exception:  # the C name array is only needed for launches
        c_names = None
    return ChunkPlan(layer_names=list(names), c_names=c_names, page_off=page_off, chunk_offsets=offs,
                     chunk_pages=pages, chunk_blk_off=blk_off, block_ids=ids, chunk_sizes=sizes,
                     total_bytes=int(sizes.sum()))


class ReusedKVLoader:
    """Fused reused-KV loader bound to a set of paged KV layers, their rotary
    tables and a device staging buffer (uint8, 1-D)."""

    def __init__(self, kvcaches: dict[str, torch.Tensor], topo: CacheTopo, staging: torch.Tensor,
                 rotary: dict[str, tuple[torch.Tensor, int, bool]]):
        self.kvcaches = kvcaches
        self.topo = topo
        self.staging = staging
        self.copier = CacheCopier()
        self.bpb = {}
        for n, t in kvcaches.items():
            pf = bool(topo.layers[n].page_first)
            self.copier.register_layer(n, t, pf)
            self.bpb[n] = layer_block_bytes(t, pf)
            table, rot_dim, neox = rotary[n]
            self.copier.register_rotary(n, table, rot_dim, neox)
        self.copier.register_store(staging)

    def plan(self, block_ids_list, layer_name: Optional[str] = None, base_offset: int = 0) -> LoadPlan:
        dev = self.staging.device
        return build_load_plan(self.topo, self.bpb, block_ids_list, dev, layer_name, base_offset)

    def plan_chunks(self, block_ids_list, base_offset: int = 0, group: int = 0) -> ChunkPlan:
        """Chunk plan (build_chunk_plan) on this loader's staging device."""
        return build_chunk_plan(self.topo, self.bpb, block_ids_list, self.staging.device, base_offset, group)

    def load_chunks(self, cp: ChunkPlan, *, mode: str = "flexible", pos_a=None, pos_b=None, chunk_len=None,
                    scores: Optional[torch.Tensor] = None, score_col=None, layer_range=None,
                    stream: int = 0) -> None:
        """Fused load of a chunk plan (all layers, or ``layer_range``); the
        (chunk, layer) jobs are built on the device."""
        self.copier.load_chunks(cp.c_names, cp.chunk_offsets, cp.chunk_blk_off, cp.chunk_pages, cp.block_ids,
                                mode, pos_a, pos_b, chunk_len, scores=scores, score_col=score_col,
                                layer_range=layer_range, stream=stream)

    def load_layerwise(self, cp: ChunkPlan, host: torch.Tensor, host_offsets=None, *, layers_per_step: int = 4,
                       mode: str = "flexible", pos_a=None, pos_b=None, chunk_len=None,
                       scores: Optional[torch.Tensor] = None, score_col=None,
                       copy_stream: Optional[torch.cuda.Stream] = None) -> LayerwiseLoad:
        """Layer-wise pipelined load from pinned host memory (the store's
        shared memory): for each step of ``layers_per_step`` layers, the
        chunks' bytes of those layers go host -> staging on ``copy_stream``
        (one copy per chunk) while the current stream rotates and scatters
        the previous step's layers. The reference loads layer by layer with
        one store round trip each (integration/vllm/worker.py:219-231,
        management/storage.py:235-256). Returns the per-layer completion
        events. ``host_offsets``: each chunk's offset in ``host`` (default:
        the staging offsets)."""
        from .cache_ops import batched_memcpy_h2d
        compute = torch.cuda.current_stream(self.staging.device)
        if copy_stream is None:
            if getattr(self, "_copy_stream", None) is None:
                self._copy_stream = torch.cuda.Stream(self.staging.device)
            copy_stream = self._copy_stream
        # staging is rewritten: earlier work on the current stream (the
        # previous load reading it) must be done first
        copy_stream.wait_stream(compute)
        out = LayerwiseLoad()
        L = len(cp.layer_names)
        k = max(1, int(layers_per_step))
        for l0 in range(0, L, k):
            l1 = min(L, l0 + k)
            stg_off, size = cp.layer_regions(l0, l1)
            src_off, _ = cp.layer_regions(l0, l1, base=host_offsets)
            batched_memcpy_h2d(host, self.staging, src_off, stg_off, size, stream=copy_stream.cuda_stream)
            ev = torch.cuda.Event()
            ev.record(copy_stream)
            compute.wait_event(ev)
            self.load_chunks(cp, mode=mode, pos_a=pos_a, pos_b=pos_b, chunk_len=chunk_len, scores=scores,
                             score_col=score_col, layer_range=(l0, l1))
            done = torch.cuda.Event(enable_timing=True)
            done.record(compute)
            out.events.append((l1, done))
        return out

    def load(self, plan: LoadPlan, *, mode: str = "flexible", pos_a: Sequence[int], pos_b=None,
             chunk_len: Sequence[int], scores: Optional[torch.Tensor] = None,
             score_col: Optional[Sequence[int]] = None, stream: int = 0) -> None:
        """Scatters + re-rotates every chunk of ``plan``. ``mode`` "flexible":
        pos_a = saved positions, pos_b = new positions; "delta": pos_a =
        deltas. With ``scores`` [num_layers, T], token t of chunk m in layer j
        gets its deviation at [j, score_col[m] + t]."""
        kw = {}
        if scores is not None:
            kw = dict(scores=scores, job_score_row=plan.job_layer, meta_score_col=score_col)
        self.copier.rerotate_scatter_pages(
            plan.c_names, plan.offsets, plan.byte_sizes, plan.indices_flat, plan.indices_offsets,
            plan.job_meta, mode, pos_a, pos_b, chunk_len, stream=stream, **kw)
