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

__all__ = ["LoadPlan", "ReusedKVLoader", "build_load_plan", "layer_block_bytes"]


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
