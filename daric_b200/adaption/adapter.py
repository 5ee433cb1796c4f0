"""Re-rotation adapter: drop-in for the reference ``daric.adaption.Adapter``
(daric/adaption/adapter.py:91-402).

Same public methods and argument meanings: ``register_kvcaches``,
``register_rotary_embed``, ``register_done``, ``apply_rerotate_multi``
(strict PIC), ``apply_rerotate_load`` (flexible PIC) and
``get_recompute_length``. Instead of building per-token gather indices and
cos/sin tensors on the host and launching the Triton kernel once per layer
(adapter.py:147-194, 225-295), each KV group is rotated by one launch of the
sm_100a in-place kernel over all its layers; the kernel reads the model's
cos/sin table rows itself. Added: ``recompute_slots`` (policy ranges ->
positions and slots on the GPU).
"""
from __future__ import annotations

from collections import defaultdict
from typing import List, Optional

import numpy as np
import torch

from ..cache_ops import CacheCopier
from ..select import ptrs_to_slots
from ..topo import CacheTopo
from .policy import DARICPolicy


def _policy_class():
    """The recompute policy: DARIC's own DARICPolicy when this runs inside a
    DARIC installation (the scheduler logic stays the reference's), else the
    bit-exact restatement in daric_b200.adaption.policy."""
    try:
        from daric.adaption.policy import DARICPolicy as reference_policy  # type: ignore
        return reference_policy
    except Exception:
        return DARICPolicy

__all__ = ["Adapter", "AdaptionConfig"]


class AdaptionConfig:
    """Fields of the reference ``AdaptionConfig`` (configs/engine.py:164-171)."""

    def __init__(self, rerotate: bool = True, recompute: bool = True, recompute_policy: Optional[str] = "daric",
                 recompute_avg_num: int = 16, function: str = "linear", r: float = 0.1):
        self.rerotate = rerotate
        self.recompute = recompute
        self.recompute_policy = recompute_policy
        self.recompute_avg_num = recompute_avg_num
        self.function = function
        self.r = r


def _reference_topo():
    try:  # the reference's process-global topology, when running inside DARIC
        from daric.configs import ProcessLocalConfig  # type: ignore
        return CacheTopo.from_reference(ProcessLocalConfig.cache_topo)
    except Exception as e:  # pragma: no cover - depends on the host process
        raise RuntimeError("Adapter needs a cache topology (cache_topo=...)") from e


def _block_array(ids) -> np.ndarray:
    if isinstance(ids, torch.Tensor):
        return ids.to("cpu", torch.int32).numpy().reshape(-1)
    return np.asarray(ids, dtype=np.int32).reshape(-1)


def _block_list(ids) -> list[int]:
    return _block_array(ids).tolist()


class Adapter:
    def __init__(self, config, cache_topo: Optional[CacheTopo] = None):
        self.config = config
        self.cache_topo = cache_topo if cache_topo is not None else _reference_topo()
        self.num_layers = len(self.cache_topo.get_all_layer_names())
        self.kvcaches: dict[str, torch.Tensor] = {}
        self.rotary_embeds: dict[str, object] = {}
        if config.recompute_policy == "daric":
            self.recompute_policy = _policy_class()(config.recompute_avg_num, function=config.function,
                                                     r=config.r)
        else:
            self.recompute_policy = None
        self.rerotate = config.rerotate
        self._copier: Optional[CacheCopier] = None
        self._table_ptr: dict[str, int] = {}
        self._groups: dict[tuple, dict] = {}  # layer-name tuple -> {group: (names, C name array)}

    # ----------------------------------------------------------- registry --
    def register_kvcaches(self, kvcaches: dict[str, torch.Tensor]) -> None:
        self.kvcaches = kvcaches
        self._copier = CacheCopier()
        for name, t in kvcaches.items():
            self._copier.register_layer(name, t, bool(self.cache_topo.layers[name].page_first))
        self._table_ptr.clear()
        self._groups.clear()

    def register_rotary_embed(self, layer_name: str, rotary_embed) -> None:
        if layer_name not in self.rotary_embeds:
            self.rotary_embeds[layer_name] = rotary_embed

    def register_done(self) -> bool:
        return len(self.rotary_embeds) == self.num_layers

    def _sync_table(self, layer_name: str) -> None:
        # The rotary module may replace its table (vLLM casts it to the query
        # dtype/device on first use), so the pointer is re-read on every call,
        # as the reference reads rotary.cos_sin_cache at call time.
        rot = self.rotary_embeds[layer_name]
        table = rot.cos_sin_cache
        key = (table.data_ptr(), table.device, table.dtype)
        if self._table_ptr.get(layer_name) != key or not self._copier.has_rotary(layer_name):
            self._copier.register_rotary(layer_name, table, int(rot.rotary_dim), bool(rot.is_neox_style))
            self._table_ptr[layer_name] = key

    def _layers_by_group(self, names) -> dict[int, tuple]:
        """KV group -> (layer names, their C name array), cached per name list."""
        key = tuple(names)
        hit = self._groups.get(key)
        if hit is None:
            from .._lib import names_array
            out = defaultdict(list)
            for n in names:
                if n in self.kvcaches:
                    out[self.cache_topo.get_group_idx(n)].append(n)
            hit = {g: (ls, names_array(ls)) for g, ls in out.items()}
            self._groups[key] = hit
        return hit

    # ------------------------------------------------------------ strict --
    def apply_rerotate_multi(self, group_ptrs: List[List[int]], block_ids_list: List[tuple]) -> None:
        """Strict PIC (adapter.py:118-194): every middle group i of a request is
        rotated by delta_i = group_ptr[i] - group_ptr[0] over its tokens."""
        if not self.rerotate:
            return
        assert len(group_ptrs) == len(block_ids_list)
        segs = []  # (request, token start, length, delta)
        for req, gp in enumerate(group_ptrs):
            n_groups = len(gp) - 1
            if n_groups <= 2:
                continue
            base = gp[0]
            for i in range(1, n_groups - 1):
                glen = gp[i + 1] - gp[i]
                if glen > 0:
                    segs.append((req, gp[i] - base, glen, gp[i] - base))
        if not segs:
            return
        for g_idx, (layers, c_names) in self._layers_by_group(self.kvcaches.keys()).items():
            for n in layers:
                self._sync_table(n)
            table, blk_off = self._block_table(
                [block_ids_list[r][g_idx] for r in range(len(block_ids_list))], layers[0])
            self._copier.rerotate_inplace(
                c_names, "delta", table,
                seg_blk_off=[blk_off[r] for r, *_ in segs],
                seg_tok_start=[s for _, s, _, _ in segs],
                seg_tok_len=[n for _, _, n, _ in segs],
                seg_pos_a=[d for *_, d in segs])

    # ---------------------------------------------------------- flexible --
    def apply_rerotate_load(self, metas, layer_name: Optional[str] = None) -> None:
        """Flexible PIC (adapter.py:196-295): chunk tokens saved at
        saved_pos + t are moved to ptr[0] + t with the bf16-combined table."""
        if not self.rerotate:
            return
        plan = []
        for m in metas:
            old_pos, new_pos = int(m.saved_pos), int(m.ptr[0])
            chunk_len = int(m.ptr[1] - m.ptr[0])
            if chunk_len <= 0 or old_pos == new_pos:
                continue
            plan.append((m, old_pos, new_pos, chunk_len))
        if not plan:
            return
        names = [layer_name] if layer_name is not None else list(self.kvcaches.keys())
        for g_idx, (layers, c_names) in self._layers_by_group(names).items():
            for n in layers:
                self._sync_table(n)
            table, blk_off = self._block_table([m.block_ids[g_idx] for m, *_ in plan], layers[0])
            self._copier.rerotate_inplace(
                c_names, "flexible", table,
                seg_blk_off=blk_off,
                seg_tok_start=[0] * len(plan),
                seg_tok_len=[c for *_, c in plan],
                seg_pos_a=[o for _, o, _, _ in plan],
                seg_pos_b=[nw for _, _, nw, _ in plan])

    def _block_table(self, tables, layer_name: str):
        arrs = [_block_array(t) for t in tables]
        offs = np.concatenate([[0], np.cumsum([len(x) for x in arrs])[:-1]]).astype(np.int64).tolist()
        flat = np.concatenate(arrs).astype(np.int32, copy=False) if arrs else np.zeros(0, np.int32)
        dev = self.kvcaches[layer_name].device
        if flat.size == 0:
            flat = np.zeros(1, np.int32)
        # pinned source: the upload is queued on the stream, not run by the
        # host (the caching host allocator keeps the buffer until it has run)
        return torch.from_numpy(flat).pin_memory().to(dev, non_blocking=True), offs

    # --------------------------------------------------------- recompute --
    def get_recompute_length(self, group_ptr: List[int]) -> List[List[int]]:
        if self.recompute_policy is None:
            return []
        return self.recompute_policy.get_recompute_ptrs(group_ptr)

    def recompute_slots(self, group_ptr: List[int], block_ids, block_size: int,
                        no_recompute_length: int = 0):
        """Policy ranges of one request -> (positions, slots) on the GPU,
        keeping the ranges that end beyond ``no_recompute_length``
        (worker.py:324-325)."""
        ranges = [r for r in self.get_recompute_length(group_ptr) if r[1] > no_recompute_length]
        dev = next(iter(self.kvcaches.values())).device
        bt = torch.as_tensor(_block_list(block_ids), dtype=torch.int32).to(dev)
        return ptrs_to_slots(ranges, bt, block_size)
