"""KV-cache layer topology used by the re-rotation paths.

Mirrors the fields of the reference's ``LayerCacheTopo`` / ``CacheTopo``
(daric/configs/engine.py:11-70) that the hot path reads: per layer its KV
group, logical block size, block byte size and whether the layer tensor is
page-first. ``from_reference`` adapts a live reference topology object.
"""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class LayerCacheTopo:
    group_idx: int
    logical_block_size: int
    block_byte_size: int
    page_first: bool
    is_mamba: bool = False


@dataclass
class CacheTopo:
    layers: dict[str, LayerCacheTopo]
    groups: list[list[str]] = field(default_factory=list)

    def get_all_layer_names(self) -> list[str]:
        # sorted order = the store's per-chunk layer order (engine.py:25-27)
        return sorted(self.layers.keys())

    def get_layer_idx(self, layer_name: str) -> int:
        return self.get_all_layer_names().index(layer_name)

    def get_group_idx(self, layer_name: str) -> int:
        for g, members in enumerate(self.groups):
            if layer_name in members:
                return g
        raise ValueError(f"Layer {layer_name} not found in any group.")

    def get_all_group_block_size(self) -> list[int]:
        out = []
        for members in self.groups:
            sizes = {self.layers[n].logical_block_size for n in members}
            if len(sizes) != 1:
                raise AssertionError(f"All layers in a group must have the same logical_block_size. Group: {members}")
            out.append(sizes.pop())
        return out

    @staticmethod
    def single_group(layer_names, block_size: int, block_byte_size: int, page_first: bool = False) -> "CacheTopo":
        names = list(layer_names)
        layers = {n: LayerCacheTopo(0, block_size, block_byte_size, page_first) for n in names}
        return CacheTopo(layers=layers, groups=[names])

    @staticmethod
    def from_reference(topo) -> "CacheTopo":
        """Copies a reference ``CacheTopo`` (duck-typed)."""
        layers = {n: LayerCacheTopo(l.group_idx, l.logical_block_size, l.block_byte_size, bool(l.page_first),
                                    bool(getattr(l, "is_mamba", False)))
                  for n, l in topo.layers.items()}
        return CacheTopo(layers=layers, groups=[list(g) for g in topo.groups])
