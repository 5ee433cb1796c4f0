"""TEST INFRASTRUCTURE ONLY — restatement of the reference's RoPE re-rotation
of K in paged KV caches (daric/adaption/adapter.py).

  k_geometry        stride resolution of _launch_triton_rerotate (adapter.py:311-368)
  flexible_factors  bf16-combined table of apply_rerotate_load (adapter.py:276-283)
  delta_factors     table rows of apply_rerotate_multi (adapter.py:181-183)
  rotate_tokens     _fused_rerotate_kernel (adapter.py:30-88): fp32 rotation,
                    result rounded to the cache dtype (RTNE; no FMA contraction)
  apply_rerotate_load / apply_rerotate_multi  the two drivers (adapter.py:118-295)

Layers are raw numpy arrays (uint16 for bf16/f16, float32, uint8 for fp8)
holding the layer's memory in element order, with the tensor's sizes and
strides in elements.
"""
from __future__ import annotations

from collections import defaultdict
from dataclasses import dataclass

import numpy as np

from .numerics import DTYPES


@dataclass
class KLayer:
    raw: np.ndarray     # 1-D raw elements of the layer (modified in place)
    sizes: tuple
    strides: tuple
    page_first: bool
    dtype: str          # "bf16" | "f16" | "f32" | "fp8"


@dataclass
class Rotary:
    table: np.ndarray   # raw [max_pos, rot_dim] in table dtype
    dtype: str          # "bf16" | "f16" | "f32"
    rotary_dim: int
    is_neox: bool


def k_geometry(layer: KLayer):
    """(base, stride_b, stride_s, stride_h, page_size, num_head, head_dim) in
    elements, as _launch_triton_rerotate resolves them (adapter.py:311-368)."""
    s, st = layer.sizes, layer.strides
    if len(s) == 5:
        _, _, page_size, num_head, head_dim = s
        if layer.page_first:
            return 0, st[0], st[2], st[3], page_size, num_head, head_dim
        return 0, st[1], st[2], st[3], page_size, num_head, head_dim  # kv_layer[0]
    if len(s) == 4:
        if not layer.page_first:
            raise ValueError("Invalid 4D KV cache for rerotate: page_first must be true")
        _, num_head, page_size, packed = s
        return 0, st[0], st[2], st[1], page_size, num_head, packed // 2
    if len(s) == 3:
        _, page_size, hidden = s
        return 0, st[0], st[1], 0, page_size, 1, hidden
    raise ValueError(f"Unsupported KV cache rank for rerotate: {len(s)}")


def _table_f32(rot: Rotary, positions):
    to_f = DTYPES[rot.dtype][1]
    rows = rot.table[np.asarray(positions, np.int64)]
    half = rot.rotary_dim // 2
    return to_f(np.ascontiguousarray(rows[:, :half])), to_f(np.ascontiguousarray(rows[:, half:]))


def delta_factors(rot: Rotary, positions):
    """cos_sin_cache.index_select(0, positions).chunk(2) (adapter.py:181-182)."""
    return _table_f32(rot, positions)


def flexible_factors(rot: Rotary, old_pos, new_pos):
    """combined_cos = new_cos*old_cos + new_sin*old_sin,
    combined_sin = new_sin*old_cos - new_cos*old_sin, each op rounded to the
    table dtype (torch elementwise ops on the model-dtype table, adapter.py:276-283)."""
    rnd = DTYPES[rot.dtype][3]
    oc, os_ = _table_f32(rot, old_pos)
    nc, ns = _table_f32(rot, new_pos)
    c = rnd(rnd(nc * oc) + rnd(ns * os_))
    s = rnd(rnd(ns * oc) - rnd(nc * os_))
    return c.astype(np.float32), s.astype(np.float32)


def _from_f32_trunc(dtype):
    # fp32 -> bf16 by dropping the low 16 bits: the cast of Triton's CPU
    # interpreter, used only to pin this restatement to the interpreter's
    # golden outputs bit for bit.
    if dtype == "bf16":
        return lambda x: (np.ascontiguousarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)
    return DTYPES[dtype][2]


def rotate_tokens(layer: KLayer, rot: Rotary, gather_idx, cos, sin, rounding: str = "rtne"):
    """_fused_rerotate_kernel (adapter.py:30-88) over tokens `gather_idx`
    (slot = block*page_size + offset) and all heads; returns the per-token
    deviation sum over heads and rotary elements of (K' - K)^2 (fp32).
    rounding "rtne" (GPU casts) or "trunc" (Triton interpreter's bf16 cast)."""
    _, to_f, from_f, _ = DTYPES[layer.dtype]
    if rounding == "trunc":
        from_f = _from_f32_trunc(layer.dtype)
    base, sb, ss, sh, ps, nh, hd = k_geometry(layer)
    idx = np.asarray(gather_idx, np.int64)
    blk, slot = idx // ps, idx % ps
    ho = base + blk * sb + slot * ss                          # [T]
    ho = ho[:, None] + np.arange(nh, dtype=np.int64)[None, :] * sh  # [T, H]
    half = rot.rotary_dim // 2
    d = np.arange(half, dtype=np.int64)
    if rot.is_neox:
        i1 = ho[:, :, None] + d[None, None, :]
        i2 = i1 + half
    else:
        i1 = ho[:, :, None] + 2 * d[None, None, :]
        i2 = i1 + 1
    k1 = to_f(layer.raw[i1])
    k2 = to_f(layer.raw[i2])
    c = np.asarray(cos, np.float32)[:, None, :]
    s = np.asarray(sin, np.float32)[:, None, :]
    o1 = (k1 * c).astype(np.float32) - (k2 * s).astype(np.float32)
    o2 = (k2 * c).astype(np.float32) + (k1 * s).astype(np.float32)
    r1, r2 = from_f(o1), from_f(o2)
    layer.raw[i1] = r1
    layer.raw[i2] = r2
    dev = (to_f(r1) - k1) ** 2 + (to_f(r2) - k2) ** 2
    return dev.astype(np.float32).sum(axis=(1, 2), dtype=np.float32)


def rotate_dense(k_raw: np.ndarray, rot: Rotary, dtype: str, cos, sin):
    """_fused_rerotate_kernel's math (adapter.py:30-88) on a dense block of K
    rows: k_raw [..., T, H, D] raw elements (any leading dims, e.g. layers),
    cos/sin [T, rotary_dim/2] fp32 factors of each token. Returns the rotated
    raw block (RTNE to the cache dtype) and the per-token deviation
    [..., T] = sum over heads and rotary elements of (K' - K)^2 (fp32)."""
    _, to_f, from_f, _ = DTYPES[dtype]
    half = rot.rotary_dim // 2
    out = np.array(k_raw, copy=True)
    d = np.arange(half)
    if rot.is_neox:
        i1, i2 = d, d + half
    else:
        i1, i2 = 2 * d, 2 * d + 1
    k1 = to_f(np.ascontiguousarray(k_raw[..., i1]))
    k2 = to_f(np.ascontiguousarray(k_raw[..., i2]))
    c = np.asarray(cos, np.float32)[:, None, :]
    s = np.asarray(sin, np.float32)[:, None, :]
    o1 = (k1 * c).astype(np.float32) - (k2 * s).astype(np.float32)
    o2 = (k2 * c).astype(np.float32) + (k1 * s).astype(np.float32)
    r1, r2 = from_f(o1), from_f(o2)
    out[..., i1] = r1
    out[..., i2] = r2
    dev = (to_f(r1) - k1) ** 2 + (to_f(r2) - k2) ** 2
    return out, dev.astype(np.float32).sum(axis=(-2, -1), dtype=np.float32)


def gather_index(block_ids, page_size, start, n_tok):
    """slot of positions [start, start+n_tok): block_ids[p//ps]*ps + p%ps (adapter.py:169-170)."""
    pos = np.arange(start, start + n_tok, dtype=np.int64)
    bl = np.asarray(block_ids, np.int64)
    return bl[pos // page_size] * page_size + pos % page_size


def apply_rerotate_multi(layers: dict, rotary: dict, group_of: dict, group_ptrs, block_ids_list,
                         rounding: str = "rtne"):
    """Strict PIC driver (adapter.py:118-194)."""
    delta_list, len_list, spans = [], [], []
    for req, gp in enumerate(group_ptrs):
        n_groups = len(gp) - 1
        if n_groups <= 2:
            continue
        base, n_tok = gp[0], 0
        for i in range(1, n_groups - 1):
            glen = gp[i + 1] - gp[i]
            if glen > 0:
                delta_list.append(gp[i] - base)
                len_list.append(glen)
                n_tok += glen
        if n_tok > 0:
            spans.append((req, gp[1] - base, n_tok))
    if not spans:
        return
    positions = np.repeat(np.asarray(delta_list, np.int64), np.asarray(len_list, np.int64))
    by_group = defaultdict(list)
    for name in layers:
        by_group[group_of[name]].append(name)
    for g, names in by_group.items():
        ps = k_geometry(layers[names[0]])[4]
        idx = np.concatenate([gather_index(block_ids_list[r][g], ps, st, n) for r, st, n in spans])
        for name in names:
            c, s = delta_factors(rotary[name], positions)
            rotate_tokens(layers[name], rotary[name], idx, c, s, rounding)


def apply_rerotate_load(layers: dict, rotary: dict, group_of: dict, metas, layer_name=None,
                        rounding: str = "rtne"):
    """Flexible PIC driver (adapter.py:196-295). metas: objects with
    saved_pos, ptr [start, end) and block_ids (tuple per KV group)."""
    plan = [(m, int(m.saved_pos), int(m.ptr[0]), int(m.ptr[1] - m.ptr[0])) for m in metas]
    plan = [p for p in plan if p[3] > 0 and p[1] != p[2]]
    if not plan:
        return
    old = np.concatenate([np.arange(o, o + n, dtype=np.int64) for _, o, _, n in plan])
    new = np.concatenate([np.arange(w, w + n, dtype=np.int64) for _, _, w, n in plan])
    names = [layer_name] if layer_name is not None else list(layers)
    by_group = defaultdict(list)
    for name in names:
        if name in layers:
            by_group[group_of[name]].append(name)
    for g, gnames in by_group.items():
        ps = k_geometry(layers[gnames[0]])[4]
        idx = np.concatenate([gather_index(m.block_ids[g], ps, 0, n) for m, _, _, n in plan])
        for name in gnames:
            c, s = flexible_factors(rotary[name], old, new)
            rotate_tokens(layers[name], rotary[name], idx, c, s, rounding)


def ulp_diff(a_bits: np.ndarray, b_bits: np.ndarray, dtype: str) -> np.ndarray:
    """Distance in units of last place between two raw arrays (bf16/f16 bits)."""
    def ordered(b):
        b = b.astype(np.int64)
        sign = b & 0x8000
        mag = b & 0x7FFF
        return np.where(sign != 0, -mag, mag)
    if dtype in ("bf16", "f16"):
        return np.abs(ordered(a_bits) - ordered(b_bits))
    raise ValueError(dtype)


def rope_table(max_pos: int, rotary_dim: int, base: float, dtype: str = "bf16") -> np.ndarray:
    """vLLM RotaryEmbedding._compute_cos_sin_cache in fp32 (inv_freq =
    1/base^(arange(0, rd, 2)/rd), t = arange(max_pos), cat(cos, sin)), cast to
    the model dtype. Computed with numpy, so its fp32 cos/sin may differ in
    the last bit from torch's; the kernels consume whatever table is given."""
    inv = (1.0 / (np.float32(base) ** (np.arange(0, rotary_dim, 2, dtype=np.float32) / np.float32(rotary_dim))))
    inv = inv.astype(np.float32)
    t = np.arange(max_pos, dtype=np.float32)
    f = np.outer(t, inv).astype(np.float32)
    cache = np.concatenate([np.cos(f), np.sin(f)], axis=-1).astype(np.float32)
    return DTYPES[dtype][2](cache)
