"""Case builders shared by the GPU parity tests."""
from __future__ import annotations

import numpy as np
import torch

from oracle import numerics as N
from oracle import pages as P
from oracle import rerotate as R

TORCH_DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32, "fp8": torch.uint8}
RAW_NP = {"bf16": np.uint16, "f16": np.uint16, "f32": np.float32, "fp8": np.uint8}


def layout_shape(layout: str, nb: int, bs: int, H: int, D: int):
    """(shape, page_first) of the vLLM KV layouts the reference handles."""
    if layout == "5d":
        return (2, nb, bs, H, D), False
    if layout == "5dpf":
        return (nb, 2, bs, H, D), True
    if layout == "4d":
        return (nb, H, bs, 2 * D), True
    if layout == "3d":
        return (nb, bs, H * D), True
    raise ValueError(layout)


def random_values(shape, dt: str, gen: torch.Generator, device="cuda", outliers: bool = True) -> torch.Tensor:
    x = torch.randn(shape, generator=gen, dtype=torch.float32)
    if outliers and x.shape[-1] >= 8:
        ch = torch.randperm(x.shape[-1], generator=gen)[:4]
        x[..., ch] *= 8.0
    if dt == "fp8":
        bits = N.f32_to_e4m3((x * 4).numpy())
        return torch.from_numpy(bits).to(device)
    return x.to(TORCH_DT[dt]).to(device)


def raw_np(t: torch.Tensor, dt: str) -> np.ndarray:
    """Raw element array of a contiguous tensor (copy on the host)."""
    b = t.contiguous().view(torch.uint8).cpu().numpy().reshape(-1)
    return b.view(RAW_NP[dt]).copy()


def bytes_np(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.uint8).cpu().numpy().reshape(-1).copy()


def table_tensor(max_pos: int, rot_dim: int, base: float, tab_dt: str, device="cuda"):
    raw = R.rope_table(max_pos, rot_dim, base, tab_dt)
    t = torch.from_numpy(raw.view(np.int16) if raw.dtype == np.uint16 else raw)
    if tab_dt == "bf16":
        t = t.view(torch.bfloat16)
    elif tab_dt == "f16":
        t = t.view(torch.float16)
    return t.to(device), raw


def oracle_layer(t: torch.Tensor, dt: str, page_first: bool):
    """(LayerMem for byte copies, KLayer for rotation) sharing one host buffer."""
    mem = bytes_np(t)
    es = t.element_size()
    lm = P.LayerMem(mem, tuple(t.shape), tuple(t.stride()), es, page_first)
    kl = R.KLayer(mem.view(RAW_NP[dt]), tuple(t.shape), tuple(t.stride()), page_first, dt)
    return lm, kl


def unique_blocks(rng: np.random.Generator, nb: int, counts, with_null: bool = False):
    """Disjoint block-id lists (ids >= 1); optionally one id 0 in the first list."""
    total = int(sum(counts))
    assert total <= nb - 1
    perm = rng.permutation(np.arange(1, nb))[:total]
    out, k = [], 0
    for c in counts:
        out.append([int(x) for x in perm[k:k + c]])
        k += c
    if with_null and out and out[0]:
        out[0][min(1, len(out[0]) - 1)] = 0
    return out
