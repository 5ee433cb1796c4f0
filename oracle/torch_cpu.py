"""TEST INFRASTRUCTURE ONLY — multi-threaded torch-CPU restatement of the
reused-KV step, timed as the CPU baseline (``bench.py --impl reference`` and
the ``cpu_baseline`` leg). The reference has no CPU implementation of this
path (its scatter is CUDA, csrc/cache_ops/kernels.cu:86-123; its rotation is
Triton, daric/adaption/adapter.py:30-88), so the baseline is the reference's
math on torch CPU ops with every host thread:

  * scatter: staging pages -> paged layer via index_copy_ (kernels.cu:86-123)
  * flexible re-rotation of K with the bf16-combined table (adapter.py:230-295)
  * top-k selection per layer + slot mapping (torch.topk)

Checked bit-exact against the numpy oracle by tests/test_host.py.
"""
from __future__ import annotations

import torch


def combined_table(table: torch.Tensor, old_pos: torch.Tensor, new_pos: torch.Tensor):
    """adapter.py:276-283 on CPU tensors in the table dtype."""
    oc, os_ = table.index_select(0, old_pos).chunk(2, dim=-1)
    nc, ns = table.index_select(0, new_pos).chunk(2, dim=-1)
    return (nc * oc + ns * os_).contiguous(), (ns * oc - nc * os_).contiguous()


def rotate_neox_(k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> None:
    """In place: k [T, H, D] (cache dtype), cos/sin [T, D/2] -> fp32 rotation
    rounded to the cache dtype (adapter.py:64-73)."""
    half = cos.shape[-1]
    k1 = k[..., :half].float()
    k2 = k[..., half:2 * half].float()
    c = cos.float()[:, None, :]
    s = sin.float()[:, None, :]
    o1 = k1 * c - k2 * s
    o2 = k2 * c + k1 * s
    k[..., :half] = o1.to(k.dtype)
    k[..., half:2 * half] = o2.to(k.dtype)


def reused_kv_step(kv_layers: list[torch.Tensor], staging: torch.Tensor, chunk_blocks: list[torch.Tensor],
                   chunk_len: list[int], old_pos: list[int], new_pos: list[int], table: torch.Tensor,
                   scores: torch.Tensor, k: int, block_table: torch.Tensor, block_size: int):
    """One CPU pass over chunks stored layer-major in ``staging`` (per chunk,
    per layer [2][n_pages][bs][H][D]) into non-page-first layers
    (2, nb, bs, H, D); then per-layer top-k + slots. Returns (idx, slots)."""
    L = len(kv_layers)
    _, nb, bs, H, D = kv_layers[0].shape
    page = bs * H * D
    off = 0
    stg = staging.view(kv_layers[0].dtype)
    for m, blocks in enumerate(chunk_blocks):
        n = blocks.numel()
        t = torch.arange(chunk_len[m])
        cos = sin = None
        if old_pos[m] != new_pos[m] and chunk_len[m] > 0:
            cos, sin = combined_table(table, old_pos[m] + t, new_pos[m] + t)
        for l in range(L):
            src = stg[off:off + 2 * n * page].view(2, n, bs, H, D)
            dst = kv_layers[l]
            kv = src.clone()
            if cos is not None:
                kt = kv[0].reshape(n * bs, H, D)[: chunk_len[m]]
                rotate_neox_(kt, cos, sin)
                kv[0].reshape(n * bs, H, D)[: chunk_len[m]] = kt
            keep = blocks != 0
            dst[0].index_copy_(0, blocks[keep].long(), kv[0][keep])
            dst[1].index_copy_(0, blocks[keep].long(), kv[1][keep])
            off += 2 * n * page
    top = torch.topk(scores, k, dim=-1).indices.sort(dim=-1).values
    slots = block_table.long()[top // block_size] * block_size + top % block_size
    return top, slots
