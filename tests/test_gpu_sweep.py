"""Parity on the data-parallel sweep shape (scaled down):
requests of U[2048, 8192] tokens in 512-token chunks of which a hit-ratio
share is reused, Mistral-7B KV shape (8 heads x 128, theta 1e6), 4 layers.

* the fused load (one pass) equals the two-pass path the reference runs,
  plain scatter_pages and then the Adapter's flexible re-rotation, bit for
  bit, at hit ratios 50% and 95%;
* the selection at recompute ratios 5/15/30% equals the oracle's top-k per
  (layer, request), with its paged-KV slots.
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from daric_b200 import _lib
from daric_b200.adaption import Adapter, AdaptionConfig
from daric_b200.cache_ops import CacheCopier
from daric_b200.select import topk_count
from oracle import select as S

pytestmark = pytest.mark.gpu


def _workload(hit, seed):
    import bench
    cfg = dict(bench.CONFIGS[5], layers=4, requests=4, req_len=(2048, 8192), hit=hit)
    bench.CONFIGS[105] = cfg
    try:
        wl = bench.Workload(torch.device("cuda", 0), seed=seed, config=105)
    finally:
        del bench.CONFIGS[105]
    return wl


@pytest.mark.parametrize("hit", [0.5, 0.95])
def test_fused_load_equals_two_pass_at_hit_ratio(hit):
    wl = _workload(hit, seed=11)
    wl.load()
    torch.cuda.synchronize()
    assert _lib.device_errors(0) == 0
    kv2 = {n: torch.zeros_like(t) for n, t in wl.kv.items()}
    copier = CacheCopier()
    for n, t in kv2.items():
        copier.register_layer(n, t, False)
    copier.register_store(wl.staging)
    p = wl.plan
    copier.scatter_pages(p.c_names, p.offsets, p.byte_sizes, p.indices_flat, p.indices_offsets)
    ad = Adapter(AdaptionConfig(), cache_topo=wl.loader.topo)
    ad.register_kvcaches(kv2)
    for n in kv2:
        ad.register_rotary_embed(n, SimpleNamespace(cos_sin_cache=wl.table, rotary_dim=128, is_neox_style=True))
    metas = [SimpleNamespace(ptr=[new, new + ln], saved_pos=old, block_ids=(blocks,))
             for new, old, ln, blocks in zip(wl.new_pos, wl.old_pos, wl.chunk_len, wl.chunk_blocks)]
    ad.apply_rerotate_load(metas)
    torch.cuda.synchronize()
    assert _lib.device_errors(0) == 0
    for n in wl.kv:
        assert torch.equal(wl.kv[n].view(torch.int16), kv2[n].view(torch.int16)), n


@pytest.mark.parametrize("ratio", [0.05, 0.15, 0.30])
def test_selection_at_recompute_ratio(ratio):
    import bench
    wl = _workload(0.75, seed=12)
    wl.cfg = dict(wl.cfg, ratio=ratio)
    sel = wl.select()
    torch.cuda.synchronize()
    sc = wl.scores_host.numpy()
    bt = wl.block_table.cpu().numpy()
    col = 0
    for r, n in enumerate(wl.seg_len):
        k = topk_count(n, ratio)
        for layer in range(sc.shape[0]):
            exp = S.topk_positions(sc[layer, col:col + n], k)
            idx, slot = sel.get(layer, r)
            np.testing.assert_array_equal(idx.cpu().numpy(), exp)
            np.testing.assert_array_equal(slot.cpu().numpy(),
                                          S.slots(bt[wl.seg_blk_off[r]:], exp, bench.CONFIGS[5]["block_size"]))
        col += n
    assert _lib.device_errors(0) == 0
