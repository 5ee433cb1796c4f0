"""Full-size (32 layers x 8K tokens, 2.1 GB per load)
properties of the fused load:

* the fused kernel (one pass, copy-engine pipeline) equals the two-pass path
  the reference runs — plain scatter_pages, then the Adapter's flexible
  re-rotation in place — bit for bit over every layer;
* sampled pages equal the CPU oracle.
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from daric_b200 import _lib
from daric_b200.adaption import Adapter, AdaptionConfig
from daric_b200.cache_ops import CacheCopier
from oracle import numerics as N
from oracle import rerotate as R

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def loaded():
    import bench
    wl = bench.Workload(torch.device("cuda", 0), seed=3)
    wl.load()
    torch.cuda.synchronize()
    assert _lib.device_errors(0) == 0
    yield wl
    del wl
    torch.cuda.empty_cache()


def test_fused_equals_scatter_then_inplace_rotation(loaded):
    wl = loaded
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


def test_sampled_pages_match_oracle(loaded):
    wl = loaded
    rng = np.random.default_rng(0)
    L = len(wl.names)
    table = wl.table.view(torch.int16).cpu().numpy().view(np.uint16)
    rot = R.Rotary(table, "bf16", 128, True)
    page_bytes = 16 * 8 * 128 * 2
    for _ in range(24):
        m = int(rng.integers(len(wl.chunk_blocks)))
        l = int(rng.integers(L))
        pg = int(rng.integers(len(wl.chunk_blocks[m])))
        j = m * L + l
        off = int(wl.plan.offsets[j])
        n_sel = len(wl.chunk_blocks[m])
        k_src = wl.staging[off + pg * page_bytes: off + (pg + 1) * page_bytes]
        v_src = wl.staging[off + (n_sel + pg) * page_bytes: off + (n_sel + pg + 1) * page_bytes]
        raw = np.concatenate([k_src.cpu().numpy(), v_src.cpu().numpy()]).view(np.uint16)
        layer = R.KLayer(raw.copy(), (2, 1, 16, 8, 128), (16 * 8 * 128, 16 * 8 * 128, 8 * 128, 128, 1), False, "bf16")
        t = pg * 16 + np.arange(16)
        c, s = R.flexible_factors(rot, wl.old_pos[m] + t, wl.new_pos[m] + t)
        if wl.old_pos[m] != wl.new_pos[m]:
            R.rotate_tokens(layer, rot, np.arange(16), c, s)
        blk = wl.chunk_blocks[m][pg]
        name = wl.plan.layer_names[j]  # the store orders layers by sorted name
        got = wl.kv[name][:, blk].contiguous().view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)
        np.testing.assert_array_equal(got, layer.raw)
