"""Full-size parity of the fused load with the CPU oracle, at the BASELINE
shapes (bench.Workload inputs):

* config 1 (one layer, one 512-token chunk moved by a random delta): every
  page and every deviation score;
* config 2 (32 layers x 8K tokens, 2.1 GB per load): every page of every
  layer against the oracle: K rotated by the flexible factors, V copied,
  byte for byte;
* config 4, the 70B shape as the rank-0 KV-head shard of TP8 (1 head) and
  TP4 (2 heads), 80 layers x 32K tokens, with the per-token deviation
  scores: every page against the oracle and every score at rtol 1e-3;
* config 3 (64 requests x 6 chunks of 256-1024 tokens, 28 layers, 4 heads,
  28 GB): the oracle on every 8th chunk (all layers), and on the GPU the V
  planes of every chunk equal to the staged bytes;
* the fused kernel also equals the two-pass path the reference runs (plain
  scatter_pages, then the Adapter's flexible re-rotation in place).
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from daric_b200 import _lib
from daric_b200.adaption import Adapter, AdaptionConfig
from daric_b200.cache_ops import CacheCopier
from oracle import rerotate as R

pytestmark = pytest.mark.gpu


def _raw16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def check_against_oracle(wl, chunks, scores=None):
    """Chunk m, layer l (store order) of the fused load against the oracle."""
    c = wl.cfg
    L, H, D, bs = c["layers"], wl.heads, c["head_dim"], c["block_size"]
    rot = R.Rotary(_raw16(wl.table).reshape(-1, D), "bf16", D, True)
    sc = scores.cpu().numpy() if scores is not None else None
    for m in chunks:
        names = wl.plan.layer_names[m * L:(m + 1) * L]
        blocks = wl.chunk_blocks[m]
        n_sel, n_tok = len(blocks), wl.chunk_len[m]
        off = int(wl.plan.chunk_offsets[m])
        size = int(wl.plan.chunk_sizes[m])
        stg = _raw16(wl.staging[off:off + size]).reshape(L, 2, n_sel * bs, H, D)
        bt = torch.tensor(blocks, dtype=torch.long, device=wl.device)
        got = _raw16(torch.stack([wl.kv[n].index_select(1, bt) for n in names])).reshape(L, 2, n_sel * bs, H, D)
        t = np.arange(n_tok)
        old, new = wl.old_pos[m], wl.new_pos[m]
        exp_k = stg[:, 0].copy()
        dev = np.zeros((L, n_tok), np.float32)
        if old != new:
            cs, sn = R.flexible_factors(rot, old + t, new + t)
            exp_k[:, :n_tok], dev = R.rotate_dense(stg[:, 0, :n_tok], rot, "bf16", cs, sn)
        bad = np.nonzero(got[:, 0] != exp_k)
        assert bad[0].size == 0, f"chunk {m}: {bad[0].size} K elements differ (layers {np.unique(bad[0])[:4]})"
        np.testing.assert_array_equal(got[:, 1], stg[:, 1], err_msg=f"chunk {m}: V differs")
        if sc is not None:
            col = int(wl.score_col[m])
            np.testing.assert_allclose(sc[:, col:col + n_tok], dev, rtol=1e-3, atol=1e-5,
                                       err_msg=f"chunk {m}: deviation scores")


def _workload(config, seed, **kw):
    import bench
    wl = bench.Workload(torch.device("cuda", 0), seed=seed, config=config, **kw)
    if wl.cfg["scores"] == "deviation":
        wl.scores.fill_(-1.0)
    wl.load()
    torch.cuda.synchronize()
    assert _lib.device_errors(0) == 0
    return wl


@pytest.fixture(scope="module")
def loaded():
    wl = _workload(2, seed=3)
    yield wl
    del wl
    torch.cuda.empty_cache()


def test_config2_every_page_matches_oracle(loaded):
    check_against_oracle(loaded, range(len(loaded.chunk_len)))


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


@pytest.mark.parametrize("tp", [8, 4])
def test_config4_tp_shard_pages_and_scores_match_oracle(tp):
    """Rank 0's KV-head shard of the 70B shape (80 layers, 32K tokens) with
    deviation scores, every chunk."""
    wl = _workload(4, seed=0, rank=0, world=tp)
    assert wl.heads == 8 // tp
    check_against_oracle(wl, range(len(wl.chunk_len)), scores=wl.scores)
    del wl
    torch.cuda.empty_cache()


def test_config1_single_layer_matches_oracle():
    """one layer, one 512-token chunk rotated by a random
    position delta, deviation scores written by the fused load."""
    wl = _workload(1, seed=0)
    assert len(wl.chunk_len) == 1 and wl.new_pos[0] != wl.old_pos[0]
    check_against_oracle(wl, [0], scores=wl.scores)
    sel = wl.select()
    assert int(sel.count.cpu()[0, 0]) == int(0.15 * 512)
    assert _lib.device_errors(0) == 0
    del wl
    torch.cuda.empty_cache()


def test_config3_batch_matches_oracle():
    """64 requests x 6 chunks of 256-1024 tokens: the oracle on every 8th
    chunk, V of every chunk equal to the staged bytes."""
    wl = _workload(3, seed=0)
    M, L = len(wl.chunk_len), wl.cfg["layers"]
    assert M == 64 * 6 and len(set(wl.chunk_len)) > 10
    check_against_oracle(wl, range(0, M, 8))
    H, D, bs = wl.heads, wl.cfg["head_dim"], wl.cfg["block_size"]
    page = bs * H * D * 2
    for m in range(M):
        n_sel = len(wl.chunk_blocks[m])
        bt = torch.tensor(wl.chunk_blocks[m], dtype=torch.long, device=wl.device)
        for l in range(L):
            j = m * L + l
            off = int(wl.plan.offsets[j]) + n_sel * page
            v_stg = wl.staging[off:off + n_sel * page]
            v_got = wl.kv[wl.plan.layer_names[j]][1].index_select(0, bt).reshape(-1).view(torch.uint8)
            assert torch.equal(v_stg, v_got), (m, l)
    del wl
    torch.cuda.empty_cache()
