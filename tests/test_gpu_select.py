"""GPU parity of the recompute selection (bit-exact index lists and slots)."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from daric_b200 import _lib
from daric_b200.adaption import Adapter, AdaptionConfig
from daric_b200.select import ptrs_to_slots, score_select, topk_count
from daric_b200.topo import CacheTopo
from oracle import select as S

pytestmark = pytest.mark.gpu


def _scores(L, T, seed, ties=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.distributions.LogNormal(0.0, 1.0).sample((L, T)) if not ties else \
        torch.randint(0, 7, (L, T), generator=g).float()
    if not ties:
        spikes = torch.rand(L, T, generator=g) < 0.02
        x = torch.where(spikes, x * 20, x)
    return x.float()


# long rows are split over a cluster of up to 8 CTAs (8192: eight slices of
# 1024; 32768: eight of 4096), so ties and the k-th key straddle slices
@pytest.fixture(params=["auto", "1", "2", "8"])
def select_cluster(request, monkeypatch):
    """Runs a test with the planned cluster size and with it pinned."""
    if request.param == "auto":
        monkeypatch.delenv("DARIC_SELECT_CLUSTER", raising=False)
    else:
        monkeypatch.setenv("DARIC_SELECT_CLUSTER", request.param)
    return request.param


@pytest.mark.parametrize("T,ratio,ties", [(512, 0.15, False), (8192, 0.15, False), (1000, 0.3, True),
                                          (33, 0.5, True), (32768, 0.2, False), (8192, 0.3, True),
                                          (20000, 0.05, True)])
def test_topk_matches_oracle(T, ratio, ties, select_cluster):
    L, bs = 4, 16
    sc = _scores(L, T, seed=T, ties=ties)
    nblk = (T + bs - 1) // bs
    bt = torch.randperm(4 * nblk)[:nblk].int() + 1
    out = score_select(sc.cuda(), bt.cuda(), bs, ratio=ratio)
    k = topk_count(T, ratio)
    for l in range(L):
        exp = S.topk_positions(sc[l].numpy(), k)
        idx, slot = out.get(l)
        np.testing.assert_array_equal(idx.cpu().numpy(), exp)
        np.testing.assert_array_equal(slot.cpu().numpy(), S.slots(bt.numpy(), exp, bs))
    assert _lib.device_errors(0) == 0


def test_ragged_segments_threshold_and_edge_cases():
    bs = 16
    lens = [300, 0, 17, 1024, 5]
    ks = [45, 3, 17, 100, 9]        # k == len, k > len
    T = sum(lens)
    sc = _scores(3, T, seed=1)
    sc[0, 3] = float("nan")
    # layer 1, request 3 (columns 317..1340, k=100): 90 scores of 10 and 20
    # ties of 7 across the k boundary -> the 10 lowest-index sevens are taken
    sc[1, 317:1341] = torch.rand(1024) * 0.5
    sc[1, 317 + torch.randperm(1024)[:110]] = 7.0
    sc[1, 317 + torch.randperm(1024)[:90]] = 10.0
    pos0 = [0, 0, 16, 32, 3]
    tables = [torch.randint(1, 1000, ((p + n + bs - 1) // bs + 1,)).int() for p, n in zip(pos0, lens)]
    blk_off = np.concatenate([[0], np.cumsum([len(t) for t in tables])[:-1]])
    bt = torch.cat(tables)
    out = score_select(sc.cuda(), bt.cuda(), bs, seg_len=lens, seg_pos0=pos0, seg_blk_off=blk_off, k=ks)
    col = np.concatenate([[0], np.cumsum(lens)[:-1]])
    for l in range(3):
        for s in range(len(lens)):
            row = sc[l, col[s]:col[s] + lens[s]].numpy()
            exp = S.topk_positions(row, ks[s]) + pos0[s]
            idx, slot = out.get(l, s)
            np.testing.assert_array_equal(idx.cpu().numpy(), exp)
            np.testing.assert_array_equal(slot.cpu().numpy(), S.slots(tables[s].numpy(), exp, bs))
    thr = 2.5
    out = score_select(sc.cuda(), bt.cuda(), bs, seg_len=lens, seg_pos0=pos0, seg_blk_off=blk_off, threshold=thr)
    for l in range(3):
        for s in range(len(lens)):
            row = sc[l, col[s]:col[s] + lens[s]].numpy()
            exp = S.threshold_positions(row, thr) + pos0[s]
            idx, slot = out.get(l, s)
            np.testing.assert_array_equal(idx.cpu().numpy(), exp)
            np.testing.assert_array_equal(slot.cpu().numpy(), S.slots(tables[s].numpy(), exp, bs))


def test_ragged_long_segments_split_over_a_cluster(select_cluster):
    """Segments of very different lengths in one call: the long ones set a
    cluster size of 4, the short ones leave some CTAs with empty slices."""
    bs = 16
    lens = [8000, 0, 17, 3000, 5, 1100]
    ks = [1200, 3, 17, 2999, 0, 1100]
    T = sum(lens)
    g = torch.Generator().manual_seed(5)
    sc = torch.randint(0, 50, (3, T), generator=g).float()  # many ties
    sc[2, 100:200] = float("nan")
    pos0 = [0, 0, 16, 32, 3, 7]
    tables = [torch.randint(1, 1000, ((p + n + bs - 1) // bs + 1,), generator=g).int() for p, n in zip(pos0, lens)]
    blk_off = np.concatenate([[0], np.cumsum([len(t) for t in tables])[:-1]])
    bt = torch.cat(tables)
    col = np.concatenate([[0], np.cumsum(lens)[:-1]])
    kw = dict(seg_len=lens, seg_pos0=pos0, seg_blk_off=blk_off)
    for sel in (dict(k=ks), dict(threshold=25.0)):
        out = score_select(sc.cuda(), bt.cuda(), bs, **kw, **sel)
        for l in range(3):
            for s in range(len(lens)):
                row = sc[l, col[s]:col[s] + lens[s]].numpy()
                exp = (S.topk_positions(row, ks[s]) if "k" in sel else S.threshold_positions(row, 25.0)) + pos0[s]
                idx, slot = out.get(l, s)
                np.testing.assert_array_equal(idx.cpu().numpy(), exp)
                np.testing.assert_array_equal(slot.cpu().numpy(), S.slots(tables[s].numpy(), exp, bs))
    assert _lib.device_errors(0) == 0


def test_ptrs_to_slots_matches_oracle_and_policy():
    bs = 16
    bt = torch.randperm(2000)[:600].int() + 1
    ranges = [[512, 528], [1024, 1049], [1536, 1570], [2026, 2111], [5, 5]]
    idx, slot = ptrs_to_slots(ranges, bt.cuda(), bs)
    exp = S.ranges_to_positions(ranges)
    np.testing.assert_array_equal(idx.cpu().numpy(), exp)
    np.testing.assert_array_equal(slot.cpu().numpy(), S.slots(bt.numpy(), exp, bs))
    # Adapter.recompute_slots: policy ranges beyond adjusted_group_ptr[1]
    topo = CacheTopo.single_group(["l"], bs, 1, False)
    ad = Adapter(AdaptionConfig(recompute_avg_num=32, r=0.5), cache_topo=topo)
    ad.kvcaches = {"l": torch.zeros(1, device="cuda")}
    gp = list(range(0, 8193, 512)) + [8256]
    i2, s2 = ad.recompute_slots(gp, bt.tolist(), bs, no_recompute_length=512)
    rr = [r for r in ad.get_recompute_length(gp) if r[1] > 512]
    e2 = S.ranges_to_positions(rr)
    np.testing.assert_array_equal(i2.cpu().numpy(), e2)
    np.testing.assert_array_equal(s2.cpu().numpy(), S.slots(bt.numpy(), e2, bs))


def test_batched_memcpy_roundtrip():
    from daric_b200.cache_ops import batched_memcpy_d2h, batched_memcpy_h2d
    host = torch.randint(0, 255, (1 << 20,), dtype=torch.uint8).pin_memory()
    stg = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    batched_memcpy_h2d(host, stg, [0, 5000, 70000], [100, 9000, 500000], [4000, 60000, 1000])
    back = torch.zeros_like(host).pin_memory()
    batched_memcpy_d2h(stg, back, [100, 9000, 500000], [0, 5000, 70000], [4000, 60000, 1000])
    torch.cuda.synchronize()
    for a, b, n in [(0, 100, 4000), (5000, 9000, 60000), (70000, 500000, 1000)]:
        assert torch.equal(stg[b:b + n].cpu(), host[a:a + n])
        assert torch.equal(back[a:a + n], host[a:a + n])
