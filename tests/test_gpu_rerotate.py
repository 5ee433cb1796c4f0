"""GPU parity of the in-place re-rotation (Adapter drop-in) against the
reference kernel's golden outputs and the oracle drivers."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from daric_b200 import _lib
from daric_b200.adaption import Adapter, AdaptionConfig
from daric_b200.reuse import layer_block_bytes
from daric_b200.topo import CacheTopo
from golden_io import CASES, DT, load_case, metas_of
from gpu_util import RAW_NP, bytes_np, layout_shape, oracle_layer, random_values, table_tensor, unique_blocks
from oracle import rerotate as R

pytestmark = pytest.mark.gpu

_TORCH = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}

# in-place kernel variants: the copy-engine pipeline as planned (flexible
# mode reads a factor pre-pass), with the factors read from the table per
# task, pinned to 1 and 2 CTAs per SM, with 3-page units (ragged last units)
# and 4 consumer warps, and the SIMT kernel with its factor pre-pass
_INPLACE = {
    "bulk": {},
    "bulk-table": {"DARIC_INPLACE_FACTORS": "table"},
    "bulk-1cta": {"DARIC_INPLACE_CTAS": "1"},
    "bulk-2cta": {"DARIC_INPLACE_CTAS": "2"},
    "bulk-u3-4w": {"DARIC_INPLACE_UNIT_PAGES": "3", "DARIC_INPLACE_CWARPS": "4"},
    "simt": {"DARIC_PAGE_KERNEL": "simt"},
}


@pytest.fixture(params=list(_INPLACE), autouse=True)
def inplace_kernel(request, monkeypatch):
    """Runs every test of this module with each in-place kernel."""
    for k in ("DARIC_PAGE_KERNEL", "DARIC_INPLACE_CTAS", "DARIC_INPLACE_UNIT_PAGES", "DARIC_INPLACE_CWARPS",
              "DARIC_INPLACE_FACTORS"):
        monkeypatch.delenv(k, raising=False)
    for k, v in _INPLACE[request.param].items():
        monkeypatch.setenv(k, v)
    return request.param


def _from_raw(raw, shape, dt):
    t = torch.from_numpy(raw.view(np.int16) if raw.dtype == np.uint16 else raw).reshape(shape)
    return t.view(_TORCH[dt]).cuda() if dt in ("bf16", "f16") else t.cuda()


@pytest.mark.parametrize("case", CASES)
def test_adapter_matches_reference_golden(case):
    meta, arr = load_case(case)
    dt = DT[meta["dtype"]]
    shape = tuple(meta["shape"])
    kv = _from_raw(arr["kv_in"].reshape(-1), shape, dt)
    table = _from_raw(arr["table"].reshape(-1), (meta["max_pos"], meta["rotary_dim"]), dt)
    name = meta["layer"]
    topo = CacheTopo.single_group([name], shape[2] if len(shape) >= 4 else shape[1],
                                  layer_block_bytes(kv, meta["page_first"]), meta["page_first"])
    ad = Adapter(AdaptionConfig(recompute_avg_num=16), cache_topo=topo)
    ad.register_kvcaches({name: kv})
    ad.register_rotary_embed(name, SimpleNamespace(cos_sin_cache=table, rotary_dim=meta["rotary_dim"],
                                                   is_neox_style=meta["is_neox"]))
    if meta["mode"] == "flexible":
        ad.apply_rerotate_load(metas_of(meta))
    else:
        ad.apply_rerotate_multi(meta["group_ptrs"], [(b,) for b in meta["block_ids"]])
    torch.cuda.synchronize()
    got = bytes_np(kv).view(np.uint16)
    gold = arr["kv_out"].reshape(-1)
    # within 1 ulp of the reference kernel (its interpreter run truncates)
    assert R.ulp_diff(got, gold, dt).max() <= 1
    # bit-exact with the RTNE restatement
    layer = R.KLayer(arr["kv_in"].reshape(-1).copy(), shape, tuple(kv.stride()), meta["page_first"], dt)
    rot = R.Rotary(arr["table"].reshape(meta["max_pos"], meta["rotary_dim"]), dt, meta["rotary_dim"],
                   meta["is_neox"])
    if meta["mode"] == "flexible":
        R.apply_rerotate_load({name: layer}, {name: rot}, {name: 0}, metas_of(meta))
    else:
        R.apply_rerotate_multi({name: layer}, {name: rot}, {name: 0}, meta["group_ptrs"],
                               [(b,) for b in meta["block_ids"]])
    np.testing.assert_array_equal(got, layer.raw)
    assert _lib.device_errors(0) == 0


def _multi_layer(layout, dt, seed, nl=3, nb=48, bs=16, H=4, D=128):
    g = torch.Generator().manual_seed(seed)
    shape, pf = layout_shape(layout, nb, bs, H, D)
    names = [f"model.layers.{i}.self_attn.attn" for i in range(nl)]
    kvs = {n: random_values(shape, dt, g) for n in names}
    topo = CacheTopo.single_group(names, bs, layer_block_bytes(kvs[names[0]], pf), pf)
    return kvs, topo, pf


@pytest.mark.parametrize("layout,dt", [("5d", "bf16"), ("5dpf", "f16"), ("4d", "bf16"), ("5d", "fp8")])
def test_adapter_flexible_multi_layer(layout, dt):
    kvs, topo, pf = _multi_layer(layout, dt, seed=5)
    rng = np.random.default_rng(5)
    lens = [64, 40, 16, 100]
    blocks = unique_blocks(rng, 48, [(n + 15) // 16 for n in lens])
    starts = [0, 64, 112, 128]
    metas = [SimpleNamespace(ptr=[s, s + n], saved_pos=sp, block_ids=(b,))
             for s, n, sp, b in zip(starts, lens, [900, 64, 5, 0], blocks)]
    table, raw = table_tensor(1200, 128, 1e6, "bf16")
    ad = Adapter(AdaptionConfig(), cache_topo=topo)
    ad.register_kvcaches(kvs)
    rot = R.Rotary(raw.reshape(1200, 128), "bf16", 128, True)
    ol = {}
    for n, t in kvs.items():
        ad.register_rotary_embed(n, SimpleNamespace(cos_sin_cache=table, rotary_dim=128, is_neox_style=True))
        ol[n] = oracle_layer(t, dt, pf)[1]
    ad.apply_rerotate_load(metas)
    R.apply_rerotate_load(ol, {n: rot for n in kvs}, {n: 0 for n in kvs}, metas)
    torch.cuda.synchronize()
    for n, t in kvs.items():
        np.testing.assert_array_equal(bytes_np(t).view(RAW_NP[dt]), ol[n].raw)
    # layer-wise call touches one layer only
    n0 = next(iter(kvs))
    before = {n: bytes_np(t) for n, t in kvs.items()}
    ad.apply_rerotate_load(metas, layer_name=n0)
    torch.cuda.synchronize()
    for n, t in kvs.items():
        assert (bytes_np(t) != before[n]).any() == (n == n0)


def test_adapter_strict_multi_request():
    kvs, topo, pf = _multi_layer("5d", "bf16", seed=9)
    table, raw = table_tensor(4096, 128, 5e5, "bf16")
    ad = Adapter(AdaptionConfig(), cache_topo=topo)
    ad.register_kvcaches(kvs)
    ol = {n: oracle_layer(t, "bf16", pf)[1] for n, t in kvs.items()}
    for n in kvs:
        ad.register_rotary_embed(n, SimpleNamespace(cos_sin_cache=table, rotary_dim=128, is_neox_style=True))
    rng = np.random.default_rng(2)
    # two requests, 4 and 5 groups, disjoint blocks
    gp = [[0, 40, 100, 160, 170], [0, 16, 48, 64, 200, 203]]
    b = unique_blocks(rng, 48, [11, 13])
    ad.apply_rerotate_multi(gp, [(b[0],), (b[1],)])
    rot = R.Rotary(raw.reshape(4096, 128), "bf16", 128, True)
    R.apply_rerotate_multi(ol, {n: rot for n in kvs}, {n: 0 for n in kvs}, gp, [(b[0],), (b[1],)])
    torch.cuda.synchronize()
    for n, t in kvs.items():
        np.testing.assert_array_equal(bytes_np(t).view(np.uint16), ol[n].raw)


def test_adapter_rereads_replaced_table():
    kvs, topo, pf = _multi_layer("5d", "bf16", seed=11, nl=1)
    n, t = next(iter(kvs.items()))
    ad = Adapter(AdaptionConfig(), cache_topo=topo)
    ad.register_kvcaches(kvs)
    rot_mod = SimpleNamespace(cos_sin_cache=table_tensor(512, 128, 5e5, "f32")[0], rotary_dim=128,
                              is_neox_style=True)
    ad.register_rotary_embed(n, rot_mod)
    metas = [SimpleNamespace(ptr=[0, 16], saved_pos=3, block_ids=([2],))]
    ad.apply_rerotate_load(metas)
    # the module swaps in a bf16 copy (as vLLM does on first forward)
    tb, raw = table_tensor(512, 128, 5e5, "bf16")
    rot_mod.cos_sin_cache = tb
    ol = oracle_layer(t, "bf16", pf)[1]
    ad.apply_rerotate_load(metas)
    R.apply_rerotate_load({n: ol}, {n: R.Rotary(raw.reshape(512, 128), "bf16", 128, True)}, {n: 0}, metas)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bytes_np(t).view(np.uint16), ol.raw)


def _inplace_case(layout, dt, tab_dt, neox, rot_dim, mode, H=2, D=128, bs=16, seed=0):
    """Segments of three requests (tokens of one request meet inside pages,
    a segment inside one page, a block id 0) rotated in place over 3 layers
    through CacheCopier.rerotate_inplace, against the oracle's rotation."""
    from daric_b200.cache_ops import CacheCopier
    g = torch.Generator().manual_seed(seed)
    nb = 40
    shape, pf = layout_shape(layout, nb, bs, H, D)
    names = [f"model.layers.{i}.self_attn.attn" for i in range(3)]
    kvs = {n: random_values(shape, dt, g) for n in names}
    max_pos = 700
    table, raw = table_tensor(max_pos, rot_dim, 5e5, tab_dt)
    rng = np.random.default_rng(seed)
    # request tables (positions -> blocks); request 2 uses block 0 once
    lens_req = [80, 51, 32]  # tokens (segments below are given in tokens)
    tables = unique_blocks(rng, nb, [(n + bs - 1) // bs for n in lens_req])
    tables[2][-1] = 0
    flat = np.concatenate([np.asarray(t, np.int32) for t in tables])
    blk_off = np.concatenate([[0], np.cumsum([len(t) for t in tables])[:-1]]).astype(np.int64)
    #        (request, start, length, pos_a, pos_b)
    segs = [(0, 3, 21, 5, 300), (0, 24, 40, 600, 2), (0, 64, 16, 64, 64 + 7),
            (1, 0, 35, 17, 170), (1, 35, 2, 1, 100), (2, 5, 9, 400, 33), (2, 17, 14, 31, 90)]
    if mode == "delta":
        segs = [(r, st, n, a, 0) for r, st, n, a, _ in segs]
    copier = CacheCopier()
    for n, t in kvs.items():
        copier.register_layer(n, t, pf)
        copier.register_rotary(n, table, rot_dim, neox)
    ol = {n: oracle_layer(t, dt, pf)[1] for n, t in kvs.items()}
    bt = torch.from_numpy(flat).cuda()
    copier.rerotate_inplace(names, mode, bt, [int(blk_off[r]) for r, *_ in segs], [st for _, st, *_ in segs],
                            [n for _, _, n, _, _ in segs], [a for *_, a, _ in segs],
                            [b for *_, b in segs] if mode == "flexible" else None)
    rot = R.Rotary(raw.reshape(max_pos, rot_dim), tab_dt, rot_dim, neox)
    for r, st, n, a, b in segs:
        idx = R.gather_index(tables[r], bs, st, n)
        t = np.arange(n)
        c, s = R.flexible_factors(rot, a + t, b + t) if mode == "flexible" else R.delta_factors(rot, np.full(n, a))
        for name in names:
            R.rotate_tokens(ol[name], rot, idx, c, s)
    torch.cuda.synchronize()
    assert _lib.device_errors(0) == 0
    for n, t in kvs.items():
        got = bytes_np(t).view(RAW_NP[dt])
        bad = np.nonzero(got != ol[n].raw)[0]
        assert bad.size == 0, f"{n}: {bad.size} elements differ, first at {bad[:5]}"


@pytest.mark.parametrize("mode", ["delta", "flexible"])
@pytest.mark.parametrize("layout", ["5d", "5dpf", "4d", "3d"])
def test_inplace_layouts(layout, mode):
    _inplace_case(layout, "bf16", "bf16", True, 128, mode)


@pytest.mark.parametrize("dt,tab", [("f16", "f16"), ("f32", "f32"), ("fp8", "bf16"), ("bf16", "f32")])
@pytest.mark.parametrize("mode", ["delta", "flexible"])
def test_inplace_dtypes(dt, tab, mode):
    _inplace_case("5d", dt, tab, True, 128, mode, seed=1)


@pytest.mark.parametrize("neox,rot_dim", [(False, 128), (True, 64), (False, 64)])
def test_inplace_gptj_and_partial_rotary(neox, rot_dim):
    _inplace_case("5d", "bf16", "bf16", neox, rot_dim, "flexible", seed=3)
    _inplace_case("4d", "bf16", "bf16", neox, rot_dim, "delta", seed=4)


@pytest.mark.parametrize("H,D,bs", [(8, 128, 16), (1, 64, 16), (8, 256, 8), (4, 128, 32)])
def test_inplace_head_shapes(H, D, bs):
    _inplace_case("5d", "bf16", "bf16", True, D, "delta", H=H, D=D, bs=bs, seed=H + D)
