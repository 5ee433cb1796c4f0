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
