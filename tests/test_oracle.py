"""Self-checks of the CPU oracle against torch's own CPU arithmetic."""
import numpy as np
import pytest
import torch

from oracle import numerics as N
from oracle import pages as P
from oracle import rerotate as R
from oracle import select as S


def _bits(t):
    return t.view(torch.int16).numpy().view(np.uint16)


def test_bf16_rounding_matches_torch():
    x = torch.randn(200000, dtype=torch.float32) * torch.logspace(-30, 30, 200000)
    np.testing.assert_array_equal(N.f32_to_bf16(x.numpy()), _bits(x.to(torch.bfloat16)))


def test_f16_rounding_matches_torch():
    x = torch.randn(100000, dtype=torch.float32) * 100
    np.testing.assert_array_equal(N.f32_to_f16(x.numpy()), _bits(x.to(torch.float16)))


def test_e4m3_rounding_matches_torch_in_range():
    x = (torch.randn(100000) * 50).clamp(-448, 448)
    ref = x.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(N.f32_to_e4m3(x.numpy()), ref)
    assert N.f32_to_e4m3(np.array([1000.0, -1e9], np.float32)).tolist() == [0x7E, 0xFE]


@pytest.mark.parametrize("dtype,name", [(torch.bfloat16, "bf16"), (torch.float16, "f16"), (torch.float32, "f32")])
def test_flexible_factors_match_torch_ops(dtype, name):
    table = torch.from_numpy(N.DTYPES["f32"][1](R.rope_table(5000, 128, 5e5, "f32"))).to(dtype)
    raw = _bits(table) if dtype != torch.float32 else table.numpy()
    rot = R.Rotary(raw, name, 128, True)
    old = torch.randint(0, 5000, (300,))
    new = torch.randint(0, 5000, (300,))
    oc, os_ = table.index_select(0, old).chunk(2, -1)
    nc, ns = table.index_select(0, new).chunk(2, -1)
    c_ref = (nc * oc + ns * os_).float().numpy()
    s_ref = (ns * oc - nc * os_).float().numpy()
    c, s = R.flexible_factors(rot, old.numpy(), new.numpy())
    np.testing.assert_array_equal(c, c_ref)
    np.testing.assert_array_equal(s, s_ref)


def test_rotation_matches_torch_fp32_math():
    g = torch.Generator().manual_seed(0)
    kv = torch.randn(2, 4, 16, 2, 128, generator=g).to(torch.bfloat16)
    table = torch.from_numpy(N.bf16_to_f32(R.rope_table(64, 128, 5e5))).to(torch.bfloat16)
    layer = R.KLayer(_bits(kv).reshape(-1).copy(), tuple(kv.shape), kv.stride(), False, "bf16")
    rot = R.Rotary(_bits(table), "bf16", 128, True)
    idx = np.array([16 + 3, 32 + 0, 48 + 15])
    pos = np.array([5, 9, 63])
    c, s = R.delta_factors(rot, pos)
    R.rotate_tokens(layer, rot, idx, c, s)
    k = kv[0].reshape(-1, 2, 128)[torch.from_numpy(idx)].float()
    cc, ss = torch.from_numpy(c)[:, None], torch.from_numpy(s)[:, None]
    o1 = k[..., :64] * cc - k[..., 64:] * ss
    o2 = k[..., 64:] * cc + k[..., :64] * ss
    ref = torch.cat([o1, o2], -1).to(torch.bfloat16)
    got = torch.from_numpy(layer.raw.view(np.int16)).view(torch.bfloat16).reshape(kv.shape)[0].reshape(-1, 2, 128)
    assert torch.equal(got[torch.from_numpy(idx)], ref)


def test_page_copy_shape_and_roundtrip():
    kv = np.arange(2 * 8 * 16 * 4 * 8, dtype=np.uint16)
    sizes, strides = (2, 8, 16, 4, 8), (8 * 16 * 32, 16 * 32, 32, 8, 1)
    L = P.LayerMem(kv.view(np.uint8), sizes, strides, 2, False)
    assert P.page_copy_shape(sizes, strides, 2, False) == (8, 2, 16 * 32 * 2, 16 * 32 * 2, 8 * 16 * 32 * 2)
    ids = np.array([3, 0, 5], np.int32)
    suffix = 16 * 32 * 2
    store = np.zeros(2 * 3 * suffix, np.uint8)
    P.gather_pages({"l": L}, store, ["l"], [0], [2 * 3 * suffix], ids, [0, 3])
    assert not store[suffix:2 * suffix].any()  # block 0 skipped
    L2 = P.LayerMem(np.zeros_like(L.mem), sizes, strides, 2, False)
    P.scatter_pages({"l": L2}, store, ["l"], [0], [2 * 3 * suffix], ids, [0, 3])
    v1 = L.mem.view(np.uint16).reshape(sizes)
    v2 = L2.mem.view(np.uint16).reshape(sizes)
    assert np.array_equal(v1[:, [3, 5]], v2[:, [3, 5]])
    assert not v2[:, [0, 1, 2, 4, 6, 7]].any()
    with pytest.raises(P.OracleError, match="byte_size mismatch"):
        P.scatter_pages({"l": L2}, store, ["l"], [0], [7], ids, [0, 3])
    with pytest.raises(P.OracleError, match="dense physical span"):
        P.page_copy_shape((2, 8, 16, 4, 8), (8 * 16 * 64, 16 * 64, 64, 8, 1), 2, False)


def test_topk_matches_torch_on_distinct_scores():
    x = torch.randn(5000).numpy()
    got = S.topk_positions(x, 700)
    ref = np.sort(torch.topk(torch.from_numpy(x), 700).indices.numpy())
    np.testing.assert_array_equal(got, ref)
    # ties go to the lower index; NaN ranks first
    y = np.array([1, 3, 3, 3, np.nan, 0], np.float32)
    assert S.topk_positions(y, 3).tolist() == [1, 2, 4]
    assert S.topk_positions(y, 0).tolist() == []
    assert S.threshold_positions(y, 3.0).tolist() == [1, 2, 3]


def test_rotate_dense_matches_rotate_tokens():
    """The dense-block form of the rotation (used by the full-size GPU
    checks) equals the per-token form on a paged layer, both styles."""
    from oracle.numerics import f32_to_bf16
    rng = np.random.default_rng(0)
    T, H, D = 40, 4, 128
    shape, strides = (2, 5, 8, H, D), (5 * 8 * H * D, 8 * H * D, H * D, D, 1)
    kv = f32_to_bf16((rng.standard_normal(shape) * 3).astype(np.float32)).reshape(-1)
    table = R.rope_table(600, 128, 5e5, "bf16").reshape(600, 128)
    for neox in (True, False):
        rot = R.Rotary(table, "bf16", 128, neox)
        layer = R.KLayer(kv.copy(), shape, strides, False, "bf16")
        t = np.arange(T)
        c, s = R.flexible_factors(rot, 3 + t, 300 + t)
        dev1 = R.rotate_tokens(layer, rot, np.arange(T), c, s)
        out, dev2 = R.rotate_dense(kv.reshape(shape)[0].reshape(T, H, D), rot, "bf16", c, s)
        np.testing.assert_array_equal(layer.raw.reshape(shape)[0].reshape(T, H, D), out)
        np.testing.assert_allclose(dev1, dev2, rtol=1e-6)
