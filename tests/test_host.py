"""Host-side logic on CPU: load-plan layout (store wire format), and the
torch-CPU baseline restatement against the numpy oracle."""
import numpy as np
import torch

from daric_b200.reuse import build_load_plan
from daric_b200.topo import CacheTopo, LayerCacheTopo
from oracle import numerics as N
from oracle import pages as P
from oracle import rerotate as R
from oracle.torch_cpu import reused_kv_step


def test_load_plan_matches_store_wire_format():
    # two KV groups; layers in sorted order; per chunk layer-major jobs
    layers = {"b.attn": LayerCacheTopo(0, 16, 1000, False), "a.attn": LayerCacheTopo(1, 16, 300, False),
              "c.attn": LayerCacheTopo(0, 16, 1000, False)}
    topo = CacheTopo(layers=layers, groups=[["b.attn", "c.attn"], ["a.attn"]])
    bpb = {"a.attn": 300, "b.attn": 1000, "c.attn": 1000}
    chunks = [([5, 6, 7], [9]), ([8], [10, 11])]
    plan = build_load_plan(topo, bpb, chunks, "cpu", base_offset=100)
    assert plan.layer_names == ["a.attn", "b.attn", "c.attn"] * 2
    # chunk 0: a (group 1, 1 block) 300 B, b 3000 B, c 3000 B
    assert plan.byte_sizes.tolist() == [300, 3000, 3000, 600, 1000, 1000]
    assert plan.offsets.tolist() == [100, 400, 3400, 6400, 7000, 8000]
    assert plan.indices_offsets.tolist() == [0, 1, 4, 7, 9, 10, 11]
    assert plan.indices_flat.tolist() == [9, 5, 6, 7, 5, 6, 7, 10, 11, 8, 8]
    assert plan.chunk_offsets.tolist() == [100, 6400] and plan.chunk_sizes.tolist() == [6300, 2600]
    assert plan.job_meta.tolist() == [0, 0, 0, 1, 1, 1]
    assert plan.job_layer.tolist() == [0, 1, 2, 0, 1, 2]


def test_torch_cpu_baseline_matches_oracle():
    g = torch.Generator().manual_seed(0)
    L, nb, bs, H, D = 2, 12, 16, 2, 128
    kv = [torch.zeros((2, nb, bs, H, D), dtype=torch.bfloat16) for _ in range(L)]
    lens, old, new = [32, 16], [5, 40], [100, 40]
    blocks = [torch.tensor([3, 7]), torch.tensor([0])]
    n_pages = [2, 1]
    total = sum(2 * p * bs * H * D * 2 * L for p in n_pages)
    stg = torch.randn(total // 2, generator=g).to(torch.bfloat16).view(torch.uint8)
    table_raw = R.rope_table(256, D, 5e5, "bf16")
    table = torch.from_numpy(table_raw.view(np.int16)).view(torch.bfloat16)
    sc = torch.rand(L, 48, generator=g)
    bt = torch.tensor([3, 7, 9], dtype=torch.int32)
    reused_kv_step(kv, stg, blocks, lens, old, new, table, sc, 5, bt, bs)
    # numpy oracle: scatter then rotate
    topo = CacheTopo.single_group([f"l{i}" for i in range(L)], bs, 2 * bs * H * D * 2, False)
    plan = build_load_plan(topo, {f"l{i}": 2 * bs * H * D * 2 for i in range(L)},
                           [(b.tolist(),) for b in blocks], "cpu")
    mems = {f"l{i}": np.zeros(2 * nb * bs * H * D * 2, np.uint8) for i in range(L)}
    shape, strides = (2, nb, bs, H, D), tuple(kv[0].stride())
    P.scatter_pages({n: P.LayerMem(m, shape, strides, 2, False) for n, m in mems.items()}, stg.numpy(),
                    plan.layer_names, plan.offsets, plan.byte_sizes, plan.indices_flat.numpy(),
                    plan.indices_offsets)
    rot = R.Rotary(table_raw, "bf16", D, True)
    t = np.arange(32)
    c, s = R.flexible_factors(rot, old[0] + t, new[0] + t)
    for n, m in mems.items():
        R.rotate_tokens(R.KLayer(m.view(np.uint16), shape, strides, False, "bf16"), rot,
                        R.gather_index([3, 7], bs, 0, 32), c, s)
    for i in range(L):
        got = kv[i].view(torch.int16).numpy().view(np.uint16).reshape(-1)
        np.testing.assert_array_equal(got, mems[f"l{i}"].view(np.uint16))


def test_chunk_plan_covers_the_load_plan_jobs():
    """The chunk plan (one descriptor per chunk) describes the same store
    bytes as the per-(chunk, layer) job plan of the reference's copy plan,
    and its layer ranges are contiguous slices of each chunk."""
    from daric_b200.reuse import build_chunk_plan
    names = [f"model.layers.{i}.attn" for i in range(11)]
    topo = CacheTopo.single_group(names, 16, 2048, False)
    bpb = {n: 2048 + 512 * (i % 3) for i, n in enumerate(sorted(names))}
    chunks = [([5, 6, 7],), ([8],), ([],), ([10, 11, 12, 13],)]
    lp = build_load_plan(topo, bpb, chunks, "cpu", base_offset=64)
    cp = build_chunk_plan(topo, bpb, chunks, "cpu", base_offset=64)
    L = len(names)
    assert cp.layer_names == lp.layer_names[:L]
    np.testing.assert_array_equal(cp.chunk_offsets, lp.chunk_offsets)
    np.testing.assert_array_equal(cp.chunk_sizes, lp.chunk_sizes)
    assert cp.block_ids.tolist() == [5, 6, 7, 8, 10, 11, 12, 13]
    for m in range(len(chunks)):
        for j in range(L):
            off, size = cp.layer_regions(j, j + 1)
            assert (off[m], size[m]) == (lp.offsets[m * L + j], lp.byte_sizes[m * L + j])
            ids = lp.indices_flat[lp.indices_offsets[m * L + j]:lp.indices_offsets[m * L + j + 1]].tolist()
            b0 = int(cp.chunk_blk_off[m])
            assert ids == cp.block_ids[b0:b0 + int(cp.chunk_pages[m])].tolist()
        off, size = cp.layer_regions(2, 7)
        assert off[m] == lp.offsets[m * L + 2] and size[m] == sum(lp.byte_sizes[m * L + 2:m * L + 7])
