"""GPU parity of the page kernels against the CPU oracle (bit-exact):
scatter_pages / gather_pages (reference kernels.cu) and the fused
rerotate_scatter_pages (scatter + adapter.py re-rotation)."""
import numpy as np
import pytest
import torch

from daric_b200 import _lib
from daric_b200.cache_ops import CacheCopier
from daric_b200.reuse import build_chunk_plan, build_load_plan, layer_block_bytes
from daric_b200.topo import CacheTopo
from gpu_util import (layout_shape, oracle_layer, random_values, table_tensor, unique_blocks, bytes_np,
                      RAW_NP)
from oracle import pages as P
from oracle import rerotate as R

pytestmark = pytest.mark.gpu


def _setup(layout, dt, nb=24, bs=16, H=2, D=128, nlayers=2, seed=0):
    g = torch.Generator().manual_seed(seed)
    shape, pf = layout_shape(layout, nb, bs, H, D)
    names = [f"model.layers.{i}.self_attn.attn" for i in range(nlayers)]
    layers = {n: random_values(shape, dt, g) for n in names}
    topo = CacheTopo.single_group(names, bs, layer_block_bytes(layers[names[0]], pf), pf)
    return g, layers, topo, pf


# page-kernel variants: the bulk-copy pipeline as planned (bf16 tables:
# factors stored as bf16, staged with the pages; small pages: 4 CTAs per
# SM), with fp32 factors, with factors
# read from L2 in 3-page units (ragged last units), with 1 and 2 CTAs per SM,
# with 4 consumer-warp groups, with one factor buffer, with 16 consumer
# warps, with consumer stores (as planned, and in 3-page units at one CTA
# per SM), and the SIMT vector kernel
_VARIANTS = {
    "bulk": {},
    "bulk-f32": {"DARIC_BULK_FACTOR_FORMAT": "f32"},
    "bulk-l2-u3": {"DARIC_BULK_FACTORS": "l2", "DARIC_BULK_UNIT_PAGES": "3"},
    "bulk-1cta": {"DARIC_BULK_CTAS": "1"},
    "bulk-2cta": {"DARIC_BULK_CTAS": "2"},
    "bulk-4groups": {"DARIC_BULK_CGROUPS": "4"},
    "bulk-1facbuf": {"DARIC_BULK_FACTOR_BUFFERS": "1"},
    "bulk-16warps": {"DARIC_BULK_CWARPS": "16"},
    "bulk-cstore": {"DARIC_BULK_CSTORE": "1"},
    "bulk-cstore-1cta-u3": {"DARIC_BULK_CSTORE": "1", "DARIC_BULK_CTAS": "1", "DARIC_BULK_UNIT_PAGES": "3"},
    "simt": {"DARIC_PAGE_KERNEL": "simt"},
}


@pytest.fixture(params=list(_VARIANTS))
def page_kernel(request, monkeypatch):
    """Runs a test with each page-kernel implementation."""
    for k in ("DARIC_PAGE_KERNEL", "DARIC_BULK_FACTOR_FORMAT", "DARIC_BULK_FACTORS", "DARIC_BULK_UNIT_PAGES",
              "DARIC_BULK_CTAS", "DARIC_BULK_CGROUPS", "DARIC_BULK_FACTOR_BUFFERS", "DARIC_BULK_CWARPS",
              "DARIC_BULK_CSTORE"):
        monkeypatch.delenv(k, raising=False)
    for k, v in _VARIANTS[request.param].items():
        monkeypatch.setenv(k, v)
    return request.param


@pytest.mark.parametrize("layout", ["5d", "5dpf", "4d", "3d"])
@pytest.mark.parametrize("direction", ["scatter", "gather"])
def test_plain_copy_matches_oracle(layout, direction, page_kernel):
    g, layers, topo, pf = _setup(layout, "bf16")
    rng = np.random.default_rng(1)
    blocks = unique_blocks(rng, 24, [3, 5, 2], with_null=True)
    copier = CacheCopier()
    for n, t in layers.items():
        copier.register_layer(n, t, pf)
    bpb = {n: layer_block_bytes(t, pf) for n, t in layers.items()}
    plan = build_load_plan(topo, bpb, [(b,) for b in blocks], "cuda", base_offset=64)
    store = torch.randint(0, 255, (plan.total_bytes + 128,), dtype=torch.uint8, generator=g).cuda()
    copier.register_store(store)
    ol = {n: oracle_layer(t, "bf16", pf)[0] for n, t in layers.items()}
    st = bytes_np(store)
    idx = plan.indices_flat.cpu().numpy()
    args = (plan.layer_names, plan.offsets.tolist(), plan.byte_sizes.tolist(), plan.indices_flat,
            plan.indices_offsets.tolist())
    if direction == "scatter":
        copier.scatter_pages(*args)
        P.scatter_pages(ol, st, plan.layer_names, plan.offsets, plan.byte_sizes, idx, plan.indices_offsets)
        torch.cuda.synchronize()
        for n, t in layers.items():
            np.testing.assert_array_equal(bytes_np(t), ol[n].mem)
    else:
        copier.gather_pages(*args)
        P.gather_pages(ol, st, plan.layer_names, plan.offsets, plan.byte_sizes, idx, plan.indices_offsets)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(bytes_np(store), st)
    assert _lib.device_errors(0) == 0


def test_plain_copy_unaligned_byte_path():
    # 3-D layer with 30-byte pages: not 16-byte aligned -> byte-granular kernel
    g = torch.Generator().manual_seed(3)
    t = random_values((9, 3, 5), "bf16", g, outliers=False)
    copier = CacheCopier()
    copier.register_layer("l", t, True)
    suffix = 3 * 5 * 2
    store = torch.randint(0, 255, (7 + 4 * suffix,), dtype=torch.uint8, generator=g).cuda()
    copier.register_store(store)
    ids = torch.tensor([4, 0, 8, 2], dtype=torch.int32, device="cuda")
    ol = {"l": oracle_layer(t, "bf16", True)[0]}
    st = bytes_np(store)
    copier.scatter_pages(["l"], [7], [4 * suffix], ids, [0, 4])
    P.scatter_pages(ol, st, ["l"], [7], [4 * suffix], ids.cpu().numpy(), [0, 4])
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bytes_np(t), ol["l"].mem)


def test_copy_argument_errors_match_reference():
    g, layers, topo, pf = _setup("5d", "bf16", nb=8)
    copier = CacheCopier()
    n = next(iter(layers))
    copier.register_layer(n, layers[n], pf)
    ids = torch.tensor([1, 2], dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError, match="store buffer not registered"):
        copier.scatter_pages([n], [0], [0], ids, [0, 2])
    store = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    copier.register_store(store)
    with pytest.raises(RuntimeError, match="byte_size mismatch at job 0"):
        copier.scatter_pages([n], [0], [123], ids, [0, 2])
    with pytest.raises(RuntimeError, match="layer not registered"):
        copier.scatter_pages(["nope"], [0], [0], ids, [0, 2])
    with pytest.raises(RuntimeError, match="indices_flat must be int32"):
        copier.scatter_pages([n], [0], [0], ids.long(), [0, 2])
    with pytest.raises(RuntimeError, match="store range out of bounds"):
        copier.scatter_pages([n], [(1 << 20) - 10], [2 * 2 * 16 * 2 * 128 * 2], ids, [0, 2])
    with pytest.raises(RuntimeError, match="indices_offsets size"):
        copier.scatter_pages([n], [0], [0], ids, [0])


def test_out_of_range_block_is_skipped_and_flagged():
    g, layers, topo, pf = _setup("5d", "bf16", nb=8, nlayers=1)
    n, t = next(iter(layers.items()))
    before = bytes_np(t)
    copier = CacheCopier()
    copier.register_layer(n, t, pf)
    page = 2 * 16 * 2 * 128 * 2
    store = torch.zeros(2 * page, dtype=torch.uint8, device="cuda")
    copier.register_store(store)
    ids = torch.tensor([99], dtype=torch.int32, device="cuda")  # >= num_pages
    _lib.device_errors(0)
    copier.scatter_pages([n], [0], [page], ids, [0, 1])
    assert _lib.device_errors(0) & 1
    np.testing.assert_array_equal(bytes_np(t), before)


# ------------------------------------------------------------------ fused --
def _fused_case(layout, dt, tab_dt, neox, rot_dim, mode, H=2, D=128, bs=16, seed=0, scores=True, api="jobs"):
    """api: "jobs" (rerotate_scatter_pages on the reference's per-job plan),
    "chunks" (load_chunks, one descriptor per chunk) or "chunks-layerwise"
    (load_chunks one layer range at a time)."""
    g, layers, topo, pf = _setup(layout, dt, nb=40, bs=bs, H=H, D=D, seed=seed)
    rng = np.random.default_rng(seed)
    lens = [32, 40, 16, 48, 5]          # partial pages in chunks 1 and 4
    counts = [(n + bs - 1) // bs for n in lens]
    blocks = unique_blocks(rng, 40, counts, with_null=True)
    max_pos = 600
    table, table_raw = table_tensor(max_pos, rot_dim, 5e5, tab_dt)
    copier = CacheCopier()
    for n, t in layers.items():
        copier.register_layer(n, t, pf)
        copier.register_rotary(n, table, rot_dim, neox)
    bpb = {n: layer_block_bytes(t, pf) for n, t in layers.items()}
    plan = build_load_plan(topo, bpb, [(b,) for b in blocks], "cuda", base_offset=32)
    nelem = (plan.total_bytes + 64) // torch.empty(0, dtype=layers[plan.layer_names[0]].dtype).element_size()
    store = random_values((nelem,), dt, g, outliers=False).view(torch.uint8).reshape(-1)
    copier.register_store(store)
    if mode == "flexible":
        pos_a = [0, 7, 300, 100, 550]      # saved positions
        pos_b = [50, 7, 10, 400, 500]      # new positions (chunk 1: old == new -> copy)
    else:
        pos_a = [16, 0, 300, 99, 583]      # deltas
        pos_b = None
    # oracle
    ol = {n: oracle_layer(t, dt, pf) for n, t in layers.items()}
    st = bytes_np(store)
    idx = plan.indices_flat.cpu().numpy()
    P.scatter_pages({n: v[0] for n, v in ol.items()}, st, plan.layer_names, plan.offsets, plan.byte_sizes, idx,
                    plan.indices_offsets)
    rot = R.Rotary(table_raw.reshape(max_pos, rot_dim), tab_dt, rot_dim, neox)
    T = sum(lens)
    col = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    exp_scores = np.zeros((len(layers), T), np.float32)
    for j, (name, m) in enumerate(zip(plan.layer_names, plan.job_meta)):
        li = int(plan.job_layer[j])
        n_tok = lens[m]
        if mode == "flexible" and pos_a[m] == pos_b[m]:
            continue
        ids = np.asarray(blocks[m], np.int64)
        t = np.arange(n_tok)
        keep = ids[t // bs] != 0
        t = t[keep]
        gidx = ids[t // bs] * bs + t % bs
        if mode == "flexible":
            c, s = R.flexible_factors(rot, pos_a[m] + t, pos_b[m] + t)
        else:
            c, s = R.delta_factors(rot, np.full(len(t), pos_a[m]))
        dev = R.rotate_tokens(ol[name][1], rot, gidx, c, s)
        exp_scores[li, col[m] + t] = dev
    sc = torch.full((len(layers), T), -1.0, device="cuda") if scores else None
    if api == "jobs":
        kw = dict(scores=sc, job_score_row=plan.job_layer, meta_score_col=col) if scores else {}
        copier.rerotate_scatter_pages(plan.layer_names, plan.offsets, plan.byte_sizes, plan.indices_flat,
                                      plan.indices_offsets, plan.job_meta, mode, pos_a, pos_b, lens, **kw)
    else:
        cp = build_chunk_plan(topo, bpb, [(b,) for b in blocks], "cuda", base_offset=32)
        L = len(cp.layer_names)
        ranges = [(0, L)] if api == "chunks" else [(j, j + 1) for j in range(L)]
        for rg in ranges:
            copier.load_chunks(cp.c_names, cp.chunk_offsets, cp.chunk_blk_off, cp.chunk_pages, cp.block_ids, mode,
                               pos_a, pos_b, lens, scores=sc, score_col=col if scores else None, layer_range=rg)
    torch.cuda.synchronize()
    assert _lib.device_errors(0) == 0
    for n, t in layers.items():
        got = bytes_np(t).view(RAW_NP[dt])
        exp = ol[n][0].mem.view(RAW_NP[dt])
        bad = np.nonzero(got != exp)[0]
        assert bad.size == 0, f"{bad.size} elements differ, first {bad[:5]}: {got[bad[:5]]} vs {exp[bad[:5]]}"
    if scores:
        np.testing.assert_allclose(sc.cpu().numpy(), exp_scores, rtol=1e-3, atol=1e-6)


@pytest.mark.parametrize("mode", ["flexible", "delta"])
@pytest.mark.parametrize("layout", ["5d", "5dpf", "4d", "3d"])
def test_fused_bf16_neox_layouts(layout, mode, page_kernel):
    _fused_case(layout, "bf16", "bf16", True, 128, mode)


@pytest.mark.parametrize("dt,tab", [("f16", "f16"), ("f32", "f32"), ("fp8", "bf16"), ("bf16", "f32")])
@pytest.mark.parametrize("mode", ["flexible", "delta"])
def test_fused_dtypes(dt, tab, mode, page_kernel):
    _fused_case("5d", dt, tab, True, 128, mode)


@pytest.mark.parametrize("neox,rot_dim", [(False, 128), (True, 64), (False, 64)])
def test_fused_gptj_and_partial_rotary(neox, rot_dim, page_kernel):
    _fused_case("5d", "bf16", "bf16", neox, rot_dim, "flexible", seed=3)
    _fused_case("4d", "bf16", "bf16", neox, rot_dim, "delta", seed=4)


@pytest.mark.parametrize("H,D,bs", [(8, 128, 16), (4, 128, 32), (1, 64, 16), (8, 256, 8), (8, 128, 64)])
def test_fused_head_shapes(H, D, bs, page_kernel):
    _fused_case("5d", "bf16", "bf16", True, D, "flexible", H=H, D=D, bs=bs, seed=H + D)


def test_fused_without_scores():
    _fused_case("5d", "bf16", "bf16", True, 128, "flexible", scores=False)


@pytest.mark.parametrize("api", ["chunks", "chunks-layerwise"])
@pytest.mark.parametrize("mode", ["flexible", "delta"])
@pytest.mark.parametrize("layout", ["5d", "5dpf", "4d", "3d"])
def test_chunk_level_load_matches_oracle(layout, mode, api, page_kernel):
    _fused_case(layout, "bf16", "bf16", True, 128, mode, api=api)


@pytest.mark.parametrize("dt,tab", [("f16", "f16"), ("fp8", "bf16"), ("bf16", "f32")])
def test_chunk_level_load_dtypes(dt, tab):
    _fused_case("5d", dt, tab, True, 128, "flexible", api="chunks")
    _fused_case("5d", dt, tab, False, 64, "delta", api="chunks-layerwise", seed=2)


@pytest.mark.parametrize("H,D,bs", [(8, 128, 16), (1, 64, 16), (4, 128, 32)])
def test_chunk_level_load_head_shapes(H, D, bs):
    _fused_case("5d", "bf16", "bf16", True, D, "flexible", H=H, D=D, bs=bs, seed=H + D, api="chunks")


def test_chunk_level_plain_scatter_matches_scatter_pages():
    g, layers, topo, pf = _setup("5d", "bf16", nb=40, nlayers=3)
    rng = np.random.default_rng(1)
    blocks = unique_blocks(rng, 40, [3, 5, 2], with_null=True)
    bpb = {n: layer_block_bytes(t, pf) for n, t in layers.items()}
    plan = build_load_plan(topo, bpb, [(b,) for b in blocks], "cuda", base_offset=16)
    cp = build_chunk_plan(topo, bpb, [(b,) for b in blocks], "cuda", base_offset=16)
    store = random_values(((plan.total_bytes + 64) // 2,), "bf16", g, outliers=False).view(torch.uint8).reshape(-1)
    a = {n: t.clone() for n, t in layers.items()}
    ca, cb = CacheCopier(), CacheCopier()
    for n in layers:
        ca.register_layer(n, a[n], pf)
        cb.register_layer(n, layers[n], pf)
    ca.register_store(store)
    cb.register_store(store)
    ca.scatter_pages(plan.layer_names, plan.offsets, plan.byte_sizes, plan.indices_flat, plan.indices_offsets)
    cb.load_chunks(cp.c_names, cp.chunk_offsets, cp.chunk_blk_off, cp.chunk_pages, cp.block_ids, "none")
    torch.cuda.synchronize()
    for n in layers:
        assert torch.equal(a[n].view(torch.int16), layers[n].view(torch.int16)), n


def test_chunk_level_load_argument_errors():
    g, layers, topo, pf = _setup("5d", "bf16", nb=8, nlayers=2)
    copier = CacheCopier()
    for n, t in layers.items():
        copier.register_layer(n, t, pf)
    bpb = {n: layer_block_bytes(t, pf) for n, t in layers.items()}
    cp = build_chunk_plan(topo, bpb, [([1, 2],)], "cuda")
    copier.register_store(torch.zeros(cp.total_bytes - 16, dtype=torch.uint8, device="cuda"))
    with pytest.raises(_lib.DaricError, match="store range out of bounds"):
        copier.load_chunks(cp.c_names, cp.chunk_offsets, cp.chunk_blk_off, cp.chunk_pages, cp.block_ids, "none")
    copier.register_store(torch.zeros(cp.total_bytes, dtype=torch.uint8, device="cuda"))
    with pytest.raises(_lib.DaricError, match="reaches past block_ids"):
        copier.load_chunks(cp.c_names, cp.chunk_offsets, [1], cp.chunk_pages, cp.block_ids, "none")
    with pytest.raises(_lib.DaricError, match="register_rotary"):
        copier.load_chunks(cp.c_names, cp.chunk_offsets, cp.chunk_blk_off, cp.chunk_pages, cp.block_ids,
                           "flexible", [0], [5], [32])
    with pytest.raises(_lib.DaricError, match="layer range"):
        copier.load_chunks(cp.c_names, cp.chunk_offsets, cp.chunk_blk_off, cp.chunk_pages, cp.block_ids, "none",
                           layer_range=(1, 3))


@pytest.mark.parametrize("step,gap", [(1, 0), (2, 4096), (5, 0)])
def test_layerwise_load_from_host_matches_whole_load(step, gap):
    """load_layerwise (host -> staging per layer step on a copy stream,
    overlapped with the fused kernel of the previous step) writes the same
    paged KV and scores as one whole load of a staged chunk plan."""
    from daric_b200.reuse import ReusedKVLoader
    g, layers, topo, pf = _setup("5d", "bf16", nb=48, nlayers=5, seed=7)
    rng = np.random.default_rng(7)
    lens = [32, 40, 16, 48]
    blocks = unique_blocks(rng, 48, [(n + 15) // 16 for n in lens])
    table, _ = table_tensor(700, 128, 5e5, "bf16")
    bpb = {n: layer_block_bytes(t, pf) for n, t in layers.items()}
    chunks = [(b,) for b in blocks]
    total = sum(len(b) for b in blocks) * sum(bpb.values())
    host = random_values((total // 2,), "bf16", g, outliers=False).view(torch.uint8).reshape(-1).cpu().pin_memory()
    staging = torch.zeros(total, dtype=torch.uint8, device="cuda")
    kv_a = {n: t.clone() for n, t in layers.items()}
    rot = {n: (table, 128, True) for n in layers}
    la = ReusedKVLoader(kv_a, topo, staging, rot)
    lb = ReusedKVLoader(layers, topo, staging, rot)
    pos = dict(mode="flexible", pos_a=[0, 300, 17, 600], pos_b=[40, 72, 112, 128], chunk_len=lens)
    col = np.concatenate([[0], np.cumsum(lens)[:-1]]).tolist()
    sa = torch.full((5, sum(lens)), -1.0, device="cuda")
    sb = sa.clone()
    cp = la.plan_chunks(chunks)
    staging.copy_(host)
    la.load_chunks(cp, scores=sa, score_col=col, **pos)
    torch.cuda.synchronize()
    staging.zero_()
    # the store keeps its chunks elsewhere in its shared memory: each chunk
    # `gap` bytes further than the one before (host_offsets)
    host_off = cp.chunk_offsets + gap * (1 + np.arange(len(chunks)))
    shm = torch.zeros(total + gap * (len(chunks) + 1), dtype=torch.uint8).pin_memory()
    for m in range(len(chunks)):
        o, n = int(cp.chunk_offsets[m]), int(cp.chunk_sizes[m])
        shm[int(host_off[m]):int(host_off[m]) + n] = host[o:o + n]
    lw = lb.load_layerwise(lb.plan_chunks(chunks), shm, host_offsets=host_off, layers_per_step=step, scores=sb,
                           score_col=col, **pos)
    for j in range(5):
        lw.wait_layer(j)
    torch.cuda.synchronize()
    assert _lib.device_errors(0) == 0
    for n in layers:
        assert torch.equal(kv_a[n].view(torch.int16), layers[n].view(torch.int16)), n
    assert torch.equal(sa, sb)
    with pytest.raises(IndexError):
        lw.wait_layer(5)


def test_fused_load_sees_a_table_written_just_before_registration():
    """The factor pre-pass runs on a side stream; after a rotary table is
    (re)registered it first waits for the caller's stream, so a table that
    is still being written there (queued behind a long kernel) is read only
    once written."""
    g, layers, topo, pf = _setup("5d", "bf16", nb=24, nlayers=2, seed=5)
    rng = np.random.default_rng(5)
    blocks = unique_blocks(rng, 24, [2, 3])
    lens = [32, 48]
    copier = CacheCopier()
    t1, raw1 = table_tensor(600, 128, 5e5, "bf16")
    _, raw2 = table_tensor(600, 128, 1e4, "bf16")
    for n, t in layers.items():
        copier.register_layer(n, t, pf)
        copier.register_rotary(n, t1, 128, True)
    bpb = {n: layer_block_bytes(t, pf) for n, t in layers.items()}
    plan = build_load_plan(topo, bpb, [(b,) for b in blocks], "cuda")
    store = random_values(((plan.total_bytes + 64) // 2,), "bf16", g, outliers=False).view(torch.uint8).reshape(-1)
    copier.register_store(store)
    args = (plan.layer_names, plan.offsets, plan.byte_sizes, plan.indices_flat, plan.indices_offsets, plan.job_meta,
            "flexible", [3, 100], [50, 7], lens)
    copier.rerotate_scatter_pages(*args)
    torch.cuda.synchronize()
    ol = {n: oracle_layer(t, "bf16", pf) for n, t in layers.items()}  # before the second load
    t2 = torch.zeros_like(t1)
    src = torch.from_numpy(raw2.view(np.int16)).view(torch.bfloat16).pin_memory()
    if hasattr(torch.cuda, "_sleep"):
        torch.cuda._sleep(20_000_000)  # ~10 ms of GPU time queued before the table is written
    t2.copy_(src, non_blocking=True)
    for n in layers:
        copier.register_rotary(n, t2, 128, True)
    copier.rerotate_scatter_pages(*args)
    P.scatter_pages({n: v[0] for n, v in ol.items()}, bytes_np(store), plan.layer_names, plan.offsets,
                    plan.byte_sizes, plan.indices_flat.cpu().numpy(), plan.indices_offsets)
    rot = R.Rotary(raw2.reshape(600, 128), "bf16", 128, True)
    for j, (name, m) in enumerate(zip(plan.layer_names, plan.job_meta)):
        t = np.arange(lens[m])
        c, s = R.flexible_factors(rot, [3, 100][m] + t, [50, 7][m] + t)
        R.rotate_tokens(ol[name][1], rot, R.gather_index(blocks[m], 16, 0, lens[m]), c, s)
    torch.cuda.synchronize()
    for n, t in layers.items():
        np.testing.assert_array_equal(bytes_np(t).view(np.uint16), ol[n][0].mem.view(np.uint16))


def test_pipeline_wait_time_out_reports_and_leaves_the_device_usable(monkeypatch):
    """With each CTA's first unit left unarmed (a barrier nothing completes,
    DARIC_TEST_UNARMED) and a 2 ms wait limit (DARIC_WAIT_NS), the pipelines'
    waits run out: the calls return, daric_device_errors reports bit 8, and
    the next calls produce the oracle's bytes (the kernels drain their copies
    in flight before returning; nothing faults)."""
    g, layers, topo, pf = _setup("5d", "bf16", nb=40, nlayers=2, seed=9)
    rng = np.random.default_rng(9)
    blocks = unique_blocks(rng, 40, [3, 4])
    table, _ = table_tensor(600, 128, 5e5, "bf16")
    copier = CacheCopier()
    for n, t in layers.items():
        copier.register_layer(n, t, pf)
        copier.register_rotary(n, table, 128, True)
    bpb = {n: layer_block_bytes(t, pf) for n, t in layers.items()}
    plan = build_load_plan(topo, bpb, [(b,) for b in blocks], "cuda")
    store = random_values(((plan.total_bytes + 64) // 2,), "bf16", g, outliers=False).view(torch.uint8).reshape(-1)
    copier.register_store(store)
    bt = torch.tensor(blocks[0] + blocks[1], dtype=torch.int32, device="cuda")
    assert _lib.device_errors(0) == 0
    monkeypatch.setenv("DARIC_WAIT_NS", "2000000")
    monkeypatch.setenv("DARIC_TEST_UNARMED", "1")
    copier.rerotate_scatter_pages(plan.layer_names, plan.offsets, plan.byte_sizes, plan.indices_flat,
                                  plan.indices_offsets, plan.job_meta, "flexible", [3, 100], [50, 7], [48, 64])
    assert _lib.device_errors(0) == 8
    copier.rerotate_inplace(list(layers), "delta", bt, [0, 3], [0, 0], [48, 64], [17, 29])
    assert _lib.device_errors(0) == 8
    monkeypatch.delenv("DARIC_WAIT_NS")
    monkeypatch.delenv("DARIC_TEST_UNARMED")
    _fused_case("5d", "bf16", "bf16", True, 128, "flexible", seed=9)
    _fused_case("5d", "bf16", "bf16", True, 128, "delta", seed=10, api="chunks")
