"""Multi-rank host logic on CPU (gloo, world_size 2): data-parallel request
assignment, the tensor-parallel KV-head split, and the all-reduce of partial
deviation scores after which every rank makes the same selection."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from daric_b200.shard import allreduce_scores, assign_requests, tp_head_range
from oracle import numerics as N
from oracle import rerotate as R
from oracle import select as S


def test_assign_requests_is_balanced_and_complete():
    rng = np.random.default_rng(0)
    sizes = rng.integers(2048, 16384, size=512) * 8192
    for world in (1, 2, 4, 8):
        parts = assign_requests(sizes, world)
        assert sorted(i for p in parts for i in p) == list(range(512))
        loads = [sum(int(sizes[i]) for i in p) for p in parts]
        assert max(loads) - min(loads) <= int(sizes.max())


def test_tp_head_range():
    assert [tp_head_range(r, 4, 8) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        tp_head_range(0, 3, 8)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _partial_scores(rank, world, seed=0, T=96, H=8, D=128):
    """Per-token deviation over this rank's head shard (oracle math), for 3
    layers of one chunk rotated from position 5 to position 700."""
    g = np.random.default_rng(seed)
    kv = (g.standard_normal((3, 2, 8, 16, H, D)) * 2).astype(np.float32)
    table = R.rope_table(1024, D, 5e5, "bf16")
    rot = R.Rotary(table, "bf16", D, True)
    h0, h1 = tp_head_range(rank, world, H)
    out = np.zeros((3, T), np.float32)
    t = np.arange(T)
    c, s = R.flexible_factors(rot, 5 + t, 700 + t)
    for l in range(3):
        local = np.ascontiguousarray(kv[l][..., h0:h1, :])
        layer = R.KLayer(N.f32_to_bf16(local).reshape(-1), local.shape, tuple(np.array(
            [local.shape[1] * local.shape[2] * local.shape[3] * local.shape[4], local.shape[2] * local.shape[3] *
             local.shape[4], local.shape[3] * local.shape[4], local.shape[4], 1])), False, "bf16")
        out[l] = R.rotate_tokens(layer, rot, R.gather_index(list(range(1, 7)), 16, 0, T), c, s)
    return out


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        part = torch.from_numpy(_partial_scores(rank, world))
        full = allreduce_scores(part.clone())
        k = int(0.2 * full.shape[1])
        sel = [S.topk_positions(full[l].numpy(), k).tolist() for l in range(full.shape[0])]
        q.put((rank, full.numpy(), sel))
    finally:
        dist.destroy_process_group()


def test_tp_scores_allreduce_gives_identical_selection():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict((r, (f, s)) for r, f, s in (q.get(timeout=120) for _ in range(world)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # every rank holds the same summed scores and makes the same selection
    np.testing.assert_array_equal(res[0][0], res[1][0])
    assert res[0][1] == res[1][1]
    # the sum over head shards is the full-head deviation (fp32 sum order only)
    np.testing.assert_allclose(res[0][0], _partial_scores(0, 1), rtol=1e-5)
