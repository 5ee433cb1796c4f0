"""daric_score_select_noalloc: the recompute selection for callers that must
not allocate device memory once running (for example a serving process that
handed all free device memory to its KV cache at start-up). Called through
the C ABI and compared with daric_score_select and with the CPU selection
restatement on the same inputs, two calls in a row; the device's free memory
must not move across calls once the kernels are loaded. The file name makes
pytest collect it after every other test."""
import ctypes as C

import numpy as np
import pytest
import torch

from daric_b200 import _lib
from oracle import select as S

pytestmark = pytest.mark.gpu


def _call(fn_name, scores, bt, bs, lens, ks, pos0, blk_off, mode, threshold, out=None):
    """Runs one selection entry point; returns (count, [(idx, slot) per (layer, request)]) on the host.
    ``out``: preallocated (idx, slot, count) device tensors to write into."""
    lib = _lib.load()
    L, T = scores.shape
    nseg = len(lens)
    lens_a, lp = _lib.i64(lens)
    cols_a, cp = _lib.i64(np.concatenate([[0], np.cumsum(lens)[:-1]]))
    pos_a, pp = _lib.i64(pos0)
    blk_a, bp = _lib.i64(blk_off)
    caps = np.minimum(ks, lens) if mode == _lib.SELECT_TOPK else np.asarray(lens)
    k_a, kp = _lib.i64(ks)
    off_a, op = _lib.i64(np.concatenate([[0], np.cumsum(caps)[:-1]]))
    if out is None:
        out_ld = max(int(np.sum(caps)), 1)
        idx = torch.full((L, out_ld), -7, dtype=torch.int32, device="cuda")
        slot = torch.full((L, out_ld), -7, dtype=torch.int64, device="cuda")
        cnt = torch.full((L, nseg), -7, dtype=torch.int32, device="cuda")
    else:
        idx, slot, cnt = out
        out_ld = idx.stride(0)
        assert out_ld >= int(np.sum(caps)) and cnt.numel() >= L * nseg
    stream = torch.cuda.current_stream().cuda_stream
    rc = getattr(lib, fn_name)(
        C.c_void_p(scores.data_ptr()), L, scores.stride(0), nseg, cp, lp, pp, kp, mode, C.c_float(threshold),
        C.c_void_p(bt.data_ptr()), bt.numel(), bp, bs, C.c_void_p(idx.data_ptr()), C.c_void_p(slot.data_ptr()),
        C.c_void_p(cnt.data_ptr()), out_ld, op, 0, C.c_void_p(stream))
    _lib.check(rc)
    torch.cuda.synchronize()
    counts = cnt.view(-1)[: L * nseg].view(L, nseg).cpu().numpy()
    offs = off_a
    out = []
    for l in range(L):
        for s in range(nseg):
            n = int(counts[l, s])
            o = int(offs[s])
            out.append((idx[l, o:o + n].cpu().numpy(), slot[l, o:o + n].cpu().numpy()))
    return counts, out


def _case(seed, L, lens, ratio):
    g = torch.Generator().manual_seed(seed)
    T = int(sum(lens))
    scores = torch.distributions.LogNormal(0.0, 1.0).sample((L, T)).float()
    scores[:, ::7] = 3.0  # ties at many ranks
    bs = 16
    pos0 = [16 * i for i in range(len(lens))]
    tables = [torch.randint(1, 5000, ((p + n + bs - 1) // bs + 1,), generator=g).int() for p, n in zip(pos0, lens)]
    blk_off = np.concatenate([[0], np.cumsum([len(t) for t in tables])[:-1]])
    ks = [int(np.floor(ratio * n + 1e-9)) for n in lens]
    return scores.cuda(), torch.cat(tables).cuda(), bs, lens, ks, pos0, blk_off


def _oracle(scores, bt, bs, lens, ks, pos0, blk_off, mode, thr):
    """Per (layer, request) positions and slots from the CPU restatement."""
    sc = scores.cpu().numpy()
    table = bt.cpu().numpy().astype(np.int64)
    cols = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    out = []
    for l in range(sc.shape[0]):
        for s, n in enumerate(lens):
            row = sc[l, cols[s]:cols[s] + n]
            j = S.topk_positions(row, ks[s]) if mode == _lib.SELECT_TOPK else S.threshold_positions(row, thr)
            p = pos0[s] + j
            out.append((p, table[blk_off[s] + p // bs] * bs + p % bs))
    return out


def test_noalloc_select_matches_select_two_calls_in_a_row():
    cases = [_case(1, 4, [512, 300, 0, 77], 0.15), _case(2, 3, [8192, 1024], 0.2)]
    for scores, bt, bs, lens, ks, pos0, blk_off in cases:  # two calls in a row, different shapes
        for mode, thr in ((_lib.SELECT_TOPK, 0.0), (_lib.SELECT_THRESHOLD, 2.5)):
            ref = _call("daric_score_select", scores, bt, bs, lens, ks, pos0, blk_off, mode, thr)
            exp = _oracle(scores, bt, bs, lens, ks, pos0, blk_off, mode, thr)
            for _ in range(2):
                got = _call("daric_score_select_noalloc", scores, bt, bs, lens, ks, pos0, blk_off, mode, thr)
                np.testing.assert_array_equal(got[0], ref[0])
                for (gi, gs), (ri, rs), (ei, es) in zip(got[1], ref[1], exp):
                    np.testing.assert_array_equal(gi, ri)
                    np.testing.assert_array_equal(gs, rs)
                    np.testing.assert_array_equal(gi, ei)
                    np.testing.assert_array_equal(gs, es)


def test_noalloc_select_allocates_no_device_memory():
    cases = [_case(3, 4, [512, 300, 0, 77], 0.15), _case(4, 3, [8192, 1024], 0.2), _case(5, 2, [40] * 700, 0.3)]
    L = max(c[0].shape[0] for c in cases)
    nseg = max(len(c[3]) for c in cases)
    ld = max(int(sum(c[3])) for c in cases)
    out = (torch.empty((L, ld), dtype=torch.int32, device="cuda"), torch.empty((L, ld), dtype=torch.int64,
           device="cuda"), torch.empty(L * nseg, dtype=torch.int32, device="cuda"))
    args = [(c, m, t) for c in cases for m, t in ((_lib.SELECT_TOPK, 0.0), (_lib.SELECT_THRESHOLD, 2.5))]
    c, m, t = args[0]
    _call("daric_score_select_noalloc", *c, m, t, out=out)  # loads the kernels (lazy module loading)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    results = []
    for rep in range(10):
        c, m, t = args[rep % len(args)]
        results.append(_call("daric_score_select_noalloc", *c, m, t, out=out))
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"device free memory moved by {free0 - free1} bytes across calls"
    for rep, got in enumerate(results):  # and the results are still the selection
        c, m, t = args[rep % len(args)]
        for (gi, gs), (ei, es) in zip(got[1], _oracle(*c, m, t)):
            np.testing.assert_array_equal(gi, ei)
            np.testing.assert_array_equal(gs, es)


def test_noalloc_select_block_table_too_short_gives_slot_minus_one():
    scores, bt, bs, lens, ks, pos0, blk_off = _case(6, 2, [256], 0.5)
    short = bt[:5].contiguous()  # positions 0..79 have a block, the rest do not
    assert _lib.device_errors(0) == 0
    got = _call("daric_score_select_noalloc", scores, short, bs, lens, ks, pos0, [0], _lib.SELECT_TOPK, 0.0)
    assert _lib.device_errors(0) == 0  # the library's device error word is not used by this entry point
    table = short.cpu().numpy().astype(np.int64)
    for l, (gi, gs) in enumerate(got[1]):
        exp = S.topk_positions(scores[l].cpu().numpy(), ks[0])
        np.testing.assert_array_equal(gi, exp)
        inside = exp // bs < len(table)
        assert (~inside).any() and inside.any()
        np.testing.assert_array_equal(gs[inside], table[exp[inside] // bs] * bs + exp[inside] % bs)
        assert (gs[~inside] == -1).all()


def test_noalloc_select_rejects_too_many_requests():
    # header limit: DARIC_NOALLOC_MAX_SEGMENTS = 1024
    lens = [2] * 1025
    scores = torch.rand(1, sum(lens), device="cuda")
    bt = torch.ones(4096, dtype=torch.int32, device="cuda")
    with pytest.raises(_lib.DaricError, match="1024"):
        _call("daric_score_select_noalloc", scores, bt, 16, lens, [1] * 1025, [0] * 1025, [0] * 1025,
              _lib.SELECT_TOPK, 0.0)
