"""Generates the golden fixtures of tests/golden/ from the reference itself.

Run in a container where the reference checkout is available:

    python tests/golden/make_golden.py --reference <path-to-DARIC-checkout>

It imports the reference's own modules (nothing is copied):
  * daric.adaption.policy.DARICPolicy  -> policy_cases.json
  * daric.adaption.adapter.Adapter with TRITON_INTERPRET=1, i.e. the
    reference Triton kernel _fused_rerotate_kernel executed by Triton's CPU
    interpreter, on small seeded paged caches -> rerotate_<case>.npz
The interpreter casts fp32 results to bf16 by truncation (fp16 by RTNE); the
tests account for that (see tests/test_golden.py).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def policy_cases(DARICPolicy) -> list[dict]:
    rng = np.random.default_rng(1234)
    cases = []
    fixed = [
        [0, 512], [0, 512, 1024], [0, 512, 1024, 1536, 2048, 2112],
        list(range(0, 8193, 512)) + [8256], [0, 16, 32, 48], [0, 100, 101, 400, 401, 800],
    ]
    params = [(16, 0.1, "linear"), (32, 0.5, "linear"), (76, 0.5, "linear"), (8, 0.2, "exp"),
              (16, 0.5, "log"), (1228, 0.5, "linear"), (51, 0.3, "linear")]
    for gp in fixed:
        for avg, r, fn in params:
            cases.append((gp, avg, r, fn))
    for _ in range(300):
        n = int(rng.integers(1, 24))
        lens = rng.integers(1, 700, size=n)
        gp = [0] + np.cumsum(lens).tolist()
        avg, r, fn = params[int(rng.integers(0, len(params)))]
        cases.append((gp, avg, r, fn))
    out = []
    for gp, avg, r, fn in cases:
        pol = DARICPolicy(avg, r=r, function=fn)
        try:
            res = pol.get_recompute_ptrs([int(x) for x in gp])
            out.append({"group_ptr": [int(x) for x in gp], "avg_num": avg, "r": r, "function": fn,
                        "ptrs": [[int(a), int(b)] for a, b in res]})
        except Exception as e:  # recorded so the restatement must raise too
            out.append({"group_ptr": [int(x) for x in gp], "avg_num": avg, "r": r, "function": fn,
                        "error": type(e).__name__})
    return out


def rope_table_torch(torch, max_pos, rot_dim, base, dtype):
    inv = 1.0 / (base ** (torch.arange(0, rot_dim, 2, dtype=torch.float) / rot_dim))
    t = torch.arange(max_pos, dtype=torch.float)
    f = torch.einsum("i,j -> ij", t, inv)
    return torch.cat((f.cos(), f.sin()), dim=-1).to(dtype)


class _Rot:
    def __init__(self, table, rot_dim, neox):
        self.cos_sin_cache = table
        self.rotary_dim = rot_dim
        self.is_neox_style = neox


def raw(torch, t):
    """Tensor -> raw numpy array (bits) of its storage in element order."""
    t = t.contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    if t.dtype == torch.float32:
        return t.numpy().copy()
    return t.numpy().copy()


def rerotate_cases(ref_root: str) -> dict:
    os.environ["TRITON_INTERPRET"] = "1"
    import torch
    from daric.adaption.adapter import Adapter
    from daric.configs import AdaptionConfig, ProcessLocalConfig
    from daric.configs.engine import CacheTopo, LayerCacheTopo
    from daric.reuse_controller.kvcache import KVCache

    g = torch.Generator().manual_seed(7)

    def make_kv(shape, dtype, kplane):
        x = torch.randn(shape, generator=g, dtype=torch.float32)
        # outlier channels: 4 random K channels per head scaled x8
        k = kplane(x)
        hd = k.shape[-1]
        ch = torch.randperm(hd, generator=g)[:4]
        k[..., ch] *= 8.0
        return x.to(dtype)

    cases = {}
    specs = [
        # name, shape, page_first, dtype, rot_dim, neox, table dtype, mode
        ("flex_5d_bf16_neox", (2, 8, 16, 2, 128), False, torch.bfloat16, 128, True, "flexible"),
        ("strict_5d_bf16_neox", (2, 6, 16, 2, 128), False, torch.bfloat16, 128, True, "strict"),
        ("flex_5dpf_f16_gptj", (8, 2, 16, 2, 64), True, torch.float16, 64, False, "flexible"),
        ("strict_4d_bf16_neox_partial", (6, 2, 16, 2 * 64), True, torch.bfloat16, 32, True, "strict"),
    ]
    for name, shape, pf, dtype, rot_dim, neox, mode in specs:
        if len(shape) == 5:
            kplane = (lambda x: x[:, 0]) if pf else (lambda x: x[0])
        else:
            kplane = lambda x: x[..., : shape[-1] // 2]
        kv = make_kv(shape, dtype, kplane)
        max_pos = 320
        table = rope_table_torch(torch, max_pos, rot_dim, 500000.0, dtype)
        layer = "model.layers.0.self_attn.attn"
        bs = 16
        bpb = int(np.prod(shape[1:] if pf else (shape[0],) + shape[2:])) * kv.element_size()
        topo = CacheTopo(layers={layer: LayerCacheTopo(0, bs, bpb, pf)}, groups=[[layer]])
        ProcessLocalConfig.cache_topo = topo
        cfg = AdaptionConfig(rerotate=True, recompute=True, recompute_policy="daric", recompute_avg_num=16)
        ad = Adapter(cfg)
        kv_in = kv.clone()
        ad.register_kvcaches({layer: kv})
        ad.register_rotary_embed(layer, _Rot(table, rot_dim, neox))
        meta_rec = {}
        if mode == "flexible":
            metas = [
                KVCache("a", [0, 32], saved_pos=0, block_ids=([3, 5],)),
                KVCache("b", [48, 88], saved_pos=7, block_ids=([1, 4, 2],)),  # partial last block
                KVCache("c", [96, 112], saved_pos=96, block_ids=([7],)),     # old == new: skipped
                KVCache("d", [200, 216], saved_pos=300, block_ids=([6],)),    # moves backwards
            ]
            ad.apply_rerotate_load(metas)
            meta_rec = {"ptr": [m.ptr for m in metas], "saved_pos": [m.saved_pos for m in metas],
                        "block_ids": [list(m.block_ids[0]) for m in metas]}
        else:
            group_ptrs = [[0, 16, 40, 64, 80], [0, 32, 48, 50]]
            block_ids = [([1, 2, 3, 4, 5],), ([3, 1, 5, 2],)]
            ad.apply_rerotate_multi(group_ptrs, block_ids)
            meta_rec = {"group_ptrs": group_ptrs, "block_ids": [list(b[0]) for b in block_ids]}
        cases[name] = {
            "arrays": {"kv_in": raw(torch, kv_in), "kv_out": raw(torch, kv), "table": raw(torch, table)},
            "meta": {"shape": list(shape), "page_first": pf, "dtype": str(dtype).replace("torch.", ""),
                     "rotary_dim": rot_dim, "is_neox": neox, "mode": mode, "max_pos": max_pos,
                     "layer": layer, **meta_rec},
        }
    return cases


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference DARIC checkout")
    args = ap.parse_args()
    os.environ["TRITON_INTERPRET"] = "1"  # must be set before triton is imported
    sys.path.insert(0, args.reference)
    from daric.adaption.policy import DARICPolicy

    (HERE / "policy_cases.json").write_text(json.dumps(policy_cases(DARICPolicy)))
    for name, c in rerotate_cases(args.reference).items():
        np.savez_compressed(HERE / f"rerotate_{name}.npz", **c["arrays"])
        (HERE / f"rerotate_{name}.json").write_text(json.dumps(c["meta"]))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
