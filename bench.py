#!/usr/bin/env python
"""Benchmark of the reused-KV hot path.

Workload ("llama3-8b-8k-prompt"): one 8192-token prompt made of 16 reused
512-token chunks placed at shuffled positions, Llama-3-8B KV shape (32
layers, 8 KV heads x 128, bf16, block size 16, RoPE theta 5e5). One step =
the fused store-staging -> re-rotated paged-KV load of every chunk and layer
(flexible PIC: rotate from the saved to the new position) + top-15%
recompute selection per layer on lognormal deviation scores (2% x20), with
the index list and slot mapping as output.

  value : reused-KV GB/s over all ranks, inputs resident in HBM. Algorithmic
          bytes = 4 * H * D * 2 B per token per layer (K,V read from staging
          and written to the paged cache) = 8 KiB; 2.147 GB per prompt.
  e2e   : the same step through the public API from pinned host buffers:
          store shm -> staging H2D (batched_memcpy_h2d), scores H2D, the
          fused load, the selection, D2H of index list + slots.
Multi-GPU (torchrun): requests shard data-parallel, no collective on the
data path; each rank loads its own prompt ("scaling": "weak").

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
METRIC = "reused-KV GB/s per GPU (fraction of HBM peak); µs per 8K-token prompt, 1/2/4/8 GPU"
CFG = dict(layers=32, kv_heads=8, head_dim=128, block_size=16, tokens=8192, chunk=512, theta=5e5,
           ratio=0.15, max_pos=8192)  # config 2, also the reference arm's sample
FALLBACK_HBM_GBS = 6650.0


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def algorithmic_bytes(tokens, layers, heads, dim):
    return tokens * layers * 4 * heads * dim * 2


def rope_table(max_pos, rot_dim, base, dtype):
    # vLLM RotaryEmbedding._compute_cos_sin_cache (fp32 on CPU), cast to the model dtype
    inv = 1.0 / (base ** (torch.arange(0, rot_dim, 2, dtype=torch.float) / rot_dim))
    t = torch.arange(max_pos, dtype=torch.float)
    f = torch.einsum("i,j -> ij", t, inv)
    return torch.cat((f.cos(), f.sin()), dim=-1).to(dtype)


CONFIGS = {
    # the reference's CPU-runnable case, one layer and one reused
    # 512-token chunk rotated by a position delta of U[0, 4096); deviation scores from the
    # fused load, 15% selected (a launch-bound call: its line reports us per call)
    1: dict(name="llama3-8b-single-layer", layers=1, kv_heads=8, head_dim=128, block_size=16, theta=5e5,
            ratio=0.15, requests=1, chunks=1, chunk_len=(512, 512), suffix=0, scores="deviation", tp=False,
            delta=(0, 4096)),
    # one 8K prompt of 16 reused 512-token chunks (default)
    2: dict(name="llama3-8b-8k-prompt", layers=32, kv_heads=8, head_dim=128, block_size=16, theta=5e5,
            ratio=0.15, requests=1, chunks=16, chunk_len=(512, 512), suffix=0, scores="lognormal", tp=False),
    # 64 requests x 6 chunks of U[256, 1024] (multiple of 16) + 64 uncached tokens
    3: dict(name="qwen2.5-7b-64req", layers=28, kv_heads=4, head_dim=128, block_size=16, theta=1e6,
            ratio=0.10, requests=64, chunks=6, chunk_len=(256, 1024), suffix=64, scores="lognormal", tp=False),
    # 70B shape, 32K prompt of 64 x 512 chunks, KV heads split over the ranks,
    # deviation scores all-reduced before a top-20% selection
    4: dict(name="llama3-70b-32k-tp", layers=80, kv_heads=8, head_dim=128, block_size=16, theta=5e5,
            ratio=0.20, requests=1, chunks=64, chunk_len=(512, 512), suffix=0, scores="deviation", tp=True),
    # Mistral-7B shape, requests of U[2048, 16384] tokens in 512-token chunks of
    # which a hit-ratio share is reused (loaded), the rest uncached; one step = a batch of 16
    # requests per rank (the 512-request job runs as 512 / (16 N) steps per rank);
    # --hit and --recompute sweep the two ratios
    5: dict(name="mistral-7b-dp-sweep", layers=32, kv_heads=8, head_dim=128, block_size=16, theta=1e6,
            ratio=0.15, requests=16, req_len=(2048, 16384), chunk=512, hit=0.75, suffix=0,
            scores="lognormal", tp=False),
}


class Workload:
    """Synthetic inputs of one config, seeded: block layout and positions are
    shared by all ranks (seed), values differ per rank (seed + rank)."""

    def __init__(self, device, seed=0, config=2, rank=0, world=1):
        from daric_b200.reuse import ReusedKVLoader, layer_block_bytes
        from daric_b200.shard import tp_head_range
        from daric_b200.topo import CacheTopo
        c = CONFIGS[config]
        self.cfg = c
        self.device = device
        g = torch.Generator(device="cpu").manual_seed(seed)
        L, D, bs = c["layers"], c["head_dim"], c["block_size"]
        H = c["kv_heads"]
        if c["tp"]:
            h0, h1 = tp_head_range(rank, world, H)
            H = h1 - h0
        self.heads = H
        # reused chunks per request: (length, start in the request); placement and
        # shuffled saved positions
        reqs = []
        for r in range(c["requests"]):
            if "req_len" in c:  # request of U[a, b] tokens, chunked; a hit-ratio share is reused
                a, b = c["req_len"]
                n = int(torch.randint(a // bs, b // bs + 1, (1,), generator=g)) * bs
                full = [min(c["chunk"], n - s0) for s0 in range(0, n, c["chunk"])]
                at = np.concatenate([[0], np.cumsum(full)[:-1]]).tolist()
                hit = (torch.rand(len(full), generator=g) < c["hit"]).tolist()
                reqs.append([(ln, st) for ln, st, h in zip(full, at, hit) if h])
            else:
                lo, hi = c["chunk_len"]
                lens = [lo] * c["chunks"] if lo == hi else \
                    [int(x) * bs for x in torch.randint(lo // bs, hi // bs + 1, (c["chunks"],), generator=g)]
                reqs.append(list(zip(lens, np.concatenate([[0], np.cumsum(lens)[:-1]]).tolist())))
        self.chunk_len, self.new_pos, self.old_pos, self.req_of = [], [], [], []
        self.req_tokens = []
        for r, chunks in enumerate(reqs):
            lens = [ln for ln, _ in chunks]
            starts = [int(st) for _, st in chunks]
            order = torch.randperm(len(lens), generator=g).tolist()
            shuffled = [lens[o] for o in order]
            saved_starts = np.concatenate([[0], np.cumsum(shuffled)[:-1]]).tolist()
            saved = [0] * len(lens)
            for slot, o in enumerate(order):
                saved[o] = saved_starts[slot]
            if "delta" in c:  # saved at the request's start, moved by a random delta
                lo, hi = c["delta"]
                saved = list(starts)
                starts = [st + int(torch.randint(lo, hi, (1,), generator=g)) for st in starts]
            self.chunk_len += lens
            self.new_pos += starts
            self.old_pos += saved
            self.req_of += [r] * len(lens)
            self.req_tokens.append(sum(lens))
        M = len(self.chunk_len)
        pages = [n // bs for n in self.chunk_len]
        total_pages = sum(pages)
        nb = total_pages + c["requests"] * (c["suffix"] // bs + 1) + 64
        perm = (torch.randperm(nb - 1, generator=g)[:total_pages] + 1).tolist()
        self.chunk_blocks, k = [], 0
        for n in pages:
            self.chunk_blocks.append(perm[k:k + n])
            k += n
        self.block_table = torch.tensor(perm, dtype=torch.int32, device=device)  # requests back to back
        self.req_blk_off = np.concatenate([[0], np.cumsum([sum(pages[i] for i in range(M) if self.req_of[i] == r)
                                                           for r in range(c["requests"])])[:-1]]).astype(np.int64)
        max_pos = max(o + n for o, n in zip(self.old_pos + self.new_pos, self.chunk_len * 2)) + c["suffix"] + 1
        self.table = rope_table(max_pos, D, c["theta"], torch.bfloat16).to(device)
        self.names = [f"model.layers.{i}.self_attn.attn" for i in range(L)]
        self.kv = {n: torch.zeros((2, nb, bs, H, D), dtype=torch.bfloat16, device=device) for n in self.names}
        topo = CacheTopo.single_group(self.names, bs, layer_block_bytes(self.kv[self.names[0]], False), False)
        per_tok = L * 2 * H * D * 2
        total = sum(self.chunk_len) * per_tok
        self.staging = torch.empty(total, dtype=torch.uint8, device=device)
        gd = torch.Generator(device=device).manual_seed(seed + 1 + rank)
        off = 0
        for m in range(M):  # K,V ~ N(0,1); 4 K channels per head x8
            n = self.chunk_len[m] * per_tok
            x = torch.randn((L, 2, pages[m], bs, H, D), generator=gd, device=device)
            ch = torch.randperm(D, generator=g)[:4].to(device)
            x[:, 0, ..., ch] *= 8.0
            self.staging[off:off + n].view(torch.bfloat16).copy_(x.reshape(-1).to(torch.bfloat16))
            off += n
        del x
        self.loader = ReusedKVLoader(self.kv, topo, self.staging, {n: (self.table, D, True) for n in self.names})
        self.plan = self.loader.plan([(b,) for b in self.chunk_blocks])
        self.cplan = self.loader.plan_chunks([(b,) for b in self.chunk_blocks])
        assert self.plan.total_bytes == total
        T = sum(self.chunk_len)
        self.score_col = np.concatenate([[0], np.cumsum(self.chunk_len)[:-1]]).astype(np.int64)
        if c["scores"] == "lognormal":
            sc = torch.distributions.LogNormal(0.0, 1.0).sample((L, T))
            spikes = torch.rand(L, T, generator=g) < 0.02
            self.scores_host = torch.where(spikes, sc * 20, sc).float().contiguous()
        else:
            self.scores_host = torch.zeros((L, T), dtype=torch.float32)
        self.scores = self.scores_host.to(device)
        self.sel = None
        self.bytes = algorithmic_bytes(T, L, H, D)
        self.tokens = T
        self.seg_len = list(self.req_tokens)
        self.seg_blk_off = self.req_blk_off.tolist()

    def load(self, stream=0, api="chunks", scores=None):
        """The fused load of every chunk and layer: through the chunk-level
        entry point (one descriptor per chunk), or api="jobs" through the
        reference-shaped per-(chunk, layer) job plan. Deviation configs write
        their scores to ``scores`` (default: self.scores)."""
        kw = {}
        if self.cfg["scores"] == "deviation":
            kw = dict(scores=self.scores if scores is None else scores, score_col=self.score_col)
        if api == "jobs":
            self.loader.load(self.plan, mode="flexible", pos_a=self.old_pos, pos_b=self.new_pos,
                             chunk_len=self.chunk_len, stream=stream, **kw)
        else:
            self.loader.load_chunks(self.cplan, mode="flexible", pos_a=self.old_pos, pos_b=self.new_pos,
                                    chunk_len=self.chunk_len, stream=stream, **kw)

    def select(self, scores=None):
        from daric_b200.select import score_select
        self.sel = score_select(scores if scores is not None else self.scores, self.block_table,
                                self.cfg["block_size"], seg_len=self.seg_len, seg_blk_off=self.seg_blk_off,
                                ratio=self.cfg["ratio"], out=self.sel)
        return self.sel

    def step(self):
        self.load()
        if self.cfg["tp"]:
            from daric_b200.shard import allreduce_scores
            allreduce_scores(self.scores)
        return self.select()


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.15)
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            p = [x.strip() for x in l.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for nm, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


class NvmlSampler:
    """SM clock and clock-event reasons of one GPU sampled every ``period``
    seconds by a host thread (NVML), for timed regions too short for
    nvidia-smi's sampling. The GPU is found by its UUID."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device, period=0.001):
        import threading
        self.period = period
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._nv = None
        try:
            import pynvml as nv
            nv.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            try:
                self._h = nv.nvmlDeviceGetHandleByUUID(uuid)
            except Exception:
                self._h = nv.nvmlDeviceGetHandleByIndex(torch.cuda.current_device())
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(self._h, nv.NVML_CLOCK_SM))
            self._nv = nv
        except Exception:
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((float(mhz), int(bits)))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        import threading
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return None
        sm = [m for m, _ in self.samples]
        reasons = sorted({nm for _, b in self.samples for bit, nm in self.REASONS.items() if b & bit})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(sm), "source": f"NVML every {self.period * 1e3:.0f} ms during the timed region"}


def cpu_baseline_run(wl_cpu, min_seconds=3.0, max_reps=50):
    from oracle.torch_cpu import reused_kv_step
    torch.set_num_threads(os.cpu_count() or 1)
    args = wl_cpu
    reps, t0 = 0, time.perf_counter()
    while True:
        reused_kv_step(*args)
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds or reps >= max_reps:
            break
    return reps, el


def make_cpu_workload(wl, chunks=None):
    """The GPU workload copied to host tensors for the CPU path."""
    M = len(wl.chunk_blocks) if chunks is None else chunks
    L = CFG["layers"]
    per_chunk = wl.staging.numel() // len(wl.chunk_blocks)
    stg = wl.staging[: M * per_chunk].cpu()
    kv = [torch.zeros_like(wl.kv[n], device="cpu") for n in wl.names]
    blocks = [torch.tensor(b, dtype=torch.int64) for b in wl.chunk_blocks[:M]]
    k = int(np.floor(CFG["ratio"] * CFG["chunk"] * M + 1e-9))
    sc = wl.scores_host[:, : CFG["chunk"] * M].contiguous()
    bt = wl.block_table.cpu()
    return (kv, stg, blocks, wl.chunk_len[:M], wl.old_pos[:M], wl.new_pos[:M], wl.table.cpu(), sc, k, bt,
            CFG["block_size"]), algorithmic_bytes(CFG["chunk"] * M, L, CFG["kv_heads"], CFG["head_dim"])


def run_reference(args):
    """--impl reference: the reference's math on the host cores (the
    reference has no CPU implementation of this path; oracle/torch_cpu.py
    restates it on torch CPU ops with every host thread)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT))
    from oracle.torch_cpu import reused_kv_step
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    L, H, D, bs, C = CFG["layers"], CFG["kv_heads"], CFG["head_dim"], CFG["block_size"], CFG["chunk"]
    pages = C // bs
    # one step = one reused chunk x all layers (a bounded sample of the prompt)
    stg = torch.randn(L * 2 * pages * bs * H * D, generator=g).to(torch.bfloat16).view(torch.uint8)
    nb = CFG["tokens"] // bs + 64
    kv = [torch.zeros((2, nb, bs, H, D), dtype=torch.bfloat16) for _ in range(L)]
    blocks = [torch.randperm(nb - 1, generator=g)[:pages] + 1]
    table = rope_table(CFG["max_pos"], D, CFG["theta"], torch.bfloat16)
    sc = torch.distributions.LogNormal(0.0, 1.0).sample((L, C))
    k = int(np.floor(CFG["ratio"] * C + 1e-9))
    bt = blocks[0].to(torch.int32)
    step = (kv, stg, blocks, [C], [1536], [512], table, sc, k, bt, bs)
    for _ in range(args.warmup):
        reused_kv_step(*step)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        reused_kv_step(*step)
    el = time.perf_counter() - t0
    nbytes = algorithmic_bytes(C, L, H, D)
    val = nbytes * args.steps / el / 1e9
    sample = f"1 reused 512-token chunk x {L} layers per step (1/16 of the 8K prompt), torch CPU"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(val, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "llama3-8b-8k-prompt", "sample": "1 chunk x 32 layers per step",
                   "parallelism": "host cores"},
        "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(val, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def preroll():
    """A short GPU delay (about 1 ms, not timed) queued before a timed
    region, so the host has queued the first steps when timing starts, as it
    runs ahead of the GPU in a serving loop (otherwise the first step pays
    the host's enqueue latency on an idle GPU)."""
    if hasattr(torch.cuda, "_sleep"):
        torch.cuda._sleep(2_000_000)


def _events(n):
    return [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]


def _max_over_ranks(vals, dist, dev):
    """Element-wise max over ranks of a list of floats (every rank calls)."""
    t = torch.tensor([float(v) for v in vals], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]


def numa_bind(device_index):
    """Binds this process's CPU threads to the NUMA node of its GPU (from
    sysfs), before pinned host buffers are allocated, so their pages come
    from the GPU's node. Returns the node, or None when unknown; the
    previous CPU mask is kept in numa_bind.saved."""
    numa_bind.saved = os.sched_getaffinity(0)
    try:
        bus = torch.cuda.get_device_properties(device_index)
        addr = f"{bus.pci_domain_id:04x}:{bus.pci_bus_id:02x}:{bus.pci_device_id:02x}.0"
        node = int(Path(f"/sys/bus/pci/devices/{addr}/numa_node").read_text().strip())
        if node < 0:
            return None
        cpus = set()
        for part in Path(f"/sys/devices/system/node/node{node}/cpulist").read_text().strip().split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
        return node
    except Exception:
        return None


def time_paths(wl, dev, stream, peak, dist, reps=10):
    """The two unfused paths a DARIC user can run, timed with CUDA events:
      strict : strict PIC (the reference's published configuration): the
               Adapter re-rotates every middle group of the request in place
               by its group offset, all layers in one launch (adapter.py:118-194)
      dropin : the unchanged store's scatter_pages, then the Adapter's
               flexible re-rotation in place (adapter.py:196-295)
    Each gets its algorithmic GB/s (the path's bytes / device time) and the
    roofline of its kernels (bytes they must move / device time)."""
    from types import SimpleNamespace

    from daric_b200.adaption import Adapter, AdaptionConfig
    from daric_b200.cache_ops import CacheCopier
    c = wl.cfg
    L, H, D, bs = c["layers"], wl.heads, c["head_dim"], c["block_size"]
    ad = Adapter(AdaptionConfig(), cache_topo=wl.loader.topo)
    ad.register_kvcaches(wl.kv)
    for n in wl.names:
        ad.register_rotary_embed(n, SimpleNamespace(cos_sin_cache=wl.table, rotary_dim=D, is_neox_style=True))
    # strict: one request per wl request, groups = its chunks in prompt order
    gps, blists, rot_tok = [], [], 0
    for r in range(c["requests"]):
        ms = [m for m in range(len(wl.chunk_len)) if wl.req_of[m] == r]
        ms.sort(key=lambda m: wl.new_pos[m])
        gp = [0] + np.cumsum([wl.chunk_len[m] for m in ms]).tolist()
        gps.append(gp)
        blists.append(([b for m in ms for b in wl.chunk_blocks[m]],))
        rot_tok += sum(gp[i + 1] - gp[i] for i in range(1, len(gp) - 2))
    k_bytes = rot_tok * L * 2 * H * D * 2  # K read + written
    metas = [SimpleNamespace(ptr=[nw, nw + ln], saved_pos=old, block_ids=(blk,))
             for nw, old, ln, blk in zip(wl.new_pos, wl.old_pos, wl.chunk_len, wl.chunk_blocks)]
    copier = CacheCopier()
    for n, t in wl.kv.items():
        copier.register_layer(n, t, False)
        copier.register_rotary(n, wl.table, D, True)
    copier.register_store(wl.staging)
    pl = wl.plan
    # the launches the Adapter issues, with their block tables built once
    # (the kernel-only timing the roofline uses)
    s_tab = torch.tensor([b for bl in blists for b in bl[0]], dtype=torch.int32, device=dev)
    s_off = np.concatenate([[0], np.cumsum([len(bl[0]) for bl in blists])[:-1]]).tolist()
    s_seg = [(s_off[r], gp[i] - gp[0], gp[i + 1] - gp[i], gp[i] - gp[0])
             for r, gp in enumerate(gps) for i in range(1, len(gp) - 2) if gp[i + 1] > gp[i]]
    f_tab = torch.tensor([b for blk in wl.chunk_blocks for b in blk], dtype=torch.int32, device=dev)
    f_off = np.concatenate([[0], np.cumsum([len(b) for b in wl.chunk_blocks])[:-1]]).tolist()
    moving = [m for m in range(len(wl.chunk_len)) if wl.old_pos[m] != wl.new_pos[m]]

    def strict():
        ad.apply_rerotate_multi(gps, blists)

    def strict_kernel():
        copier.rerotate_inplace(wl.names, "delta", s_tab, [x[0] for x in s_seg], [x[1] for x in s_seg],
                                [x[2] for x in s_seg], [x[3] for x in s_seg])

    def dropin():
        copier.scatter_pages(pl.c_names, pl.offsets, pl.byte_sizes, pl.indices_flat, pl.indices_offsets)
        ad.apply_rerotate_load(metas)

    def dropin_kernel():
        copier.scatter_pages(pl.c_names, pl.offsets, pl.byte_sizes, pl.indices_flat, pl.indices_offsets)
        copier.rerotate_inplace(wl.names, "flexible", f_tab, [f_off[m] for m in moving], [0] * len(moving),
                                [wl.chunk_len[m] for m in moving], [wl.old_pos[m] for m in moving],
                                [wl.new_pos[m] for m in moving])

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        preroll()
        ev = _events(reps)
        for i in range(reps):
            ev[i][0].record(stream)
            fn()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
        ms = [a.elapsed_time(b) for a, b in ev]
        return _max_over_ranks([sum(ms) / reps, min(ms)], dist, dev)

    out = {}
    for name, fn, kfn in (("strict", strict, strict_kernel), ("dropin", dropin, dropin_kernel)):
        avg, mn = timed(fn)
        kavg, kmn = timed(kfn)
        if name == "strict":
            alg = moved = k_bytes
        else:
            alg = wl.bytes
            moved = wl.bytes + sum(wl.chunk_len[m] for m in moving) * L * 2 * H * D * 2
        out[name] = {
            "us": round(avg * 1e3, 2), "us_min": round(mn * 1e3, 2),
            "algorithmic_bytes": alg, "gbs": round(alg / (avg * 1e-3) / 1e9, 1),
            "kernel_us": round(kavg * 1e3, 2), "kernel_us_min": round(kmn * 1e3, 2),
            "roofline": {"bound": "hbm", "moved_bytes": moved, "achieved": round(moved / (kavg * 1e-3) / 1e9, 1),
                         "peak": peak, "unit": "GB/s", "frac": round(moved / (kavg * 1e-3) / 1e9 / peak, 4),
                         "timing": "the kernel launches of the path with their block tables built once"}}
    out["strict"]["rotated_tokens"] = rot_tok
    out["strict"]["kernel"] = "bulk_inplace_kernel (DELTA, all layers, one launch)"
    out["strict"]["us_is"] = "Adapter.apply_rerotate_multi per call (block table built and uploaded per call)"
    out["dropin"]["kernel"] = "bulk_pages_kernel (plain scatter) + bulk_inplace_kernel (FLEXIBLE)"
    out["dropin"]["us_is"] = "scatter_pages + Adapter.apply_rerotate_load per call"
    return out


def run_tp(args, dist, rank, world, dev, stream, peak):
    """BASELINE config 4 across the ranks: one 32K-token 70B-shaped prompt,
    KV heads split over the ranks (each rank loads and rotates its heads and
    writes partial per-token deviation scores), one NCCL all-reduce of the
    [80, 32768] fp32 scores, then the same top-20% selection on every rank.
    Checks: every rank's index list and slot mapping are identical (hash
    all-gather), and rank 0's equal a numpy top-k (ties to the lower index) of
    the all-reduced scores."""
    import hashlib

    from daric_b200.shard import allreduce_scores
    from daric_b200.select import topk_count
    wl = Workload(dev, seed=0, config=4, rank=rank, world=world)
    steps = max(3, min(args.steps, 20))
    for _ in range(3):
        wl.load()
        allreduce_scores(wl.scores)
        wl.select()
    torch.cuda.synchronize()
    # pipelined steps: the scores alternate between two buffers and each
    # step's selection runs on a second stream beside the next step's load
    bufs = [wl.scores, torch.empty_like(wl.scores)]
    done = [torch.cuda.Event(), torch.cuda.Event()]
    sel_stream = torch.cuda.Stream(dev)
    dist.barrier()
    torch.cuda.synchronize()
    preroll()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    for i in range(steps):
        b = i % 2
        if i >= 2:
            stream.wait_event(done[b])
        wl.load(scores=bufs[b])
        allreduce_scores(bufs[b])
        sel_stream.wait_stream(stream)
        with torch.cuda.stream(sel_stream):
            wl.select(bufs[b])
        done[b].record(sel_stream)
    stream.wait_stream(sel_stream)
    p1.record(stream)
    torch.cuda.synchronize()
    piped = p0.elapsed_time(p1) / steps
    # in-line steps: load, all-reduce and selection timed one by one
    dist.barrier()
    torch.cuda.synchronize()
    preroll()
    e = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]
    for i in range(steps):
        e[i][0].record(stream)
        wl.load()
        e[i][1].record(stream)
        allreduce_scores(wl.scores)
        e[i][2].record(stream)
        sel = wl.select()
        e[i][3].record(stream)
    torch.cuda.synchronize()
    load = sum(x[0].elapsed_time(x[1]) for x in e) / steps
    ar = sum(x[1].elapsed_time(x[2]) for x in e) / steps
    sl = sum(x[2].elapsed_time(x[3]) for x in e) / steps
    step = e[0][0].elapsed_time(e[-1][3]) / steps
    load_min = min(x[0].elapsed_time(x[1]) for x in e)
    load_m, ar_m, sl_m, step_m, piped_m = _max_over_ranks([load, ar, sl, step, piped], dist, dev)
    dist.barrier()
    # identical selection on every rank
    idx, slot, cnt = sel.idx.cpu().numpy(), sel.slot.cpu().numpy(), sel.count.cpu().numpy()
    h = hashlib.sha256(idx.tobytes() + slot.tobytes() + cnt.tobytes()).digest()[:8]
    mine = torch.tensor([int.from_bytes(h, "little", signed=True)], dtype=torch.int64, device=dev)
    allh = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(allh, mine)
    identical = len({int(x.item()) for x in allh}) == 1
    out = None
    if rank == 0:
        sc = wl.scores.cpu().numpy()
        bt = wl.block_table.cpu().numpy().astype(np.int64)
        L, T = sc.shape
        k = topk_count(T, wl.cfg["ratio"])
        ok = True
        for l in range(L):
            u = sc[l].view(np.uint32)
            key = np.where(u & 0x80000000, ~u, u | 0x80000000).astype(np.uint32)
            order = np.lexsort((np.arange(T), ~key))[:k]
            pos = np.sort(order)
            n = int(cnt[l, 0])
            ok = ok and n == k and np.array_equal(idx[l, :n], pos) and \
                np.array_equal(slot[l, :n], bt[pos // 16] * 16 + pos % 16)
        tot = wl.bytes * world
        out = {
            "workload": "llama3-70b-32k-tp (BASELINE config 4)", "tp": world, "kv_heads_per_rank": wl.heads,
            "steps": steps, "us_per_prompt": round(piped_m * 1e3, 2),
            "value_gbs": round(tot / (piped_m * 1e-3) / 1e9, 1),
            "pipelining": "selection of each step beside the next step's load (scores double-buffered)",
            "us_per_prompt_in_line": round(step_m * 1e3, 2),
            "load_us": round(load_m * 1e3, 2), "load_us_min_rank0": round(load_min * 1e3, 2),
            "per_rank_load_frac": round(wl.bytes / (load_m * 1e-3) / 1e9 / peak, 4),
            "allreduce_us": round(ar_m * 1e3, 2), "allreduce_bytes": int(wl.scores.numel() * 4),
            "select_us": round(sl_m * 1e3, 2),
            "selection_identical": identical, "selection_matches_cpu_topk": bool(ok),
            "nccl_ranks": dist.get_world_size(), "algorithmic_bytes_per_rank": wl.bytes,
            "limiter": "load kernel" if load_m >= ar_m else "all-reduce"}
    del wl, sel
    torch.cuda.empty_cache()
    dist.barrier()
    return out


def run_ours(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    numa = numa_bind(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from daric_b200 import _lib
    cfg = CONFIGS[args.config]
    tp = cfg["tp"]
    peak, peak_kind = measured_peak()
    # data parallel: every rank loads its own requests; tensor parallel: one
    # prompt, each rank its KV-head shard
    # --tp-shard N (config 4, one process): rank 0's KV-head shard of an N-way
    # split, for single-GPU profiling of the TP shapes (no all-reduce)
    shard = args.tp_shard if (tp and world == 1 and args.tp_shard) else 0
    wl = Workload(dev, seed=0 if tp else rank, config=args.config, rank=rank if tp else 0,
                  world=(shard or world) if tp else 1)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if dist is not None:
            dist.barrier()

    for _ in range(args.warmup):
        wl.step()
    torch.cuda.synchronize()
    warm_err = _lib.device_errors(local)
    if warm_err:
        raise RuntimeError(f"device error bits {warm_err} during warm-up; not timing a failing path")
    barrier()
    torch.cuda.synchronize()
    ev = _events(args.steps)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # A step's selection runs on a second stream after its load, beside the
    # next step's load, as a pipelined server runs consecutive batches
    # (--serial-select keeps it in line). Scores produced by the load
    # (config 4) alternate between two buffers, so the next load does not
    # overwrite the scores a selection still reads.
    overlap = not args.serial_select
    deviation = cfg["scores"] == "deviation"
    bufs = [wl.scores, torch.empty_like(wl.scores)] if (deviation and overlap) else [wl.scores]
    sel_done = [torch.cuda.Event(), torch.cuda.Event()]
    sel_stream = torch.cuda.Stream(dev)
    with ClockSampler(local) as clk, NvmlSampler(dev) as nvml:
        preroll()
        start.record(stream)
        h0 = time.perf_counter()
        for i in range(args.steps):
            b = i % len(bufs)
            if len(bufs) > 1 and i >= 2:
                stream.wait_event(sel_done[b])  # the selection of step i-2 has read buffer b
            ev[i][0].record(stream)
            wl.load(scores=bufs[b])
            ev[i][1].record(stream)
            if tp:
                from daric_b200.shard import allreduce_scores
                allreduce_scores(bufs[b])
            if overlap:
                sel_stream.wait_stream(stream)
                with torch.cuda.stream(sel_stream):
                    wl.select(bufs[b])
                sel_done[b].record(sel_stream)
            else:
                wl.select(bufs[b])
        host_us = (time.perf_counter() - h0) / args.steps * 1e6  # enqueue time per step
        stream.wait_stream(sel_stream)
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    kern_ms = [a.elapsed_time(b) for a, b in ev]
    ms_max = _max_over_ranks([ms], dist, dev)[0]
    errors = _lib.device_errors(local)

    # ---- the selection alone: device time of back-to-back calls
    preroll()
    sev = _events(10)
    for a, b in sev:
        a.record(stream)
        wl.select()
        b.record(stream)
    torch.cuda.synchronize()
    sel_ms = [a.elapsed_time(b) for a, b in sev]
    sel_avg, sel_min = _max_over_ranks([sum(sel_ms) / len(sel_ms), min(sel_ms)], dist, dev)

    # ---- host cost of one call with the descriptor ring free (6 steps = 12
    # of its 16 slots, enqueued after the device went idle)
    torch.cuda.synchronize()
    t_load, t_jobs, t_sel = [], [], []
    for _ in range(5):
        a = time.perf_counter()
        wl.load()
        b = time.perf_counter()
        wl.load(api="jobs")
        c = time.perf_counter()
        wl.select()
        t_load.append(b - a)
        t_jobs.append(c - b)
        t_sel.append(time.perf_counter() - c)
        torch.cuda.synchronize()
    host_call = {"load_chunks_us": round(statistics.median(t_load) * 1e6, 1),
                 "load_jobs_us": round(statistics.median(t_jobs) * 1e6, 1),
                 "select_us": round(statistics.median(t_sel) * 1e6, 1),
                 "note": "median host time per call with the descriptor ring free (no back-pressure)"}

    # ---- the unfused paths (strict PIC in place, and scatter + in-place flexible)
    # (strict PIC rotates the middle chunks of a request: none in config 1)
    paths = time_paths(wl, dev, stream, peak, dist) if not tp and cfg["chunks"] >= 3 else None

    # ---- e2e: public API from pinned host buffers; each step builds its
    # request's load plan and uploads its block ids, as a server does per
    # request. Three public paths:
    #   serial    : batched_memcpy_h2d of the chunks, the reference-shaped job
    #               plan (gpu_kv_io.py:334-379) and the fused load
    #   chunks    : the same copies, then the chunk-level load (one
    #               descriptor per chunk, jobs built on the device)
    #   layerwise : chunk plan, host -> staging per 4-layer step on a copy
    #               stream overlapped with the fused kernel of the previous step
    # then the selection and the D2H of the index list and slots.
    from daric_b200.cache_ops import batched_memcpy_h2d
    host_shm = torch.empty(wl.staging.numel(), dtype=torch.uint8).pin_memory()
    host_shm.copy_(wl.staging)
    host_scores = wl.scores_host.pin_memory()
    sel = wl.select()
    out_idx = torch.empty(sel.idx.shape, dtype=sel.idx.dtype).pin_memory()
    out_slot = torch.empty(sel.slot.shape, dtype=sel.slot.dtype).pin_memory()
    out_cnt = torch.empty(sel.count.shape, dtype=sel.count.dtype).pin_memory()
    chunk_off = wl.plan.chunk_offsets.tolist()
    chunk_size = wl.plan.chunk_sizes.tolist()
    e2e_steps = max(3, min(args.steps, 10))
    block_lists = [(b,) for b in wl.chunk_blocks]
    dev_kw = dict(scores=wl.scores, score_col=wl.score_col) if cfg["scores"] == "deviation" else {}
    pos_kw = dict(mode="flexible", pos_a=wl.old_pos, pos_b=wl.new_pos, chunk_len=wl.chunk_len)

    def finish():
        if tp:
            from daric_b200.shard import allreduce_scores
            allreduce_scores(wl.scores)
        s = wl.select()
        out_idx.copy_(s.idx, non_blocking=True)
        out_slot.copy_(s.slot, non_blocking=True)
        out_cnt.copy_(s.count, non_blocking=True)

    def e2e_serial():
        batched_memcpy_h2d(host_shm, wl.staging, chunk_off, chunk_off, chunk_size)
        if not tp:
            wl.scores.copy_(host_scores, non_blocking=True)
        wl.plan = wl.loader.plan(block_lists)
        wl.load(api="jobs")
        finish()

    def e2e_chunks():
        batched_memcpy_h2d(host_shm, wl.staging, chunk_off, chunk_off, chunk_size)
        if not tp:
            wl.scores.copy_(host_scores, non_blocking=True)
        cp = wl.loader.plan_chunks(block_lists)
        wl.loader.load_chunks(cp, **pos_kw, **dev_kw)
        finish()

    def e2e_layerwise():
        if not tp:
            wl.scores.copy_(host_scores, non_blocking=True)
        cp = wl.loader.plan_chunks(block_lists)
        wl.loader.load_layerwise(cp, host_shm, layers_per_step=4, **pos_kw, **dev_kw)
        finish()

    e2e_ms = {}
    with ClockSampler(local) as clk_e2e:
        for name, fn in (("serial", e2e_serial), ("chunks", e2e_chunks), ("layerwise", e2e_layerwise)):
            for _ in range(2):
                fn()
            torch.cuda.synchronize()
            barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(e2e_steps):
                fn()
            e1.record(stream)
            torch.cuda.synchronize()
            e2e_ms[name] = e0.elapsed_time(e1)
        # layer-wise: when the first layer step is in the paged cache (the
        # model can start its first layers) against the whole load
        if not tp:
            wl.scores.copy_(host_scores, non_blocking=True)
        torch.cuda.synchronize()
        f0 = torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        lw = wl.loader.load_layerwise(wl.loader.plan_chunks(block_lists), host_shm, layers_per_step=4,
                                      **pos_kw, **dev_kw)
        torch.cuda.synchronize()
        first_ms, all_ms = f0.elapsed_time(lw.events[0][1]), f0.elapsed_time(lw.events[-1][1])
        # the host->device ceiling: one plain pinned copy of the same bytes
        # on every rank at once
        barrier()
        torch.cuda.synchronize()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        for _ in range(3):
            wl.staging.copy_(host_shm, non_blocking=True)
        c1.record(stream)
        torch.cuda.synchronize()
    ceil_ms = c0.elapsed_time(c1) / 3
    names_e2e = ["serial", "chunks", "layerwise"]
    mx = _max_over_ranks([e2e_ms[n] for n in names_e2e] + [ceil_ms], dist, dev)
    e2e_max = dict(zip(names_e2e, mx[:3]))
    ceil_ms_max = mx[3]
    e2e_best = min(names_e2e, key=lambda n: e2e_max[n])
    e2e_ms_max = e2e_max[e2e_best]
    tot_bytes = float(wl.bytes) * world
    h2d = wl.staging.numel() + (0 if tp else wl.scores_host.numel() * 4)
    d2h = out_idx.numel() * 4 + out_slot.numel() * 8 + out_cnt.numel() * 4
    del host_shm

    # ---- tensor-parallel config 4 across the ranks (its one collective)
    tp_line = run_tp(args, dist, rank, world, dev, stream, peak) if (dist is not None and not tp) else None

    if rank == 0:
        kern_avg_ms = sum(kern_ms) / len(kern_ms)
        achieved = wl.bytes / (kern_avg_ms * 1e-3) / 1e9
        traffic = None
        tp_file = ROOT / "profiles" / "traffic.json"
        if tp_file.exists() and args.config == 2:
            traffic = json.loads(tp_file.read_text()).get("rerotate_scatter_kernel_bytes_per_launch")
        value = tot_bytes * args.steps / (ms_max * 1e-3) / 1e9
        e2e_val = tot_bytes * e2e_steps / (e2e_ms_max * 1e-3) / 1e9
        h2d_rate = h2d * world / (e2e_ms_max / e2e_steps * 1e-3) / 1e9
        ceiling = wl.staging.numel() * world / (ceil_ms_max * 1e-3) / 1e9
        clocks = nvml.summary() or clk.summary()
        clocks["reasons_whole_run"] = sorted(set(clk.summary()["reasons"]) | set(clk_e2e.summary()["reasons"]))
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 5), "higher_is_better": True,
            "scaling": "strong" if tp else "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": cfg["name"], "layers": cfg["layers"], "kv_heads": cfg["kv_heads"],
                       "kv_heads_per_gpu": wl.heads, "head_dim": cfg["head_dim"], "block_size": cfg["block_size"],
                       "tokens_per_gpu": wl.tokens, "chunks": len(wl.chunk_len), "rope": "flexible",
                       "theta": cfg["theta"], "select": f"top{int(cfg['ratio'] * 100)}%/layer/request",
                       "scores": cfg["scores"] + (" (NCCL all-reduce over KV-head shards)" if tp else ""),
                       "requests_per_gpu": cfg["requests"], "hit_ratio": cfg.get("hit"),
                       "parallelism": (f"tp{world}" if tp else f"dp{world}") +
                                      (f" (rank-0 shard of tp{shard} on one GPU)" if shard else ""),
                       "l2": "inputs larger than L2 (staging + paged cache >> 126 MB), no flush",
                       "selection": "second stream, beside the next step's load" if overlap else "in line"},
            "us_per_prompt": round(ms_max / args.steps * 1e3, 2) if args.config in (1, 2, 4) else None,
            "select_device_us": {"avg": round(sel_avg * 1e3, 2), "min": round(sel_min * 1e3, 2),
                                 "note": "the selection alone, back-to-back calls (in the step it runs beside "
                                         "the next load)"},
            "frac_of_hbm_peak": round(value / world / peak, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": "bulk_pages_kernel (fused re-rotate + scatter)", "peak_kind": peak_kind,
                         "kernel_us": round(kern_avg_ms * 1e3, 2),
                         "kernel_us_min": round(min(kern_ms) * 1e3, 2),
                         "kernel_us_median": round(statistics.median(kern_ms) * 1e3, 2),
                         "algorithmic_bytes_per_launch": wl.bytes},
            "e2e": {"value": round(e2e_val, 3), "unit": "GB/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": round(e2e_ms_max / e2e_steps, 4),
                    "path": e2e_best,
                    "layerwise_first_step_ms": round(first_ms, 3), "layerwise_all_layers_ms": round(all_ms, 3),
                    "paths_ms_per_step": {n: round(e2e_max[n] / e2e_steps, 4) for n in names_e2e},
                    "plan": "built per step (block ids uploaded per request)",
                    "h2d_gbs": round(h2d_rate, 1),
                    "h2d_ceiling_gbs": round(ceiling, 1),
                    "frac_of_h2d_ceiling": round(h2d_rate / ceiling, 4),
                    "h2d_ceiling": "plain pinned copy_ of the staging bytes on every rank at once",
                    "numa_node": numa},
            "gpu_launches": 3 * args.steps,
            "host_us_per_step": round(host_us, 1),
            "host_us_per_call": host_call,
            "clocks": clocks,
            "device_errors": errors,
        }
        if args.trace:
            line["trace_kernel_us"] = [round(x * 1e3, 1) for x in kern_ms]
        if paths is not None:
            line["paths"] = paths
        if tp_line is not None:
            line["tp"] = tp_line
        if world == 1 and args.config == 2 and not args.no_cpu_baseline:
            sys.path.insert(0, str(ROOT))
            os.sched_setaffinity(0, numa_bind.saved)  # the CPU baseline uses every host core
            cw, cbytes = make_cpu_workload(wl, chunks=args.cpu_chunks)
            reps, el = cpu_baseline_run(cw)
            line["cpu_baseline"] = {
                "value": round(cbytes * reps / el / 1e9, 3), "unit": "GB/s", "cores": torch.get_num_threads(),
                "kind": "port",
                "sample": f"{args.cpu_chunks} of 16 chunks x 32 layers per pass, {reps} passes in {el:.1f}s "
                          "(torch CPU restatement: scatter + flexible re-rotation + top-k)"}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_profile_case(args):
    """--profile-case: the small cases the ncu summaries under profiles/ were
    captured on (no timing). The workload of --config with --layers layers
    (inputs still larger than L2), then three calls of one path:
      fused   : the fused re-rotate + scatter load (chunk-level entry point)
      jobs    : the same through the reference-shaped job plan
      strict  : in-place strict-PIC rotation of the request's middle groups
      flexible: in-place flexible rotation of every chunk
      select  : the top-k selection of every layer on lognormal scores
    """
    from daric_b200 import _lib
    if args.layers:
        CONFIGS[args.config]["layers"] = args.layers
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    wl = Workload(dev, seed=0, config=args.config, rank=0, world=args.tp_shard or 1)
    from daric_b200.cache_ops import CacheCopier
    copier = CacheCopier()
    for n, t in wl.kv.items():
        copier.register_layer(n, t, False)
        copier.register_rotary(n, wl.table, wl.cfg["head_dim"], True)
    req = [m for m in range(len(wl.chunk_len)) if wl.req_of[m] == 0]
    req.sort(key=lambda m: wl.new_pos[m])
    starts = np.concatenate([[0], np.cumsum([wl.chunk_len[m] for m in req])]).tolist()
    if args.profile_case == "select":
        torch.manual_seed(1)
        wl.scores.copy_(torch.distributions.LogNormal(0.0, 1.0).sample(tuple(wl.scores.shape)))
    for _ in range(3):
        if args.profile_case == "select":
            wl.select()
        elif args.profile_case == "fused":
            wl.load()
        elif args.profile_case == "jobs":
            wl.load(api="jobs")
        elif args.profile_case == "strict":
            mid = range(1, len(req) - 1)
            copier.rerotate_inplace(wl.names, "delta", wl.block_table, [0] * len(mid), [starts[i] for i in mid],
                                    [wl.chunk_len[req[i]] for i in mid], [starts[i] for i in mid])
        else:
            copier.rerotate_inplace(wl.names, "flexible", wl.block_table, [0] * len(req),
                                    [wl.new_pos[m] for m in req], [wl.chunk_len[m] for m in req],
                                    [wl.old_pos[m] for m in req], [wl.new_pos[m] for m in req])
    torch.cuda.synchronize()
    assert _lib.device_errors(0) == 0
    print(json.dumps({"profile_case": args.profile_case, "config": args.config, "layers": wl.cfg["layers"],
                      "kv_heads": wl.heads, "algorithmic_bytes_fused": wl.bytes}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-chunks", type=int, default=4)
    ap.add_argument("--config", type=int, choices=sorted(CONFIGS), default=2,
                    help="BASELINE.json config: 1 (one layer, one 512-token chunk), 2 (default, 8K prompt), "
                         "3 (64-request batch), 4 (70B, TP heads), 5 (Mistral-7B data-parallel hit/recompute sweep)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--hit", type=float, default=None, help="config 5: reused share of the chunks (0.5/0.75/0.95)")
    ap.add_argument("--recompute", type=float, default=None, help="recompute ratio (top share per layer/request)")
    ap.add_argument("--serial-select", action="store_true",
                    help="run each step's selection in line after its load (default for input scores: on a "
                         "second stream, beside the next step's load)")
    ap.add_argument("--trace", action="store_true", help="add each timed step's load time (us) to the line")
    ap.add_argument("--profile-case", choices=["fused", "jobs", "strict", "flexible", "select"], default=None,
                    help="build the workload and run one path three times, untimed (the ncu capture cases)")
    ap.add_argument("--layers", type=int, default=0, help="with --profile-case: layers of the workload")
    ap.add_argument("--tp-shard", type=int, default=0,
                    help="config 4 on one GPU: run rank 0's KV-head shard of this TP degree (2/4/8)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.hit is not None:
        CONFIGS[5]["hit"] = args.hit
    if args.recompute is not None:
        CONFIGS[args.config]["ratio"] = args.recompute
    if args.profile_case:
        run_profile_case(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
