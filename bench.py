#!/usr/bin/env python
"""Decode-step benchmark of the B200 paged decode path (one JSON line on rank 0).

Metric: decode-step microseconds and effective KV-read GB/s per GPU against the
B200 HBM peak. Effective bytes are the reference's Workload::min_bytes (src/workload.hpp:69-74): K
and V of every live token, plus q and out. ``value`` is the whole-job GB/s (sum over ranks of
bytes per step / the slowest rank's step time).

Workloads (seeded synthetic data generated on the device):
  1  f32, 1 x 32/8 heads x 128, context 512, page 16, 64-page pool
  2  f16, context 4096, page 32, 256-page pool, split-K partition 512
  3  int8 (default; --dtype f16 for the fp16 variant), context 32768, page 128, 512-page pool  [default]
  4  f16, 64 sequences, lengths log-uniform in [512, 32768], page 16, pool 1.1 x live pages;
     sharded by sequence (LPT bin packing) across ranks, outputs all-gathered with NCCL
  5  f16 or int8, 256 sequences, 64/8 heads, lengths uniform in [8192, 131072], page 64;
     sharded by KV head across ranks, outputs all-gathered with NCCL
Configs 1-3 are single-sequence steps; with --gpus N every rank runs its own replica (weak
scaling). Inputs of configs 1-3 fit in L2 (126 MB), so each timed step reads one of R pool copies in
rotation (R * live bytes > 4 x L2); configs 4-5 are far larger than L2.

Timing: W warm-up steps, then exactly K steps between a barrier + synchronize on each side, timed
with CUDA events on the launching stream; max over ranks. Single-GPU replica steps are submitted as
CUDA-graph replays (one kernel launch per step). NVML samples SM clocks and throttle reasons during
the timed region. ``e2e`` measures the same metric through the public API (PagedDecoder ->
kvb_paged_decode_async) with per-step host->device copies of the step's inputs (q, sequence
lengths, block table) from pinned memory and a device->host read of the output; the KV pool is
device-resident state (written when a page is written), and ``e2e_pool_upload`` additionally copies
the whole pool every step. ``--impl reference`` times the reference's own CPU implementation
(oracle/_ref/kvb_ref_cpu, built from its src/reference.cpp and src/workload.hpp) on this host.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

METRIC = "decode-step µs and effective KV-read GB/s per GPU vs B200 HBM peak"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference", "torch-sdpa"], default="ours",
                    help="ours; the reference's CPU implementation; or torch SDPA on a contiguous cache")
    ap.add_argument("--config", type=int, default=3, choices=[1, 2, 3, 4, 5])
    ap.add_argument("--dtype", choices=["f32", "f16", "i8"], default=None)
    ap.add_argument("--kernel", choices=["auto", "simt", "mma", "umma"], default="auto")
    ap.add_argument("--part", type=int, default=None, help="override the split-K partition size")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="launch every step from the host")
    ap.add_argument("--ramp-s", type=float, default=1.0, help="untimed load before warm-up (clock ramp)")
    ap.add_argument("--seqs", type=int, default=None,
                    help="keep only the first N sequences of the config (a smaller case for profilers)")
    ap.add_argument("--op", choices=["decode", "quantize", "scatter"], default="decode",
                    help="decode step (default) or the page write path in front of it (one GPU)")
    return ap.parse_args()


# ---------------------------------------------------------------------------------------------------
# workloads

def workload(cfg: int, dtype):
    if cfg == 1:
        w = dict(H=32, Hkv=8, D=128, kv="f32", lens=[512], page=16, pool_blocks=64, part=0, seed=1,
                 shard="replica")
    elif cfg == 2:
        w = dict(H=32, Hkv=8, D=128, kv="f16", lens=[4096], page=32, pool_blocks=256, part=512, seed=2,
                 shard="replica")
    elif cfg == 3:
        w = dict(H=32, Hkv=8, D=128, kv="i8", lens=[32768], page=128, pool_blocks=512, part=0, seed=3,
                 shard="replica")
    elif cfg == 4:
        rng = np.random.default_rng(4)
        lens = np.rint(np.exp(rng.uniform(math.log(512), math.log(32768), 64))).astype(int).tolist()
        w = dict(H=32, Hkv=8, D=128, kv="f16", lens=lens, page=16, pool_slack=1.1, part=0, seed=4,
                 shard="sequence")
    else:
        rng = np.random.default_rng(5)
        lens = rng.integers(8192, 131072, 256, endpoint=True).tolist()
        w = dict(H=64, Hkv=8, D=128, kv="f16", lens=lens, page=64, pool_slack=1.0, part=0, seed=5,
                 shard="kv_head")
    if dtype:
        w["kv"] = dtype
    w["cfg"] = cfg
    return w


def describe(w):
    toks = sum(w["lens"])
    cut = f" (first {len(w['lens'])} sequences)" if w.get("cut") else ""
    return (f"config{w['cfg']}{cut}: {w['kv']} cache, B={len(w['lens'])}, H={w['H']}/Hkv={w['Hkv']}, D={w['D']}, "
            f"page={w['page']}, tokens={toks}, max_len={max(w['lens'])}")


def min_bytes(w, lens, Hkv, H):
    elem = {"f32": 4, "f16": 2, "i8": 1}[w["kv"]]
    return float(sum(lens)) * Hkv * w["D"] * 2 * elem + float(len(lens)) * H * w["D"] * 8


# ---------------------------------------------------------------------------------------------------
# clocks

class ClockSampler:
    """Samples SM clock, max clock and throttle reasons with NVML in a background thread."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, index: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._active = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - NVML is optional; the line then says so
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            if self._active:
                try:
                    self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                    bits = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                    for b, n in self.REASONS.items():
                        if bits & b:
                            self.reasons.add(n)
                except Exception:  # noqa: BLE001
                    pass
            time.sleep(0.005)

    def start(self):
        if self.nv:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def active(self, on: bool):
        self._active = on

    def stop(self):
        if self.nv:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.nv:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


# ---------------------------------------------------------------------------------------------------
# device data

def build_layout(lens, page, slack, pool_blocks, rng):
    nblk = [(int(l) + page - 1) // page for l in lens]
    live = sum(nblk)
    num_blocks = pool_blocks if pool_blocks else max(live, int(math.ceil(live * slack)))
    num_blocks = max(num_blocks, live, 1)
    perm = rng.permutation(num_blocks).astype(np.int32)
    max_blocks = max(nblk) if nblk else 0
    table = np.full((len(lens), max(max_blocks, 1)), -1, np.int32)
    nxt = 0
    for b, n in enumerate(nblk):
        table[b, :n] = perm[nxt:nxt + n]
        nxt += n
    return table, num_blocks


def make_pool(torch, num_blocks, hk, page, D, kv, gen, device):
    """K or V pool [num_blocks][hk][page][D], values U(-1, 1); int8 quantized per (block, KV head) with
    scale = absmax / 127 (the reference's symmetric scheme, src/reference.cpp:32-51)."""
    shape = (num_blocks, hk, page, D)
    if kv in ("f32", "f16"):
        t = torch.empty(shape, dtype=torch.float32 if kv == "f32" else torch.float16, device=device)
        step = max(1, (1 << 28) // (hk * page * D))
        for b0 in range(0, num_blocks, step):
            t[b0:b0 + step].uniform_(-1, 1, generator=gen)
        return t, None
    q8 = torch.empty(shape, dtype=torch.int8, device=device)
    sc = torch.empty((num_blocks, hk), dtype=torch.float32, device=device)
    step = max(1, (1 << 27) // (hk * page * D))
    for b0 in range(0, num_blocks, step):
        x = torch.empty((min(step, num_blocks - b0), hk, page, D), dtype=torch.float32, device=device)
        x.uniform_(-1, 1, generator=gen)
        amax = x.abs().amax(dim=(2, 3))
        s = amax / 127.0
        q8[b0:b0 + step] = torch.where(s[:, :, None, None] > 0, torch.round(x / s[:, :, None, None]),
                                       torch.zeros_like(x)).clamp_(-127, 127).to(torch.int8)
        sc[b0:b0 + step] = s
    return q8, sc


class Shard:
    """What one rank holds and computes."""

    def __init__(self, torch, w, rank, world, device, copies):
        from kv_cache_bench_b200 import shard as sh
        lens = list(w["lens"])
        self.H, self.Hkv = w["H"], w["Hkv"]
        self.seqs = list(range(len(lens)))
        self.owned = None
        if w["shard"] == "sequence" and world > 1:
            self.owned = sh.lpt_assign(lens, world)
            self.seqs = self.owned[rank]
        if w["shard"] == "kv_head" and world > 1:
            hk = sh.kv_head_ranges(w["Hkv"], world)[rank]
            self.Hkv = len(hk)
            self.H = w["H"] // world
        self.lens = [lens[b] for b in self.seqs]
        self.world, self.rank = world, rank
        rng = np.random.default_rng(w["seed"] * 1000 + rank)
        gen = torch.Generator(device=device)
        gen.manual_seed(w["seed"] * 1000 + rank)
        table, self.num_blocks = build_layout(self.lens, w["page"], w.get("pool_slack", 1.0), w.get("pool_blocks"),
                                              rng)
        D = w["D"]
        self.q = torch.empty((len(self.lens), self.H, D), dtype=torch.float32, device=device).uniform_(-1, 1,
                                                                                                         generator=gen)
        self.table = torch.from_numpy(table).to(device)
        self.seq_lens = torch.tensor(self.lens, dtype=torch.int32, device=device)
        self.out = torch.empty_like(self.q)
        self.pools = []
        for _ in range(copies):
            k, ks = make_pool(torch, self.num_blocks, self.Hkv, w["page"], D, w["kv"], gen, device)
            v, vs = make_pool(torch, self.num_blocks, self.Hkv, w["page"], D, w["kv"], gen, device)
            self.pools.append((k, v, ks, vs))
        self.max_len = max(self.lens) if self.lens else 0
        self.bytes = min_bytes(w, self.lens, self.Hkv, self.H)
        self.live_pool_bytes = float(sum(self.lens)) * self.Hkv * D * 2 * {"f32": 4, "f16": 2, "i8": 1}[w["kv"]]


# ---------------------------------------------------------------------------------------------------
# CPU baseline (the reference's own implementation, or the oracle port when it was not built)

def sample_lens(w, budget_tokens: int):
    """The first sequences of the workload, in order, up to `budget_tokens` tokens; the last one taken
    may be cut to a prefix of its context (a shorter step of the same shape)."""
    lens, left = [], max(1, int(budget_tokens))
    for l in w["lens"]:
        if left <= 0:
            break
        lens.append(min(l, left))
        left -= lens[-1]
    return lens


def time_cpu_reference(w, lens, steps: int):
    """ms per step and bytes per step (Workload::min_bytes, src/workload.hpp:69-74) of the reference's
    CPU implementation on `lens`: oracle/_ref/kvb_ref_cpu (the reference's attention_reference with
    all host threads), else the C restatement in oracle/."""
    exe = os.path.join(ROOT, "oracle", "_ref", "kvb_ref_cpu")
    threads = os.cpu_count() or 1
    if os.path.exists(exe):
        cmd = [exe, f"--heads={w['H']}", f"--kv-heads={w['Hkv']}", f"--dim={w['D']}", f"--type={w['kv']}",
               f"--page={w['page']}", f"--lens={','.join(map(str, lens))}", f"--steps={steps}",
               f"--seed={w['seed']}", f"--threads={threads}"]
        r = json.loads(subprocess.run(cmd, check=True, capture_output=True, text=True).stdout.strip().splitlines()[-1])
        return r["ms_per_step"], float(r["min_bytes"]), r["threads"], "reference", \
            "reference attention_reference (fp64, src/reference.cpp:65-100), oracle/_ref/kvb_ref_cpu"
    import oracle
    kvt = {"f32": oracle.F32, "f16": oracle.F16, "i8": oracle.I8}[w["kv"]]
    case = oracle.make_case(num_heads=w["H"], num_kv_heads=w["Hkv"], head_dim=w["D"], lens=lens, kv_type=kvt,
                            page=w["page"], seed=w["seed"])
    case.reference(threads)
    t0 = time.perf_counter()
    for _ in range(steps):
        case.reference(threads)
    ms = (time.perf_counter() - t0) / steps * 1e3
    return ms, case.min_bytes(), threads, "port", "oracle/kvb_oracle.c (C restatement)"


def cpu_sample(w, step_seconds: float):
    """Token budget of one CPU step that takes about `step_seconds` (calibrated on a short sample)."""
    probe = sample_lens(w, 4096)
    ms, _, _, _, _ = time_cpu_reference(w, probe, 1)
    tokens_per_s = sum(probe) / max(ms * 1e-3, 1e-6)
    return max(128, int(tokens_per_s * step_seconds))


def cpu_baseline(w, seconds: float = 12.0):
    """The reference's CPU step timed on a bounded sample of the workload (about `seconds` of CPU
    work): the whole step when it takes under a quarter of that, else a token-bounded prefix."""
    total = sum(w["lens"])
    budget = min(total, cpu_sample(w, seconds / 4))
    lens = sample_lens(w, budget)
    ms1, _, _, _, _ = time_cpu_reference(w, lens, 1)
    steps = int(max(2, min(1000, seconds / max(ms1 * 1e-3, 1e-6))))
    ms, nbytes, threads, kind, impl = time_cpu_reference(w, lens, steps)
    sample = (f"{len(lens)} of {len(w['lens'])} sequences, {sum(lens)} of {total} tokens "
              f"({100.0 * sum(lens) / total:.1f}% of the step), {steps} timed steps after 1 warm-up")
    return {"value": round(nbytes / (ms * 1e-3) / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": kind,
            "ms_per_step": round(ms, 3), "sample": sample, "impl": impl}


def run_reference_arm(args, w):
    """`--impl reference`: the reference's own CPU implementation of the step, on rank 0 only, each of
    the W + K steps a bounded sample of the workload so that the run ends within about a minute."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    steps = max(args.steps, 1)
    total = sum(w["lens"])
    budget = min(total, cpu_sample(w, 60.0 / (steps + max(args.warmup, 1))))
    lens = sample_lens(w, budget)
    ms, nbytes, threads, kind, impl = time_cpu_reference(w, lens, steps)
    value = round(nbytes / (ms * 1e-3) / 1e9, 4)
    sample = (f"{len(lens)} of {len(w['lens'])} sequences, {sum(lens)} of {total} tokens "
              f"({100.0 * sum(lens) / total:.1f}% of the step) per step, {steps} timed steps after 1 warm-up")
    cb = {"value": value, "unit": "GB/s", "cores": threads, "kind": kind, "ms_per_step": round(ms, 3),
          "sample": sample, "impl": impl}
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "weak" if w["shard"] == "replica" else "strong", "vs_baseline": None, "dtype": w["kv"],
        "data": "synthetic: the reference's own seeded Workload generator", "config": config_obj(w, None, world),
        "cpu_baseline": cb, "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_torch_sdpa(args, w):
    """`--impl torch-sdpa`: the library comparison point on the same GPU (the reference compares
    itself with llama.cpp and MLX on its own hardware). torch's scaled_dot_product_attention on a
    contiguous, unpaged cache [1][Hkv][L][D] of the same shape and storage type, the G query heads of a
    KV head passed as G query rows so that K and V are read once per KV head, as in our kernel. Same
    metric and algorithmic bytes; pool copies rotated past 4 x L2; CUDA-graph replays of at least 64
    steps. Single-sequence configs (1-3) with f32 or f16 storage (SDPA takes no int8 cache); rank 0."""
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    if int(os.environ.get("RANK", "0")) != 0:
        return
    if len(w["lens"]) != 1 or w["kv"] == "i8":
        print(json.dumps({"impl": "torch-sdpa", "unavailable": "single-sequence f32/f16 configs only (1-3)"}),
              flush=True)
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L, H, Hkv, D = w["lens"][0], w["H"], w["Hkv"], w["D"]
    dt = torch.float16 if w["kv"] == "f16" else torch.float32
    elem = 2 if w["kv"] == "f16" else 4
    nbytes = min_bytes(w, w["lens"], Hkv, H)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    copies = max(1, min(64, math.ceil(4 * l2 / (L * Hkv * D * 2 * elem))))
    gen = torch.Generator(device=dev)
    gen.manual_seed(w["seed"])

    def uniform(*shape):
        return (torch.rand(shape, generator=gen, device=dev) * 2 - 1).to(dt)

    ks = [uniform(1, Hkv, L, D) for _ in range(copies)]
    vs = [uniform(1, Hkv, L, D) for _ in range(copies)]
    q = uniform(1, Hkv, H // Hkv, D)
    chosen = None
    for name, be in (("flash", SDPBackend.FLASH_ATTENTION), ("cudnn", SDPBackend.CUDNN_ATTENTION),
                     ("efficient", SDPBackend.EFFICIENT_ATTENTION), ("math", SDPBackend.MATH)):
        try:
            with sdpa_kernel(be):
                F.scaled_dot_product_attention(q, ks[0], vs[0])
            torch.cuda.synchronize()
            chosen = (name, be)
            break
        except RuntimeError:
            continue
    if chosen is None:
        print(json.dumps({"impl": "torch-sdpa", "unavailable": "no SDPA backend ran this shape"}), flush=True)
        return
    name, be = chosen
    per_graph = copies * max(1, math.ceil(64 / copies))
    stream = torch.cuda.Stream(dev)
    graphs = {}

    def graph_of(n):
        if n not in graphs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream), sdpa_kernel(be):
                F.scaled_dot_product_attention(q, ks[0], vs[0])
                stream.synchronize()
                with torch.cuda.graph(g, stream=stream):
                    for i in range(n):
                        F.scaled_dot_product_attention(q, ks[i % copies], vs[i % copies])
            graphs[n] = g
        return graphs[n]

    def run_steps(n):
        full, rem = divmod(n, per_graph)
        with torch.cuda.stream(stream):
            for _ in range(full):
                graph_of(per_graph).replay()
            if rem:
                graph_of(rem).replay()

    run_steps(max(args.warmup, 3))
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record()
    run_steps(args.steps)
    with torch.cuda.stream(stream):
        e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    value = round(nbytes / (ms * 1e-3) / 1e9, 2)
    cfg = config_obj(w, None, 1)
    cfg.update({"layout": "contiguous [1][Hkv][L][D], G query rows per KV head", "sdpa_backend": name,
                "l2": f"{copies} cache copies rotated", "submission": "cuda graph replay"})
    print(json.dumps({"impl": "torch-sdpa", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": 1,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 6),
                      "higher_is_better": True, "dtype": w["kv"], "data": "synthetic: seeded U(-1,1) q/K/V",
                      "config": cfg, "torch": torch.__version__}), flush=True)


def config_obj(w, part, world):
    par = {"replica": "replicas", "sequence": f"sequence-sharded x{world} (LPT)",
           "kv_head": f"kv-head-sharded x{world}"}[w["shard"]]
    c = {"workload": describe(w), "batch": len(w["lens"]), "heads": w["H"], "kv_heads": w["Hkv"], "head_dim": w["D"],
         "seq_len": max(w["lens"]), "tokens": sum(w["lens"]), "page_size": w["page"], "parallelism": par}
    if part is not None:
        c["part_tokens"] = part
    return c


def read_traffic(w):
    """Per-launch DRAM bytes from the committed ncu summary of this workload, if any."""
    path = os.path.join(ROOT, "profiles", f"traffic_config{w['cfg']}_{w['kv']}.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith("dram_bytes_per_launch:"):
            return float(line.split(":", 1)[1])
    return None


def peak_hbm():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:  # noqa: BLE001
        return FALLBACK_HBM_GBS, "fallback"


# ---------------------------------------------------------------------------------------------------

def run_write_path(args, w):
    """`--op quantize|scatter`: the page write path (kvb_quantize_paged_i8 / kvb_scatter_paged) on the
    workload's contiguous cache, one GPU; GB/s of live bytes read and written per launch."""
    import torch

    import kv_cache_bench_b200 as kvb
    quantize = args.op == "quantize"
    kv = "i8" if quantize else (w["kv"] if w["kv"] in ("f32", "f16") else "f16")
    device = torch.device("cuda", 0)
    lens = list(w["lens"])
    B, Hkv, D, page = len(lens), w["Hkv"], w["D"], w["page"]
    max_len = max(lens)
    src_dt = torch.float32 if kv in ("i8", "f32") else torch.float16
    if B * Hkv * max_len * D * (4 if src_dt == torch.float32 else 2) > (40 << 30):
        raise SystemExit("the contiguous cache of this config does not fit the write-path bench")
    rng = np.random.default_rng(w["seed"])
    table, num_blocks = build_layout(lens, page, w.get("pool_slack", 1.0), w.get("pool_blocks"), rng)
    gen = torch.Generator(device=device)
    gen.manual_seed(w["seed"])
    contig = torch.empty((B, Hkv, max_len, D), dtype=src_dt, device=device).uniform_(-1, 1, generator=gen)
    pool = torch.zeros((num_blocks, Hkv, page, D), dtype=torch.int8 if quantize else src_dt, device=device)
    scales = torch.zeros((num_blocks, Hkv), device=device)
    tb = torch.from_numpy(table).to(device)
    ln = torch.tensor(lens, dtype=torch.int32, device=device)
    a = kvb.page_write_args(B, Hkv, D, kvb.KvType[kv], page, table.shape[1], max_len, contig=contig.data_ptr(),
                            block_table=tb.data_ptr(), seq_lens=ln.data_ptr(), pool=pool.data_ptr(),
                            num_blocks=num_blocks, scales=scales.data_ptr())
    fn = kvb.quantize_paged_i8 if quantize else kvb.scatter_paged
    stream = torch.cuda.Stream(device)
    for _ in range(max(args.warmup, 3)):
        fn(a, stream.cuda_stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream.synchronize()
    with torch.cuda.stream(stream):
        e0.record()
    for _ in range(args.steps):
        fn(a, stream.cuda_stream)
    with torch.cuda.stream(stream):
        e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    live = float(sum(lens)) * Hkv * D
    in_b = live * contig.element_size()
    out_b = live * pool.element_size() + (float(sum((l + page - 1) // page for l in lens)) * Hkv * 4 if quantize else 0)
    gbs = (in_b + out_b) / (ms * 1e-3) / 1e9
    peak, peak_kind = peak_hbm()
    print(json.dumps({
        "metric": f"page write path ({'int8 quantize' if quantize else 'scatter'}) GB/s", "op": args.op,
        "value": round(gbs, 2), "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 6), "higher_is_better": True, "dtype": kv,
        "data": "synthetic: U(-1,1) contiguous cache generated on the device",
        "config": dict(config_obj(w, None, 1), source_bytes=in_b, pool_bytes=out_b,
                       l2=f"contiguous input {in_b / 1e6:.0f} MB vs L2 {torch.cuda.get_device_properties(device).L2_cache_size / 1e6:.0f} MB"),
        "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs / peak, 4), "peak_kind": peak_kind},
        "gpu_launches": args.steps}), flush=True)


def main():
    args = parse_args()
    w = workload(args.config, args.dtype)
    if args.seqs is not None and 0 < args.seqs < len(w["lens"]):
        w["lens"], w["cut"] = w["lens"][:args.seqs], True
    if args.impl == "reference":
        run_reference_arm(args, w)
        return
    if args.impl == "torch-sdpa":
        run_torch_sdpa(args, w)
        return
    if args.op != "decode":
        run_write_path(args, w)
        return
    import torch
    import torch.distributed as dist

    import kv_cache_bench_b200 as kvb
    from kv_cache_bench_b200 import shard as sh
    from kv_cache_bench_b200.torch_ops import PagedDecoder

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # pool copies so that the data a step reads cycles through more than 4 x L2
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    elem = {"f32": 4, "f16": 2, "i8": 1}[w["kv"]]
    live_est = float(sum(w["lens"])) * w["Hkv"] * w["D"] * 2 * elem / (world if w["shard"] != "replica" else 1)
    copies = max(1, min(64, math.ceil(4 * l2 / max(live_est, 1)))) if w["shard"] == "replica" else 1
    s = Shard(torch, w, rank, world, device, copies)
    kernel = {"auto": kvb.Kernel.auto, "simt": kvb.Kernel.simt, "mma": kvb.Kernel.mma,
              "umma": kvb.Kernel.umma}[args.kernel]
    part = w["part"] if args.part is None else args.part
    dec = PagedDecoder(device)
    stream = torch.cuda.Stream(device)

    def c_args(i):
        k, v, ks, vs = s.pools[i]
        # nothing in the step loop writes the lengths or the block table: the kernel may read them
        # while the previous step finishes
        return dec.args(s.q, k, v, s.table, s.seq_lens, s.max_len, out=s.out, k_scale=ks, v_scale=vs,
                        part_tokens=part, kernel=kernel, tables_ready=True)

    cargs = [c_args(i) for i in range(copies)]
    need = kvb.paged_workspace_bytes(cargs[0])
    dec.workspace = torch.zeros(max(need, 256), dtype=torch.uint8, device=device)
    ws_ptr, ws_n = dec.workspace.data_ptr(), dec.workspace.numel()
    part_used = kvb.paged_part_tokens(cargs[0])

    gathered = None
    if world > 1 and w["shard"] == "sequence":
        pad = max(len(o) for o in s.owned)
        local_out = torch.zeros((pad, s.H, w["D"]), dtype=torch.float32, device=device)
        gathered = torch.empty((world * pad, s.H, w["D"]), dtype=torch.float32, device=device)
        gidx = torch.from_numpy(sh.sequence_gather_index(s.owned, pad)).to(device)
    elif world > 1 and w["shard"] == "kv_head":
        gathered = torch.empty((world,) + tuple(s.out.shape), dtype=torch.float32, device=device)
    final = torch.empty((len(w["lens"]), w["H"], w["D"]), dtype=torch.float32, device=device)

    def gather():
        """All-gather of the per-rank outputs into `final` (global order); nothing for replicas."""
        if gathered is None:
            return s.out
        with torch.cuda.stream(stream):
            if w["shard"] == "sequence":
                local_out[: s.out.shape[0]].copy_(s.out)
                dist.all_gather_into_tensor(gathered, local_out)
                torch.index_select(gathered, 0, gidx, out=final)
            else:
                dist.all_gather_into_tensor(gathered, s.out)
                final.copy_(gathered.permute(1, 0, 2, 3).reshape(final.shape))
        return final

    def step(i):
        kvb.paged_decode_async(cargs[i % copies], ws_ptr, ws_n, stream.cuda_stream)
        gather()

    use_graph = not args.no_graph and gathered is None
    graphs = {}

    def graph_of(n):
        if n not in graphs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                step(0)  # warm the launch path outside capture
                stream.synchronize()
                with torch.cuda.graph(g, stream=stream):
                    for i in range(n):
                        step(i)
            graphs[n] = g
        return graphs[n]

    # graphs of at least 64 steps (a whole number of pool rotations): consecutive launches inside a
    # graph overlap through programmatic dependent launch, launches across two replays do not
    per_graph = copies * max(1, math.ceil(64 / copies))

    def run_steps(n):
        if not use_graph:
            for i in range(n):
                step(i)
            return
        full, rem = divmod(n, per_graph)
        with torch.cuda.stream(stream):
            for _ in range(full):
                graph_of(per_graph).replay()
            if rem:
                graph_of(rem).replay()

    try:  # NVML numbers devices physically; map through CUDA_VISIBLE_DEVICES
        nvml_index = torch.cuda._get_nvml_device_index(local)
    except Exception:  # noqa: BLE001
        nvml_index = local
    clocks = ClockSampler(nvml_index)
    clocks.start()
    clocks.active(True)
    # untimed clock ramp, then warm-up
    barrier()
    t_end = time.time() + args.ramp_s
    while time.time() < t_end:
        run_steps(max(copies, 64))
        stream.synchronize()
    run_steps(args.warmup)
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record()
    run_steps(args.steps)
    with torch.cuda.stream(stream):
        e1.record()
    barrier()
    clocks.active(False)
    clocks.stop()
    ms_total = e0.elapsed_time(e1)
    flag = dec.error_flag(stream)
    t = torch.tensor([ms_total], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = float(t.item()) / max(args.steps, 1)
    byt = torch.tensor([s.bytes], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(byt)
    job_bytes = float(byt.item())
    value = job_bytes / (ms_step * 1e-3) / 1e9

    # end to end through the public API with host buffers (single replica path and shards alike)
    e2e = e2e_pool = None
    if not args.no_e2e:
        e2e, e2e_pool = measure_e2e(torch, dist, s, dec, part, kernel, stream, args, world, barrier, job_bytes, w,
                                    gather)

    cb = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cb = cpu_baseline(w)
        except Exception as ex:  # noqa: BLE001
            cb = {"value": None, "error": str(ex)[:200]}

    if rank == 0:
        peak, peak_kind = peak_hbm()
        per_gpu = s.bytes / (ms_step * 1e-3) / 1e9
        traffic = read_traffic(w)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 6), "us_per_step": round(ms_step * 1e3, 3),
            "gbps_per_gpu": round(per_gpu, 2), "higher_is_better": True,
            "scaling": "weak" if w["shard"] == "replica" else "strong", "vs_baseline": None, "dtype": w["kv"],
            "data": "synthetic: seeded U(-1,1) q/K/V generated on the device"
                    + ("; int8 quantized per (page, KV head), scale = absmax/127" if w["kv"] == "i8" else ""),
            "config": dict(config_obj(w, part_used, world),
                           l2=(f"{copies} rotating pool copies ({copies * s.live_pool_bytes / 1e6:.0f} MB live "
                               f"> 4 x L2 {l2 / 1e6:.0f} MB)" if copies > 1 else
                               f"inputs {s.live_pool_bytes / 1e6:.0f} MB per GPU > L2 {l2 / 1e6:.0f} MB"),
                           submission="cuda graph replay" if use_graph else "host launch per step",
                           kernel=args.kernel),
            "roofline": {"bound": "hbm", "achieved": round(per_gpu, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(per_gpu / peak, 4), "peak_kind": peak_kind,
                         "traffic": traffic, "algorithmic_bytes_per_launch": s.bytes,
                         "note": "achieved = min_bytes per launch / device time per step (one decode kernel "
                                 "per step); peak = measured copy bandwidth"},
            "gpu_launches": args.steps, "error_flag": flag, "clocks": clocks.summary(),
        }
        if e2e:
            line["e2e"] = e2e
        if e2e_pool:
            line["e2e_pool_upload"] = e2e_pool
        if cb:
            line["cpu_baseline"] = cb
        print(json.dumps(line), flush=True)
    graphs.clear()
    if world > 1:
        dist.destroy_process_group()


def measure_e2e(torch, dist, s, dec, part, kernel, stream, args, world, barrier, job_bytes, w, gather):
    """The same metric through the public C ABI with host buffers: per step, one host->device copy
    of the step's inputs (q, sequence lengths, block table, packed in one pinned staging buffer),
    kvb_paged_decode_async reading them where they landed, the output all-gather when sharded, and
    the device->host copy of the (global) output. The KV pool is device-resident state (written when a
    page is written), rotated over the same copies as the device timing.

    Unsharded steps that move more than 1 MiB of inputs and outputs are pipelined as a serving loop
    would run them: two staging and two output buffers, the input copy of step i+1 and the readback of
    step i-1 on their own streams while step i's kernel runs (events keep each buffer's writer after its
    last reader). Every step still copies its inputs in and its output out inside the timed region.
    Smaller steps (configs 1-3) run on one stream: there the cross-stream event handoffs cost more
    than the copies they would hide (config 3: 49 us pipelined against 39 us). Sharded runs keep one
    stream too (the all-gather sits between kernel and readback)."""
    import kv_cache_bench_b200 as kvb

    def align(n):
        return (n + 255) // 256 * 256

    q_b, l_b, t_b = s.q.numel() * 4, s.seq_lens.numel() * 4, s.table.numel() * 4
    off_l = align(q_b)
    off_t = off_l + align(l_b)
    total = off_t + t_b
    host = torch.empty(total, dtype=torch.uint8, pin_memory=True)
    host[:q_b].copy_(s.q.cpu().view(-1).view(torch.uint8))
    host[off_l:off_l + l_b].copy_(s.seq_lens.cpu().view(-1).view(torch.uint8))
    host[off_t:off_t + t_b].copy_(s.table.cpu().view(-1).view(torch.uint8))
    stage = torch.empty(total, dtype=torch.uint8, device=s.q.device)
    q = stage[:q_b].view(torch.float32).view(s.q.shape)
    lens = stage[off_l:off_l + l_b].view(torch.int32)
    table = stage[off_t:off_t + t_b].view(torch.int32).view(s.table.shape)
    result = gather()
    torch.cuda.synchronize()
    hout = torch.empty(result.shape, dtype=result.dtype, pin_memory=True)
    # the lengths and the table arrive by host copy each step (no kernel writes them)
    cargs = [dec.args(q, k, v, table, lens, s.max_len, out=s.out, k_scale=ks, v_scale=vs, part_tokens=part,
                      kernel=kernel, tables_ready=True) for (k, v, ks, vs) in s.pools]
    need = max(kvb.paged_workspace_bytes(c) for c in cargs)
    if need > dec.workspace.numel():
        dec.workspace = torch.zeros(need, dtype=torch.uint8, device=s.q.device)
    ws, wsn = dec.workspace.data_ptr(), dec.workspace.numel()
    h2d = total
    d2h = hout.numel() * hout.element_size()
    n = min(max(args.steps, 1), 2000)
    raw = stream.cuda_stream

    def one(i, pool_upload=None):
        with torch.cuda.stream(stream):
            stage.copy_(host, non_blocking=True)
            if pool_upload is not None:
                k, v, _, _ = s.pools[i % len(s.pools)]
                k.copy_(pool_upload[0], non_blocking=True)
                v.copy_(pool_upload[1], non_blocking=True)
            kvb.paged_decode_async(cargs[i % len(cargs)], ws, wsn, raw)
            hout.copy_(gather(), non_blocking=True)

    def timed(count, pool_upload=None):
        for i in range(3):
            one(i, pool_upload)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record()
        for i in range(count):
            one(i, pool_upload)
        with torch.cuda.stream(stream):
            e1.record()
        barrier()
        t = torch.tensor([e0.elapsed_time(e1) / count], dtype=torch.float64, device=s.q.device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    pipelined = result is s.out and h2d + d2h > (1 << 20)
    if pipelined:
        # second staging buffer and output for the double-buffered loop
        stage2 = torch.empty(total, dtype=torch.uint8, device=s.q.device)
        out2 = torch.empty_like(s.out)
        q2 = stage2[:q_b].view(torch.float32).view(s.q.shape)
        lens2 = stage2[off_l:off_l + l_b].view(torch.int32)
        table2 = stage2[off_t:off_t + t_b].view(torch.int32).view(s.table.shape)
        cargs2 = [dec.args(q2, k, v, table2, lens2, s.max_len, out=out2, k_scale=ks, v_scale=vs,
                           part_tokens=part, kernel=kernel, tables_ready=True) for (k, v, ks, vs) in s.pools]
        stages, outs, slot_args = (stage, stage2), (s.out, out2), (cargs, cargs2)
        houts = (hout, torch.empty(result.shape, dtype=result.dtype, pin_memory=True))
        s_in, s_out = torch.cuda.Stream(s.q.device), torch.cuda.Stream(s.q.device)
        ev = {(kind, b): torch.cuda.Event() for kind in ("in", "k", "out") for b in (0, 1)}
        used = set()

        def step_pipelined(i):
            b = i & 1
            with torch.cuda.stream(s_in):  # inputs of step i, once step i-2's kernel has read the buffer
                if ("k", b) in used:
                    s_in.wait_event(ev[("k", b)])
                stages[b].copy_(host, non_blocking=True)
                ev[("in", b)].record(s_in)
            with torch.cuda.stream(stream):  # the kernel, once its inputs landed and step i-2's readback is done
                stream.wait_event(ev[("in", b)])
                if ("out", b) in used:
                    stream.wait_event(ev[("out", b)])
                kvb.paged_decode_async(slot_args[b][i % len(cargs)], ws, wsn, raw)
                ev[("k", b)].record(stream)
            with torch.cuda.stream(s_out):  # the result of step i
                s_out.wait_event(ev[("k", b)])
                houts[b].copy_(outs[b], non_blocking=True)
                ev[("out", b)].record(s_out)
            used.update({("k", b), ("out", b)})

        def timed_pipelined(count):
            for i in range(4):
                step_pipelined(i)
            torch.cuda.synchronize()
            barrier()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                e0.record()
            s_in.wait_stream(stream)
            s_out.wait_stream(stream)
            for i in range(count):
                step_pipelined(i)
            with torch.cuda.stream(stream):
                stream.wait_stream(s_in)
                stream.wait_stream(s_out)
                e1.record()
            torch.cuda.synchronize()
            barrier()
            t = torch.tensor([e0.elapsed_time(e1) / count], dtype=torch.float64, device=s.q.device)
            if world > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())

        ms = timed_pipelined(n)
        api = ("kvb_paged_decode_async (C ABI), host launch per step, one packed input copy and one output "
               "readback per step on their own streams, overlapped with the neighbouring steps' kernels")
    else:
        ms = timed(n)
        api = "kvb_paged_decode_async (C ABI), host launch per step, one packed input copy per step"
    e2e = {"value": round(job_bytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms, 6),
           "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": n, "api": api}
    e2e_pool = None
    if w["shard"] == "replica" or world == 1:
        k0, v0, _, _ = s.pools[0]
        pin = lambda t: torch.empty(t.shape, dtype=t.dtype, pin_memory=True).copy_(t.cpu())  # noqa: E731
        hk, hv = pin(k0), pin(v0)
        m = min(n, 20)
        ms2 = timed(m, (hk, hv))
        e2e_pool = {"value": round(job_bytes / (ms2 * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms2, 6),
                    "h2d_bytes_per_step": int(h2d + hk.numel() * hk.element_size() * 2), "d2h_bytes_per_step": int(d2h),
                    "steps": m, "note": "the whole K and V pool copied host->device every step"}
    return e2e, e2e_pool


if __name__ == "__main__":
    main()
