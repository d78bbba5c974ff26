#!/usr/bin/env python
"""Decode-step benchmark of the B200 paged decode path (one JSON line on rank 0).

Metric: decode-step microseconds and effective KV-read GB/s per GPU against the
B200 HBM peak. Effective bytes are the reference's Workload::min_bytes (src/workload.hpp:69-74): K
and V of every live token, plus q and out. ``value`` is the whole-job GB/s (sum over ranks of
bytes per step / the slowest rank's step time).

Workloads (kv_cache_bench_b200.workload; seeded synthetic data written on
the device by the library's page write path, int8 by the reference-identical quantizer):
  1  f32, 1 x 32/8 heads x 128, context 512, page 16, 64-page pool
  2  f16, context 4096, page 32, 256-page pool, split-K partition 512
  3  int8 (default; --dtype f16 for the fp16 variant), context 32768, page 128, 512-page pool  [default]
  4  f16, 64 sequences, lengths log-uniform in [512, 32768], page 16, pool 1.1 x live pages;
     sharded by sequence (LPT bin packing) across ranks
  5  f16 or int8, 256 sequences, 64/8 heads, lengths uniform in [8192, 131072], page 64;
     sharded by KV head across ranks
Configs 1-3 are single-sequence steps; with --gpus N every rank runs its own replica (weak
scaling). Inputs of configs 1-3 fit in L2 (126 MB), so each timed step reads one of R pool copies in
rotation (R * live bytes > 4 x L2); configs 4-5 are far larger than L2.

``sharded`` (on by default for the single-sequence headline): configs 4 (f16, by sequence) and 5
(int8 and f16, by KV head) measured at the same N in the same run. Each step is the decode kernel,
which writes every finished output row into every rank's global output buffer in global order over
peer memory (CUDA IPC mappings, NVLink), and a one-warp step barrier, captured together in CUDA
graphs; --gather nccl replaces the in-kernel gather by an NCCL all-gather and a reorder.

Timing: W warm-up steps, then exactly K steps between a barrier + synchronize on each side, timed
with CUDA events on the launching stream; max over ranks. Steps are CUDA-graph replays; every graph
a timed run replays is captured before the timed region, and a short GPU spin ahead of the start
event keeps host submission out of the measurement. NVML samples SM clocks and throttle reasons
during the timed region. ``e2e`` measures the same metric through the public API
(kvb_paged_decode_async) with per-step host->device copies of the step's inputs (q, sequence
lengths, block table) from pinned memory and a device->host read of the output, as a serving loop
runs it: the copies and the launch of each step captured in CUDA graphs, the copies double-buffered
on side streams; ``e2e_host_launch`` is the same with every copy and launch issued from the host
each step. The KV pool is device-resident state (written when a page is written), and
``e2e_pool_upload`` additionally copies the whole pool every step. ``parity`` compares the step's own output with the fp64 oracle (outside
the timed region). ``--impl reference`` times the reference's own CPU implementation
(oracle/_ref/kvb_ref_cpu, built from its src/reference.cpp and src/workload.hpp) on this host.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import platform
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

from kv_cache_bench_b200.workload import build_layout, config as workload, min_bytes  # noqa: E402,F401

METRIC = "decode-step µs and effective KV-read GB/s per GPU vs B200 HBM peak"
FALLBACK_HBM_GBS = 6650.0
TOL = 2e-5  # the reference's kernel tolerance against the fp64 oracle (tests/gpu_tests.cpp:16)
SPIN_CYCLES = 200_000  # ~0.1 ms of GPU spin ahead of a start event
E2E_BUFS = 2  # input staging / output buffers of the graph-captured e2e loop
STEADY_STEPS = 1000  # the longer run reported beside a short K-step run


def parse_args(argv=None):
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
    ap.add_argument("--no-step-stream", action="store_true",
                    help="leave KVB_FLAG_STEP_STREAM out of the timed steps (partitions sized for one step's "
                         "latency instead of a stream of steps)")
    ap.add_argument("--latency-reps", type=int, default=200,
                    help="single steps timed alone, each after an L2 flush (0: none)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--sharded", default="auto",
                    help="sharded configs measured after the headline: 'auto' (4:f16,5:i8,5:f16 when the headline "
                         "is a single-sequence config), 'none', or a list like 4:f16,5:i8")
    ap.add_argument("--sharded-s", type=float, default=1.5, help="timed seconds per sharded config, at most")
    ap.add_argument("--gather", choices=["kernel", "nccl"], default="kernel",
                    help="sharded steps: outputs written into every rank's buffer by the decode kernel over peer "
                         "memory, or an NCCL all-gather and a reorder")
    ap.add_argument("--ramp-s", type=float, default=1.0, help="untimed load before warm-up (clock ramp)")
    ap.add_argument("--seqs", type=int, default=None,
                    help="keep only the first N sequences of the config (a smaller case for profilers)")
    ap.add_argument("--op", choices=["decode", "quantize", "scatter"], default="decode",
                    help="decode step (default) or the page write path in front of it (one GPU)")
    return ap.parse_args(argv)


def describe(w):
    toks = sum(w["lens"])
    cut = f" (first {len(w['lens'])} sequences)" if w.get("cut") else ""
    return (f"config{w['cfg']}{cut}: {w['kv']} cache, B={len(w['lens'])}, H={w['H']}/Hkv={w['Hkv']}, D={w['D']}, "
            f"page={w['page']}, tokens={toks}, max_len={max(w['lens'])}")


def sharded_list(spec: str, headline: dict):
    """(config, dtype) pairs of the sharded block."""
    if spec == "none":
        return []
    if spec == "auto":
        return [(4, "f16"), (5, "i8"), (5, "f16")] if headline["shard"] == "replica" else []
    out = []
    for item in spec.split(","):
        c, _, d = item.partition(":")
        out.append((int(c), d or None))
    return out


# ---------------------------------------------------------------------------------------------------
# graph-replayed steps

def graph_plan(n: int, per_graph: int):
    """Sizes of the graphs a run of n steps replays, in order: whole graphs of per_graph steps, then
    one graph of the remainder."""
    full, rem = divmod(max(n, 0), per_graph)
    return [per_graph] * full + ([rem] if rem else [])


class StepRunner:
    """Runs n steps as replays of captured CUDA graphs. prepare() captures every graph the given
    step counts need; run() only replays and refuses to capture, so a timed run() holds no capture,
    instantiation or eager warm-up step."""

    def __init__(self, capture, replay, per_graph: int):
        self.capture, self.replay, self.per_graph = capture, replay, per_graph
        self.graphs = {}

    def prepare(self, *counts):
        for n in counts:
            for size in graph_plan(n, self.per_graph):
                if size not in self.graphs:
                    self.graphs[size] = self.capture(size)

    def run(self, n: int):
        for size in graph_plan(n, self.per_graph):
            g = self.graphs.get(size)
            if g is None:
                raise RuntimeError(f"graph of {size} steps was not prepared")
            self.replay(g)

    def release(self):
        self.graphs.clear()


def make_runner(torch, stream, step, per_graph: int):
    def capture(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            step(0)  # the launch path warmed outside the capture
            stream.synchronize()
            with torch.cuda.graph(g, stream=stream):
                for i in range(n):
                    step(i)
        stream.synchronize()
        return g

    def replay(g):
        with torch.cuda.stream(stream):
            g.replay()

    return StepRunner(capture, replay, per_graph)


def timed_run(torch, stream, runner, n: int):
    """Device milliseconds of runner.run(n) on `stream`: a short spin first, so the start event is
    reached only after the host has queued the replays behind it."""
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        torch.cuda._sleep(SPIN_CYCLES)
        e0.record()
    runner.run(n)
    with torch.cuda.stream(stream):
        e1.record()
    return e0, e1


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
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples),
                "window": "the last 0.25 s of the untimed load before the warm-up, the warm-up and the timed steps"}


# ---------------------------------------------------------------------------------------------------
# CPU baseline and checker (the reference's own implementation, or the oracle port when it was not
# built). Everything here runs outside the timed regions.

def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


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
    return {"value": round(nbytes / (ms * 1e-3) / 1e9, 4), "unit": "GB/s", "cores": threads, "cpu": cpu_model(),
            "kind": kind, "ms_per_step": round(ms, 3), "sample": sample, "impl": impl}


def check_sequences(torch, s, out, picks, threads):
    """max |gpu - oracle| over local sequences `picks` of DeviceStep `s`, whose output rows are
    out[i]: the fp64 oracle (oracle/kvb_oracle.c, pinned to the reference's golden vectors) on the
    very pages the kernel read, copied back from the device."""
    import oracle
    kvt = {"f32": oracle.F32, "f16": oracle.F16, "i8": oracle.I8}[s.kv]
    worst = 0.0
    for i in picks:
        q, k, v, table, lens, ks, vs = s.sequence_pages(torch, i)
        ref = oracle.paged_attention(q, k, v, table, lens, num_kv_heads=s.Hkv, page=s.page, kv_type=kvt,
                                     k_scale=ks, v_scale=vs, threads=threads)
        worst = max(worst, oracle.max_abs_diff(out[i:i + 1].cpu().numpy(), ref))
    return worst


def parity_picks(lens):
    """Local sequences to check: the shortest and the longest (one sequence: itself)."""
    if not lens:
        return []
    lo = min(range(len(lens)), key=lambda i: (lens[i], i))
    hi = max(range(len(lens)), key=lambda i: (lens[i], -i))
    return sorted({lo, hi})


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
    cb = {"value": value, "unit": "GB/s", "cores": threads, "cpu": cpu_model(), "kind": kind,
          "ms_per_step": round(ms, 3), "sample": sample, "impl": impl}
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
    steps, captured before the timed region. Single-sequence configs (1-3) with f32 or f16 storage
    (SDPA takes no int8 cache); rank 0."""
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
    stream = torch.cuda.Stream(dev)

    def step(i):
        with sdpa_kernel(be):
            F.scaled_dot_product_attention(q, ks[i % copies], vs[i % copies])

    runner = make_runner(torch, stream, step, copies * max(1, math.ceil(64 / copies)))
    runner.prepare(max(args.warmup, 3), args.steps)
    runner.run(max(args.warmup, 3))
    torch.cuda.synchronize()
    e0, e1 = timed_run(torch, stream, runner, args.steps)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    runner.release()
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
        torch.cuda._sleep(SPIN_CYCLES)
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


class Ctx:
    """Process-wide pieces of one bench run: ranks, device, barrier, max-over-ranks reduction."""

    def __init__(self, torch, dist, rank, world, device):
        self.torch, self.dist, self.rank, self.world, self.device = torch, dist, rank, world, device

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def reduce(self, x: float, op: str = "max") -> float:
        t = self.torch.tensor([float(x)], dtype=self.torch.float64, device=self.device)
        if self.world > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX if op == "max" else self.dist.ReduceOp.SUM)
        return float(t.item())


def decoder_for(ctx, s, part, kernel, step_stream):
    """PagedDecoder and per-copy C arguments over DeviceStep `s`; the workspace sized and zeroed."""
    import kv_cache_bench_b200 as kvb
    from kv_cache_bench_b200.torch_ops import PagedDecoder
    dec = PagedDecoder(ctx.device)
    # nothing in the step loop writes the lengths, the block table, q, the pools or the scales: the
    # kernel may read them while the previous step finishes; the steps are a back-to-back stream
    def make(p):
        return [dec.args(s.q, k, v, s.table, s.seq_lens, s.max_len, out=s.out, k_scale=ks, v_scale=vs,
                         part_tokens=p, kernel=kernel, tables_ready=True, inputs_ready=True, step_stream=step_stream)
                for (k, v, ks, vs) in s.pools]
    cargs = make(part)
    if part == 0 and s.lens:
        # the partition from this step's lengths, which the host knows (kvb_paged_part_tokens_for)
        cargs = make(kvb.paged_part_tokens_for(cargs[0], s.lens))
    need = max(kvb.paged_workspace_bytes(c) for c in cargs) if s.lens else 256
    dec.workspace = ctx.torch.zeros(max(need, 256), dtype=ctx.torch.uint8, device=ctx.device)
    return dec, cargs


class Gather:
    """The per-rank outputs of a sharded step put together in global order on every rank. Default
    ("kernel"): the decode kernel writes each finished row into every rank's global output buffer
    over peer memory and a step barrier follows (kv_cache_bench_b200.peer); "nccl": one NCCL
    all-gather, then a reorder (a row gather for sequence shards, a head interleave for KV-head
    shards). Nothing for replicas and for one rank."""

    def __init__(self, ctx, s, w, how="kernel"):
        from kv_cache_bench_b200 import shard as sh
        torch = ctx.torch
        self.ctx, self.s, self.w = ctx, s, w
        self.mode = None if (ctx.world == 1 or w["shard"] == "replica") else w["shard"]
        self.fused = self.mode is not None and how == "kernel"
        self.peer = None
        self.final = s.out
        G = w["H"] // w["Hkv"]
        self.h0 = s.kv_heads[0] * G if self.mode == "kv_head" else 0
        if self.fused:
            from kv_cache_bench_b200.peer import PeerGather
            rows = None
            if self.mode == "sequence":
                rows = torch.tensor(s.seqs, dtype=torch.int32, device=ctx.device)
            self.peer = PeerGather(torch, ctx.dist, ctx.rank, ctx.world, len(w["lens"]), w["H"], w["D"], ctx.device,
                                   out_head0=self.h0, out_rows=rows)
            self.final = self.peer.views[0]
        elif self.mode == "sequence":
            pad = max(len(o) for o in s.owned)
            self.local = torch.zeros((pad, s.H, w["D"]), dtype=torch.float32, device=ctx.device)
            self.gathered = torch.empty((ctx.world * pad, s.H, w["D"]), dtype=torch.float32, device=ctx.device)
            self.gidx = torch.from_numpy(sh.sequence_gather_index(s.owned, pad)).to(ctx.device)
            self.final = torch.empty((len(w["lens"]), w["H"], w["D"]), dtype=torch.float32, device=ctx.device)
        elif self.mode == "kv_head":
            self.gathered = torch.empty((ctx.world,) + tuple(s.out.shape), dtype=torch.float32, device=ctx.device)
            self.final = torch.empty((len(w["lens"]), w["H"], w["D"]), dtype=torch.float32, device=ctx.device)

    def describe(self):
        if self.mode is None:
            return "decode kernel"
        if self.fused:
            return ("decode kernel writing every output row into every rank's global buffer over peer memory "
                    "+ step barrier kernel, one CUDA graph")
        return "decode kernel + NCCL all-gather + reorder, one CUDA graph"

    def launch(self, cargs, ws, wsn, stream, i):
        """Step i on `stream` (a raw cudaStream_t): the decode and the gather. Returns the step's
        global output."""
        import kv_cache_bench_b200 as kvb
        if self.fused:
            self.final = self.peer.launch(cargs, ws, wsn, stream, i)
            return self.final
        if self.s.lens:
            kvb.paged_decode_async(cargs, ws, wsn, stream)
        return self()

    def __call__(self):
        torch, dist = self.ctx.torch, self.ctx.dist
        if self.mode == "sequence":
            self.local[: self.s.out.shape[0]].copy_(self.s.out)
            dist.all_gather_into_tensor(self.gathered, self.local)
            torch.index_select(self.gathered, 0, self.gidx, out=self.final)
        elif self.mode == "kv_head":
            dist.all_gather_into_tensor(self.gathered, self.s.out)
            self.final.copy_(self.gathered.permute(1, 0, 2, 3).reshape(self.final.shape))
        return self.final

    def global_row(self, i):
        """Row of the gathered output that holds local sequence i's heads of this rank."""
        b = self.s.seqs[i]
        if self.mode == "kv_head":
            return self.final[b, self.h0:self.h0 + self.s.H]
        return self.final[b]

    def close(self):
        if self.peer is not None:
            self.peer.close()
            self.peer = None


def measure(ctx, w, args, *, part, kernel, copies, with_clocks=None, max_seconds=None):
    """Builds DeviceStep for `w` on this rank and times K decode steps (plus the gather when
    sharded) as CUDA-graph replays. Returns a dict of the step, its pieces and the timings."""
    import kv_cache_bench_b200 as kvb
    from kv_cache_bench_b200.workload import DeviceStep
    torch = ctx.torch
    s = DeviceStep(torch, w, device=ctx.device, rank=ctx.rank, world=ctx.world, copies=copies)
    dec, cargs = decoder_for(ctx, s, part, kernel, not args.no_step_stream)
    gather = Gather(ctx, s, w, args.gather)
    stream = torch.cuda.Stream(ctx.device)
    ws_ptr, ws_n = dec.workspace.data_ptr(), dec.workspace.numel()

    def step(i):
        gather.launch(cargs[i % copies], ws_ptr, ws_n, stream.cuda_stream, i)

    if gather.mode and not gather.fused:  # the communicator is set up before any capture
        with torch.cuda.stream(stream):
            gather()
        ctx.barrier()
    # graphs of at least 64 steps (a whole number of pool rotations): consecutive launches inside a
    # graph overlap through programmatic dependent launch, launches across two replays do not
    per_graph = copies * max(1, math.ceil(64 / copies))
    runner = make_runner(torch, stream, step, per_graph)
    warm = max(args.warmup, 3)
    steps = args.steps
    runner.prepare(warm)
    ctx.barrier()
    t0 = time.time()
    runner.run(warm)
    ctx.barrier()
    if max_seconds is not None:  # bound the timed run of a long step
        per_step = ctx.reduce((time.time() - t0) / warm)
        steps = int(max(5, min(args.steps, max_seconds / max(per_step, 1e-9))))
    runner.prepare(steps)
    if with_clocks is not None and args.ramp_s > 0:  # untimed clock ramp
        runner.prepare(per_graph)
        t_end = time.time() + args.ramp_s
        while time.time() < t_end:
            # NVML samples every few ms: a short timed run (20 steps of config 3 last 0.4 ms) would see
            # none, so sampling covers the last quarter second of this continuous load as well
            if time.time() > t_end - 0.25:
                with_clocks.active(True)
            runner.run(per_graph)
            stream.synchronize()
        runner.run(warm)
    ctx.barrier()
    if with_clocks is not None:
        with_clocks.active(True)
    e0, e1 = timed_run(torch, stream, runner, steps)
    ctx.barrier()
    if with_clocks is not None:
        with_clocks.active(False)
    ms_total = ctx.reduce(e0.elapsed_time(e1))
    steady = None
    if with_clocks is not None and steps < STEADY_STEPS:
        # consecutive steps overlap, so a short run pays one pipeline fill and drain: the same steps
        # over a longer run, reported beside the K-step figure
        runner.prepare(STEADY_STEPS)
        ctx.barrier()
        f0, f1 = timed_run(torch, stream, runner, STEADY_STEPS)
        ctx.barrier()
        steady = ctx.reduce(f0.elapsed_time(f1)) / STEADY_STEPS
    flag = dec.error_flag(stream) if s.lens else 0
    runner.release()
    if gather.fused:
        # outside the timing: the local output of a plain launch (the parity check reads it) and one
        # gathered step into the first buffer, complete on every rank
        with torch.cuda.stream(stream):
            if s.lens:
                kvb.paged_decode_async(cargs[0], ws_ptr, ws_n, stream.cuda_stream)
            gather.launch(cargs[0], ws_ptr, ws_n, stream.cuda_stream, 0)
        ctx.barrier()
        flag = max(flag, dec.error_flag(stream) if s.lens else 0)
    decode_ms = None
    if gather.mode is not None:
        # each rank's decode alone (its share of the step, no gather), timed the same way; every rank
        # takes the same barriers and reductions, with or without sequences of its own
        def plain(i):
            kvb.paged_decode_async(cargs[i % copies], ws_ptr, ws_n, stream.cuda_stream)
        n2 = max(5, min(steps, 200))
        alone = make_runner(torch, stream, plain, per_graph) if s.lens else None
        if alone:
            alone.prepare(n2)
        ctx.barrier()
        if alone:
            k0, k1 = timed_run(torch, stream, alone, n2)
        ctx.barrier()
        mine = k0.elapsed_time(k1) / n2 if alone else 0.0
        if alone:
            alone.release()
        decode_ms = (ctx.reduce(mine), -ctx.reduce(-mine))
    ms_step = ms_total / max(steps, 1)
    job_bytes = ctx.reduce(s.bytes, "sum")
    return dict(s=s, dec=dec, gather=gather, stream=stream, ms_step=ms_step, steps=steps, job_bytes=job_bytes,
                steady_ms_step=steady, decode_ms=decode_ms,
                flag=int(ctx.reduce(flag)), part=kvb.paged_part_tokens(cargs[0]) if s.lens else part,
                copies=copies)


def measure_latency(ctx, m, part, kernel, reps):
    """One decode step with nothing in flight, as the reference times a run (its command buffer's GPU
    time, caches flushed before every run): each step follows an L2 flush (a 256 MiB device write) and
    is timed alone by events around its launch, without flags (partitions by the latency rule, every
    read after the programmatic-launch wait). Median and minimum over `reps`, max over ranks."""
    import kv_cache_bench_b200 as kvb
    torch = ctx.torch
    s, dec, stream = m["s"], m["dec"], m["stream"]
    cargs = [dec.args(s.q, k, v, s.table, s.seq_lens, s.max_len, out=s.out, k_scale=ks, v_scale=vs,
                      part_tokens=part, kernel=kernel) for (k, v, ks, vs) in s.pools]
    need = max(kvb.paged_workspace_bytes(c) for c in cargs)
    if need > dec.workspace.numel():
        dec.workspace = torch.zeros(need, dtype=torch.uint8, device=ctx.device)
    ws, wsn = dec.workspace.data_ptr(), dec.workspace.numel()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=ctx.device)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    with torch.cuda.stream(stream):
        for i in range(3):  # warm the launch path
            kvb.paged_decode_async(cargs[i % len(cargs)], ws, wsn, stream.cuda_stream)
        for i, (e0, e1) in enumerate(ev):
            flush.fill_(i & 0xff)
            e0.record(stream)
            kvb.paged_decode_async(cargs[i % len(cargs)], ws, wsn, stream.cuda_stream)
            e1.record(stream)
    stream.synchronize()
    us = sorted(e0.elapsed_time(e1) * 1e3 for e0, e1 in ev)
    med = ctx.reduce(us[len(us) // 2])
    return {"us": round(med, 3), "min_us": round(ctx.reduce(us[0]), 3), "reps": reps,
            "gbps": round(s.bytes / (med * 1e-6) / 1e9, 2), "part_tokens": kvb.paged_part_tokens(cargs[0]),
            "flags": "none", "l2": "256 MiB device write before each step",
            "note": "one step with nothing in flight (the reference's per-run GPU time); value is the "
                    "throughput of back-to-back steps"}


def sharded_parity(ctx, m, threads):
    """Each rank checks its shortest and longest local sequences against the fp64 oracle, and that the
    gathered global output holds its rows unchanged; the worst error over ranks."""
    torch = ctx.torch
    s, gather = m["s"], m["gather"]
    picks = parity_picks(s.lens)
    err = check_sequences(torch, s, s.out, picks, threads) if picks else 0.0
    same = all(torch.equal(gather.global_row(i), s.out[i]) for i in picks)
    err = ctx.reduce(err)
    moved = ctx.reduce(0.0 if same else 1.0)
    return {"max_abs": err, "tol": TOL, "gather_exact": moved == 0.0, "ok": err <= TOL and moved == 0.0,
            "checked": f"shortest and longest sequence of each rank ({len(picks)} per rank), fp64 oracle on the pages "
                       "the kernel read"}


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
    ctx = Ctx(torch, dist, rank, world, device)
    threads = max(1, (os.cpu_count() or 1) // world)

    # pool copies so that the data a step reads cycles through more than 4 x L2
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    elem = {"f32": 4, "f16": 2, "i8": 1}[w["kv"]]
    live_est = float(sum(w["lens"])) * w["Hkv"] * w["D"] * 2 * elem / (world if w["shard"] != "replica" else 1)
    copies = max(1, min(64, math.ceil(4 * l2 / max(live_est, 1)))) if w["shard"] == "replica" else 1
    kernel = {"auto": kvb.Kernel.auto, "simt": kvb.Kernel.simt, "mma": kvb.Kernel.mma,
              "umma": kvb.Kernel.umma}[args.kernel]
    part = w["part"] if args.part is None else args.part

    try:  # NVML numbers devices physically; map through CUDA_VISIBLE_DEVICES
        nvml_index = torch.cuda._get_nvml_device_index(local)
    except Exception:  # noqa: BLE001
        nvml_index = local
    clocks = ClockSampler(nvml_index)
    clocks.start()
    m = measure(ctx, w, args, part=part, kernel=kernel, copies=copies, with_clocks=clocks)
    clocks.stop()
    s, dec = m["s"], m["dec"]
    ms_step, job_bytes, steady_ms = m["ms_step"], m["job_bytes"], m["steady_ms_step"]
    value = job_bytes / (ms_step * 1e-3) / 1e9
    latency = None
    if args.latency_reps > 0 and w["shard"] == "replica" and s.lens:
        latency = measure_latency(ctx, m, part, kernel, args.latency_reps)

    # end to end through the public API with host buffers
    e2e = e2e_pool = e2e_launch = e2e_copy = None
    if not args.no_e2e:
        e2e_launch, e2e_pool = measure_e2e(torch, dist, s, dec, part, kernel, m["stream"], args, world, ctx.barrier,
                                           job_bytes, w, m["gather"])
        e2e = e2e_launch
        if m["gather"].mode is None:
            e2e_copy = measure_e2e_graph(torch, dist, s, dec, part, kernel, args, world, ctx.barrier, job_bytes)
            e2e = measure_e2e_mapped(torch, dist, s, dec, part, kernel, args, world, ctx.barrier, job_bytes,
                                     not args.no_step_stream)

    # parity of the step's own output (the checker, outside every timed region)
    parity = None
    if not args.no_parity:
        if w["shard"] == "replica":
            err = ctx.reduce(check_sequences(torch, s, s.out, parity_picks(s.lens), threads))
            parity = {"max_abs": err, "tol": TOL, "ok": err <= TOL,
                      "checked": "every sequence of the step, fp64 oracle on the pages the kernel read"}
        else:
            parity = sharded_parity(ctx, m, threads)

    cb = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cb = cpu_baseline(w)
        except Exception as ex:  # noqa: BLE001
            cb = {"value": None, "error": str(ex)[:200]}
    per_gpu = s.bytes / (ms_step * 1e-3) / 1e9
    part_used, flag = m["part"], m["flag"]
    m["gather"].close()
    del m, s, dec
    torch.cuda.empty_cache()

    # the sharded configs at the same N
    sharded = {}
    peak, peak_kind = peak_hbm()
    for cfg, dt in sharded_list(args.sharded, w):
        ws = workload(cfg, dt)
        ms_ = measure(ctx, ws, args, part=ws["part"], kernel=kernel, copies=1, max_seconds=args.sharded_s)
        entry = {"workload": describe(ws), "parallelism": config_obj(ws, None, world)["parallelism"],
                 "us_per_step": round(ms_["ms_step"] * 1e3, 3), "steps": ms_["steps"],
                 "value": round(ms_["job_bytes"] / (ms_["ms_step"] * 1e-3) / 1e9, 2), "unit": "GB/s",
                 "frac_of_n_peak": round(ms_["job_bytes"] / (ms_["ms_step"] * 1e-3) / 1e9 / (world * peak), 4),
                 "part_tokens": ms_["part"], "error_flag": ms_["flag"],
                 "step": ms_["gather"].describe()}
        if ms_["decode_ms"]:
            entry["decode_us_per_rank"] = {"max": round(ms_["decode_ms"][0] * 1e3, 3),
                                           "min": round(ms_["decode_ms"][1] * 1e3, 3),
                                           "note": "each rank's decode alone, without the gather, back to back"}
        if not args.no_parity:
            entry["parity"] = sharded_parity(ctx, ms_, threads)
        sharded[f"config{cfg}_{ws['kv']}"] = entry
        ms_["gather"].close()
        del ms_
        torch.cuda.empty_cache()

    if rank == 0:
        traffic = read_traffic(w)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 6), "us_per_step": round(ms_step * 1e3, 3),
            "gbps_per_gpu": round(per_gpu, 2), "higher_is_better": True,
            "scaling": "weak" if w["shard"] == "replica" else "strong", "vs_baseline": None, "dtype": w["kv"],
            "data": "synthetic: seeded U(-1,1) q and fp32 K/V generated on the device"
                    + ("; int8 by the device quantizer (bit-identical to the reference's quantize_to_paged_i8)"
                       if w["kv"] == "i8" else ""),
            "config": dict(config_obj(w, part_used, world),
                           l2=(f"{copies} rotating pool copies ({copies * live_est / 1e6:.0f} MB live "
                               f"> 4 x L2 {l2 / 1e6:.0f} MB)" if copies > 1 else
                               f"inputs {live_est / 1e6:.0f} MB per GPU > L2 {l2 / 1e6:.0f} MB"),
                           submission="cuda graph replay, graphs captured before the timed region",
                           flags="TABLES_READY|INPUTS_READY" + ("" if args.no_step_stream else "|STEP_STREAM"),
                           kernel=args.kernel),
            "roofline": {"bound": "hbm", "achieved": round(per_gpu, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(per_gpu / peak, 4), "peak_kind": peak_kind,
                         "traffic": traffic, "algorithmic_bytes_per_launch": min_bytes(w, w["lens"], w["Hkv"], w["H"]),
                         "note": "achieved = min_bytes per launch / device time per step (one decode kernel "
                                 "per step); peak = measured copy bandwidth"},
            "gpu_launches": args.steps, "error_flag": flag, "clocks": clocks.summary(),
        }
        if parity:
            line["parity"] = parity
        if steady_ms is not None:
            line["steady"] = {"us_per_step": round(steady_ms * 1e3, 3), "steps": STEADY_STEPS,
                              "value": round(job_bytes / (steady_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                              "note": "the same back-to-back steps over a longer run; a K-step run includes one "
                                      "fill and drain of the steps in flight"}
        if latency:
            line["latency"] = latency
        if e2e:
            line["e2e"] = e2e
        if e2e_copy:
            line["e2e_copy_engine"] = e2e_copy
        if e2e_launch and e2e_launch is not e2e:
            line["e2e_host_launch"] = e2e_launch
        if e2e_pool:
            line["e2e_pool_upload"] = e2e_pool
        if cb:
            line["cpu_baseline"] = cb
        if sharded:
            line["sharded"] = sharded
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def measure_e2e_graph(torch, dist, s, dec, part, kernel, args, world, barrier, job_bytes):
    """End to end as a serving loop runs decode steps: CUDA graphs of 64 steps, each step a
    host->device copy of its inputs (q, sequence lengths, block table, one packed pinned buffer), the
    kvb_paged_decode_async launch reading them where they landed, and the device->host copy of its
    output into pinned memory. E2E_BUFS staging and output buffers rotate; the input copies run on
    one side stream and the readbacks on another, so later steps' inputs land and earlier steps'
    outputs leave while a step's kernel runs (graph edges keep every buffer's writer after its last
    reader). Every timed step copies its inputs in and its output out. Replicas and one rank only.

    The launches leave out KVB_FLAG_STEP_STREAM: a kernel node that also waits for a copy does not
    start early behind the previous kernel, so the steps of this loop do not overlap, and the latency
    rule's partitions serve it better (config 3 int8: 24.3 µs per step against 37.7 with the step
    stream's, four buffers)."""
    import kv_cache_bench_b200 as kvb

    def align(n):
        return (n + 255) // 256 * 256

    nb = E2E_BUFS
    dev = s.q.device
    q_b, l_b, t_b = s.q.numel() * 4, s.seq_lens.numel() * 4, s.table.numel() * 4
    off_l = align(q_b)
    off_t = off_l + align(l_b)
    total = off_t + t_b
    host = torch.empty(total, dtype=torch.uint8, pin_memory=True)
    host[:q_b].copy_(s.q.cpu().view(-1).view(torch.uint8))
    host[off_l:off_l + l_b].copy_(s.seq_lens.cpu().view(-1).view(torch.uint8))
    host[off_t:off_t + t_b].copy_(s.table.cpu().view(-1).view(torch.uint8))
    stages = [torch.empty(total, dtype=torch.uint8, device=dev) for _ in range(nb)]
    outs = [torch.empty_like(s.out) for _ in range(nb)]
    houts = [torch.empty(s.out.shape, dtype=s.out.dtype, pin_memory=True) for _ in range(nb)]
    cargs = []
    for b in range(nb):
        st = stages[b]
        q = st[:q_b].view(torch.float32).view(s.q.shape)
        lens = st[off_l:off_l + l_b].view(torch.int32)
        table = st[off_t:off_t + t_b].view(torch.int32).view(s.table.shape)
        cargs.append([dec.args(q, k, v, table, lens, s.max_len, out=outs[b], k_scale=ks, v_scale=vs,
                               part_tokens=part, kernel=kernel, tables_ready=True, inputs_ready=True)
                      for (k, v, ks, vs) in s.pools])
    need = max(kvb.paged_workspace_bytes(c) for c in cargs[0])
    if need > dec.workspace.numel():
        dec.workspace = torch.zeros(need, dtype=torch.uint8, device=dev)
    ws, wsn = dec.workspace.data_ptr(), dec.workspace.numel()
    stream, s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    copies = len(s.pools)
    unit = copies * nb // math.gcd(copies, nb)  # whole pool rotations and buffer rounds per graph
    per_graph = unit * max(1, math.ceil(64 / unit))

    def capture(n):
        with torch.cuda.stream(stream):  # warm the launch path outside the capture
            kvb.paged_decode_async(cargs[0][0], ws, wsn, stream.cuda_stream)
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        ev_in = [torch.cuda.Event() for _ in range(n)]
        ev_k = [torch.cuda.Event() for _ in range(n)]
        ev_out = [torch.cuda.Event() for _ in range(n)]
        with torch.cuda.graph(g, stream=stream):
            s_in.wait_stream(stream)
            s_out.wait_stream(stream)
            for i in range(n):
                b = i % nb
                with torch.cuda.stream(s_in):  # step i's inputs, once the buffer's previous kernel read it
                    if i >= nb:
                        s_in.wait_event(ev_k[i - nb])
                    stages[b].copy_(host, non_blocking=True)
                    ev_in[i].record(s_in)
                stream.wait_event(ev_in[i])
                if i >= nb:  # the readback of this output buffer's previous step is done
                    stream.wait_event(ev_out[i - nb])
                kvb.paged_decode_async(cargs[b][i % copies], ws, wsn, stream.cuda_stream)
                ev_k[i].record(stream)
                with torch.cuda.stream(s_out):  # step i's output
                    s_out.wait_event(ev_k[i])
                    houts[b].copy_(outs[b], non_blocking=True)
                    ev_out[i].record(s_out)
            stream.wait_stream(s_in)
            stream.wait_stream(s_out)
        stream.synchronize()
        return g

    def replay(g):
        with torch.cuda.stream(stream):
            g.replay()

    runner = StepRunner(capture, replay, per_graph)
    n = max(args.steps, 1)
    runner.prepare(per_graph, n)
    runner.run(per_graph)
    barrier()
    e0, e1 = timed_run(torch, stream, runner, n)
    barrier()
    t = torch.tensor([e0.elapsed_time(e1) / n], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    last = graph_plan(n, per_graph)[-1] - 1  # the last step of the last replayed graph
    ok = torch.equal(houts[last % nb], outs[last % nb].cpu())
    runner.release()
    return {"value": round(job_bytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms, 6),
            "h2d_bytes_per_step": int(total), "d2h_bytes_per_step": int(houts[0].numel() * 4), "steps": n,
            "readback_matches_device": bool(ok),
            "api": "kvb_paged_decode_async (C ABI) in CUDA graphs of %d steps: per step one packed pinned "
                   "host->device input copy, the launch, one device->pinned host output copy; copies on two "
                   "side streams, %d rotating buffers" % (per_graph, nb)}


def measure_e2e_mapped(torch, dist, s, dec, part, kernel, args, world, barrier, job_bytes, step_stream):
    """End to end with the step's inputs and output in pinned host memory, used in place: q, the
    sequence lengths and the block table live in page-locked host buffers, and the output goes
    into one. kvb_paged_decode_async is given those host pointers (the device reaches page-locked
    memory at the same address), so every step's kernel reads its inputs from host memory across the
    host link and writes its result there, inside the timed region; no copy-engine copy sits between
    two steps, and consecutive steps overlap as they do on device buffers (flags as the device
    timing: TABLES_READY | INPUTS_READY, and STEP_STREAM unless turned off). This is how the
    reference's own path reaches its inputs: its buffers are shared storage that the GPU reads where
    the host wrote them. The KV pool and its scales are device-resident state, rotated over the same
    copies as the device timing. Replicas and one rank only."""
    import kv_cache_bench_b200 as kvb

    hq = s.q.cpu().pin_memory()
    hl = s.seq_lens.cpu().pin_memory()
    ht = s.table.cpu().pin_memory()
    hout = torch.zeros(s.out.shape, dtype=s.out.dtype).pin_memory()
    B, H, D = s.q.shape
    num_blocks, Hkv, page, _ = s.pools[0][0].shape
    kvt = {torch.int8: kvb.KvType.i8, torch.float16: kvb.KvType.f16,
           torch.float32: kvb.KvType.f32}[s.pools[0][0].dtype]
    cargs = [kvb.device_args(kvb.Shape(B, H, Hkv, D), kvt, page, s.table.shape[1], int(s.max_len),
                             q=hq.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), block_table=ht.data_ptr(),
                             seq_lens=hl.data_ptr(), out=hout.data_ptr(), num_blocks=num_blocks, part_tokens=part,
                             k_scale=ks.data_ptr() if ks is not None else 0,
                             v_scale=vs.data_ptr() if vs is not None else 0, kernel=kernel,
                             tables_ready=True, inputs_ready=True, step_stream=step_stream)
             for (k, v, ks, vs) in s.pools]
    need = max(kvb.paged_workspace_bytes(c) for c in cargs)
    if need > dec.workspace.numel():
        dec.workspace = torch.zeros(need, dtype=torch.uint8, device=s.q.device)
    ws, wsn = dec.workspace.data_ptr(), dec.workspace.numel()
    stream = torch.cuda.Stream(s.q.device)
    copies = len(cargs)

    def step(i):
        kvb.paged_decode_async(cargs[i % copies], ws, wsn, stream.cuda_stream)

    per_graph = copies * max(1, math.ceil(64 / copies))
    runner = make_runner(torch, stream, step, per_graph)
    n = max(args.steps, 1)
    runner.prepare(per_graph, n)
    runner.run(per_graph)
    barrier()
    e0, e1 = timed_run(torch, stream, runner, n)
    barrier()
    t = torch.tensor([e0.elapsed_time(e1) / n], dtype=torch.float64, device=s.q.device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    flag = dec.error_flag(stream)
    runner.release()
    # the same launch on device buffers (every pool copy holds the same pages)
    k, v, ks, vs = s.pools[0]
    dout = torch.empty_like(s.out)
    dev_args = dec.args(s.q, k, v, s.table, s.seq_lens, s.max_len, out=dout, k_scale=ks, v_scale=vs, part_tokens=part,
                        kernel=kernel, tables_ready=True, inputs_ready=True, step_stream=step_stream)
    kvb.paged_decode_async(dev_args, ws, wsn, stream.cuda_stream)
    stream.synchronize()
    ok = torch.equal(hout, dout.cpu())
    in_bytes = hq.numel() * 4 + hl.numel() * 4 + ht.numel() * 4
    return {"value": round(job_bytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms, 6),
            "h2d_bytes_per_step": int(in_bytes), "d2h_bytes_per_step": int(hout.numel() * 4), "steps": n,
            "readback_matches_device": bool(ok), "error_flag": flag,
            "api": "kvb_paged_decode_async (C ABI) in CUDA graphs of %d steps, q, sequence lengths and block "
                   "table read by the kernel from pinned host memory and the output written into pinned host "
                   "memory every step (no staging copies)%s" % (per_graph, ", step stream" if step_stream else "")}


def measure_e2e(torch, dist, s, dec, part, kernel, stream, args, world, barrier, job_bytes, w, gather):
    """The same metric through the public C ABI with host buffers: per step, one host->device copy
    of the step's inputs (q, sequence lengths, block table, packed in one pinned staging buffer),
    kvb_paged_decode_async reading them where they landed (the in-kernel gather and the step barrier,
    or the NCCL all-gather, when sharded), and the device->host copy of the (global) output. The KV pool is device-resident state (written when a
    page is written), rotated over the same copies as the device timing.

    Unsharded steps that move more than 1 MiB of inputs and outputs are pipelined as a serving loop
    would run them: two staging and two output buffers, the input copy of step i+1 and the readback of
    step i-1 on their own streams while step i's kernel runs (events keep each buffer's writer after its
    last reader). Every step still copies its inputs in and its output out inside the timed region.
    Smaller steps (configs 1-3) run on one stream: there the cross-stream event handoffs cost more
    than the copies they would hide (config 3: 49 us pipelined against 39 us). Sharded runs keep one
    stream too (the gather sits between kernel and readback)."""
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
    result = gather.final if gather.fused else gather()
    torch.cuda.synchronize()
    hout = torch.empty(result.shape, dtype=result.dtype, pin_memory=True)
    # the inputs arrive by host copy each step (no kernel writes them)
    cargs = [dec.args(q, k, v, table, lens, s.max_len, out=s.out, k_scale=ks, v_scale=vs, part_tokens=part,
                      kernel=kernel, tables_ready=True, inputs_ready=True) for (k, v, ks, vs) in s.pools]
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
            hout.copy_(gather.launch(cargs[i % len(cargs)], ws, wsn, raw, i), non_blocking=True)

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
                           part_tokens=part, kernel=kernel, tables_ready=True, inputs_ready=True)
                 for (k, v, ks, vs) in s.pools]
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
