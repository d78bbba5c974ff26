"""bench.py's host-side pieces on the CPU: the workloads (BASELINE.json's five configs), the
algorithmic byte count (the reference's Workload::min_bytes, src/workload.hpp:69-74), the seeded
layouts, the bounded CPU samples, and the reference arm's JSON line (it needs no GPU)."""
import json
import math
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def test_workloads_match_the_configs():
    w1, w2, w3, w4, w5 = (bench.workload(c, None) for c in range(1, 6))
    assert (w1["kv"], w1["lens"], w1["page"], w1["pool_blocks"]) == ("f32", [512], 16, 64)
    assert (w2["kv"], w2["lens"], w2["page"], w2["pool_blocks"], w2["part"]) == ("f16", [4096], 32, 256, 512)
    assert (w3["kv"], w3["lens"], w3["page"], w3["pool_blocks"]) == ("i8", [32768], 128, 512)
    assert len(w4["lens"]) == 64 and 512 <= min(w4["lens"]) and max(w4["lens"]) <= 32768 and w4["page"] == 16
    assert len(w5["lens"]) == 256 and 8192 <= min(w5["lens"]) and max(w5["lens"]) <= 131072
    assert (w5["H"], w5["Hkv"], w5["page"]) == (64, 8, 64)
    assert bench.workload(3, "f16")["kv"] == "f16"


def test_min_bytes_is_the_references_count():
    w = bench.workload(3, None)
    assert bench.min_bytes(w, w["lens"], w["Hkv"], w["H"]) == 67_141_632
    w = bench.workload(3, "f16")
    assert bench.min_bytes(w, w["lens"], w["Hkv"], w["H"]) == 134_250_496
    w = bench.workload(1, None)
    assert bench.min_bytes(w, w["lens"], w["Hkv"], w["H"]) == 4_227_072
    w = bench.workload(2, None)
    assert bench.min_bytes(w, w["lens"], w["Hkv"], w["H"]) == 16_809_984


def test_layout_gives_each_sequence_distinct_blocks():
    rng = np.random.default_rng(4)
    lens = [100, 0, 17, 64]
    table, nb = bench.build_layout(lens, 16, 1.1, None, rng)
    live = [b for i, l in enumerate(lens) for b in table[i, : math.ceil(l / 16)]]
    assert len(set(live)) == len(live) and all(0 <= b < nb for b in live)
    assert (table[1] == -1).all()


def test_sample_lens_cuts_a_prefix():
    w = dict(lens=[300, 200, 100])
    assert bench.sample_lens(w, 10_000) == [300, 200, 100]
    assert bench.sample_lens(w, 450) == [300, 150]
    assert bench.sample_lens(w, 1) == [1]


@pytest.mark.skipif(not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "kvb_ref_cpu")),
                    reason="the reference's CPU timer was not built")
def test_reference_arm_prints_the_contract_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--config", "1",
                          "--steps", "3", "--warmup", "1"], check=True, capture_output=True, text=True, timeout=300)
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0 and line["unit"] == "GB/s"
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["cpu_baseline"]["kind"] == "reference" and line["cpu_baseline"]["cores"] >= 1
    assert line["metric"] == bench.METRIC and line["higher_is_better"] is True


def test_sdpa_arm_refuses_batched_and_int8_configs():
    # torch SDPA takes neither a block table nor an int8 cache: batched and int8 configs print the
    # contract's `unavailable` line (this path needs no GPU)
    for extra in (["--config", "4"], ["--config", "3"]):
        out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "torch-sdpa"] + extra,
                             check=True, capture_output=True, text=True, timeout=300)
        line = json.loads(out.stdout.strip().splitlines()[-1])
        assert line["impl"] == "torch-sdpa" and "unavailable" in line


def test_sequence_cap_names_the_cut():
    w = bench.workload(5, "i8")
    w["lens"], w["cut"] = w["lens"][:16], True
    assert "first 16 sequences" in bench.describe(w) and "B=16" in bench.describe(w)


@pytest.mark.parametrize("steps,warmup", [(20, 5), (2000, 20), (64, 0), (1, 3), (65, 64)])
def test_timed_run_replays_only_prepared_graphs(steps, warmup):
    """bench.py times K steps as replays of graphs captured beforehand: once prepare() has seen the
    warm-up and step counts, run() of either count captures nothing (a capture inside the timed
    region would time instantiation and an eager step along with the decode)."""
    captured, replayed = [], []
    runner = bench.StepRunner(capture=lambda n: captured.append(n) or ("graph", n),
                              replay=lambda g: replayed.append(g[1]), per_graph=64)
    runner.prepare(max(warmup, 3), steps)
    before = list(captured)
    runner.run(max(warmup, 3))
    runner.run(steps)
    assert captured == before  # nothing captured while running
    assert sum(replayed) == max(warmup, 3) + steps
    assert all(n <= 64 for n in replayed)


def test_unprepared_run_refuses_to_capture():
    runner = bench.StepRunner(capture=lambda n: n, replay=lambda g: None, per_graph=64)
    runner.prepare(64)
    with pytest.raises(RuntimeError, match="not prepared"):
        runner.run(20)


def test_graph_plan_covers_the_count():
    for n in (0, 1, 63, 64, 65, 2000):
        plan = bench.graph_plan(n, 64)
        assert sum(plan) == n and all(0 < k <= 64 for k in plan)


def test_sharded_block_configs():
    assert bench.sharded_list("auto", bench.workload(3, None)) == [(4, "f16"), (5, "i8"), (5, "f16")]
    assert bench.sharded_list("auto", bench.workload(4, None)) == []
    assert bench.sharded_list("none", bench.workload(3, None)) == []
    assert bench.sharded_list("5:i8", bench.workload(3, None)) == [(5, "i8")]


def test_parity_picks_shortest_and_longest():
    assert bench.parity_picks([]) == []
    assert bench.parity_picks([7]) == [0]
    assert bench.parity_picks([5, 9, 1, 9]) == [1, 2]


def test_gather_defaults_to_the_kernel_and_is_idle_on_one_rank():
    import types
    import torch
    assert bench.parse_args([]).gather == "kernel"
    assert bench.parse_args(["--gather", "nccl"]).gather == "nccl"
    with pytest.raises(SystemExit):
        bench.parse_args(["--gather", "allreduce"])
    ctx = types.SimpleNamespace(torch=torch, dist=None, rank=0, world=1, device=torch.device("cpu"))
    s = types.SimpleNamespace(out=torch.zeros(1, 4, 8), kv_heads=[0, 1], seqs=[0], lens=[5], H=4)
    for cfg in (3, 4, 5):
        g = bench.Gather(ctx, s, bench.workload(cfg, None))
        assert g.mode is None and not g.fused and g.peer is None and g.final is s.out
        assert g.describe() == "decode kernel" and g() is s.out
        g.close()
