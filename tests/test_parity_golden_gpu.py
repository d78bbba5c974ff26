"""CUDA path vs golden vectors written by the reference's own code (tests/golden/).

Tolerances are the reference's (tests/gpu_tests.cpp:16-62, README "Tolerances"): the kernel vs the
fp64 reference on the values it reads (stored fp32/fp16, dequantized int8) within 2e-5 absolute;
fp16 and int8 storage vs the unrounded fp32 data within the derived bounds; an empty sequence
gives exactly 0. Every case runs through each kernel that supports it (CUDA-core, TMA/tensor-core,
auto choice), several split-K partition sizes, and the per-query-head ablation (share_kv = 0).
"""
import numpy as np
import pytest

import kv_cache_bench_b200 as kvb
import oracle
from tests.cuda_runner import kernels_for, run_case, run_naive

pytestmark = pytest.mark.gpu
TOL = 2e-5


def _kernels(c, share_kv=True):
    G = c["num_heads"] // c["num_kv_heads"]
    return kernels_for(c["kv_type"], c["head_dim"], c["page_size"], G, share_kv)


def _parts(c):
    parts = {c["part_tokens"], 0}
    if c["name"].startswith("boundary_"):
        parts |= {1, 3, 4, 64}
    if c["name"].startswith(("grid_", "cfg")):
        parts |= {64, 100}
    return sorted(parts)


def test_golden_paged_within_kernel_tolerance(golden):
    failures, worst, runs = [], 0.0, 0
    for c in golden:
        if "page_size" not in c:
            continue
        G = c["num_heads"] // c["num_kv_heads"]
        for share_kv in ([True, False] if G > 1 else [True]):
            for kernel in _kernels(c, share_kv):
                for part in _parts(c):
                    out = run_case(c, part=part, kernel=kernel, share_kv=share_kv)
                    runs += 1
                    err = oracle.max_abs_diff(out, c["ref"])
                    worst = max(worst, err)
                    if not err <= TOL:
                        failures.append(f"{c['name']} kernel={kernel.name} part={part} share_kv={share_kv}: {err:.3g}")
                    for b, L in enumerate(c["seq_lens"]):
                        if L == 0 and np.any(out[b] != 0):
                            failures.append(f"{c['name']}: empty sequence {b} not exactly 0")
    print(f"{runs} runs, worst |gpu - ref| = {worst:.3g}")
    assert not failures, "\n".join(failures[:40])


def test_golden_storage_error_bounds(golden):
    failures = []
    for c in golden:
        if "page_size" not in c or "ref_fp32_data" not in c:
            continue
        if c["kv_type"] == oracle.F16:
            tol = oracle.fp16_bound(c["q"], c["k32"], c["v32"], c["seq_lens"], num_kv_heads=c["num_kv_heads"],
                                    max_len=c["max_len"])
        else:
            tol = oracle.i8_bound(c["q"], c["block_table"], c["seq_lens"], c["k_scale"], c["v_scale"],
                                  num_kv_heads=c["num_kv_heads"], page=c["page_size"])
        for kernel in _kernels(c):
            out = run_case(c, part=c["part_tokens"], kernel=kernel)
            err = oracle.max_abs_diff(out, c["ref_fp32_data"])
            if not err <= tol:
                failures.append(f"{c['name']} kernel={kernel.name}: {err:.3g} > {tol:.3g}")
    assert not failures, "\n".join(failures)


def test_golden_naive_within_kernel_tolerance(golden):
    n = 0
    for c in golden:
        if not c["name"].startswith("naive_"):
            continue
        out = run_naive(c)
        assert oracle.max_abs_diff(out, c["ref"]) <= TOL, c["name"]
        n += 1
    assert n >= 8


def test_known_answers_on_gpu(golden):
    by = {c["name"]: c for c in golden}
    for name in ("known_zero_query_mean_of_v", "known_dominant_key"):
        c = by[name]
        for kernel in (kvb.Kernel.simt, kvb.Kernel.auto):
            out = run_case(c, kernel=kernel)
            assert oracle.max_abs_diff(out, c["ref"]) <= TOL, (name, kernel)
