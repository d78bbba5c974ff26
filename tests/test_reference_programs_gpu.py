"""The reference's own test programs, unchanged, on the B200 through the drop-in.

oracle/_ref/gpu_tests and boundary_tests are the reference's tests/gpu_tests.cpp and
tests/boundary_tests.cpp compiled from its sources (oracle/Makefile) and linked with this project's
replacement for src/metal_attn.mm (kv_cache_bench_b200/csrc/metal_attn_cuda.cpp) and
libkvbcuda.so. They generate their own seeded workloads, run the reference's fp64 oracle, and
check the kernel: 846 checks (2e-5 kernel tolerance, fp16 and int8 storage bounds, per-query-head
ablation) and 2051 length-boundary checks (empty sequences, page/partition boundaries, capacity,
refusals before any device work, NaN-aware comparison). The reference published 0 failures for
both on its Metal kernel (results/make-test.txt).
"""
import os
import re
import subprocess

import pytest

pytestmark = pytest.mark.gpu
REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref")


def _run(name, timeout):
    exe = os.path.join(REF, name)
    if not os.path.exists(exe):
        pytest.skip(f"{exe} not built (the reference tree was absent at build time)")
    p = subprocess.run([exe], capture_output=True, text=True, timeout=timeout)
    return p.returncode, p.stdout + p.stderr


def test_reference_gpu_tests_pass_unchanged():
    rc, out = _run("gpu_tests", 1800)
    print(out[-2000:])
    m = re.search(r"(\d+) checks, (\d+) failed", out)
    assert rc == 0 and m and int(m.group(1)) == 846 and int(m.group(2)) == 0, out[-3000:]


def test_reference_boundary_tests_pass_unchanged():
    rc, out = _run("boundary_tests", 1800)
    print(out[-2000:])
    m = re.search(r"(\d+) checks, (\d+) failed", out)
    assert rc == 0 and m and int(m.group(1)) == 2051 and int(m.group(2)) == 0, out[-3000:]
