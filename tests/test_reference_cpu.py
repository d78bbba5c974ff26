"""The reference's own CPU tests (tests/cpu_tests.cpp, unchanged) and the CPU part of its boundary
tests, built from its sources into oracle/_ref (oracle/Makefile). Without a GPU, gpu_tests and
boundary_tests must load the drop-in and this project's library and exit 77 ("skipped") after their
host-only checks, as they do on a machine without Metal."""
import os
import subprocess

import pytest

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref")


def _exe(name):
    exe = os.path.join(REF, name)
    if not os.path.exists(exe):
        pytest.skip(f"{exe} not built (the reference tree was absent at build time)")
    return exe


def test_reference_cpu_tests():
    p = subprocess.run([_exe("cpu_tests")], capture_output=True, text=True, timeout=300)
    assert p.returncode == 0 and "9 passed, 0 failed" in p.stdout, p.stdout


@pytest.mark.parametrize("name", ["gpu_tests", "boundary_tests"])
def test_reference_gpu_programs_skip_cleanly_without_gpu(name):
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present: tests/test_reference_programs_gpu.py runs them")
    p = subprocess.run([_exe(name)], capture_output=True, text=True, timeout=300)
    assert p.returncode == 77, p.stdout + p.stderr
    assert "SKIP" in p.stdout
