"""CPU-side checks of the C ABI boundary: the library loads, exports every symbol include/kvb_cuda.h
declares, and refuses bad arguments with KVB_ERR_INVALID before touching a device. No kernel is
launched here (no GPU)."""
import ctypes
import os
import re

import numpy as np
import pytest

import kv_cache_bench_b200 as kvb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    syms = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            syms |= set(re.findall(r"^\s*(?:const\s+)?\w[\w\s\*]*?\b(kvb_\w+)\s*\(", text, re.M))
    return syms


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(kvb.library_path())
    syms = declared_symbols()
    assert len(syms) >= 17, syms
    for s in sorted(syms):
        assert hasattr(lib, s), s


def test_reference_auto_part_tokens_thresholds():
    # the thresholds pinned by the reference's boundary tests (tests/boundary_tests.cpp:86-92)
    s = kvb.Shape(2, 32, 8, 128)
    want = {0: 64, 1: 64, 3968: 64, 3969: 128, 7936: 128, 7937: 256, 15872: 256, 15873: 512, 1 << 20: 512}
    for L, part in want.items():
        assert kvb.auto_part_tokens(s, L) == part


def _args(**over):
    base = dict(shape=kvb.Shape(1, 8, 2, 128), type=kvb.KvType.f16, page_size=16, max_blocks=1, max_len=1,
                part_tokens=0, num_blocks=1)
    base.update(over)
    return kvb.PagedArgs(**base)


@pytest.mark.parametrize("over,msg", [
    (dict(page_size=0), "page_size"),
    (dict(part_tokens=-1), "part_tokens"),
    (dict(max_len=-1), "max_len"),
    (dict(type=kvb.KvType.i8), "scales"),
    (dict(shape=kvb.Shape(1, 8, 2, 96)), "head_dim"),
    (dict(shape=kvb.Shape(1, 6, 4, 128)), "Hkv"),
])
def test_static_refusals_need_no_device(over, msg):
    with pytest.raises(ValueError, match=msg):
        kvb.run_paged(_args(**over))


def test_naive_refuses_int8():
    with pytest.raises(ValueError, match="f32 or f16"):
        kvb.run_naive(kvb.NaiveArgs(kvb.Shape(1, 8, 2, 128), kvb.KvType.i8, 4))


def test_workspace_layout_is_monotone_in_partitions():
    # paged_workspace_bytes needs the device's SM count only for part_tokens == 0; with an explicit
    # partition size it is pure arithmetic, but the ABI still asks the runtime for the device, so
    # without a GPU it must fail cleanly instead of crashing.
    c = kvb.device_args(kvb.Shape(1, 8, 2, 128), kvb.KvType.f16, 16, 4, 64, q=16, k=16, v=16, block_table=16,
                        seq_lens=16, out=16, num_blocks=4, part_tokens=16)
    if kvb.metal_available():
        pytest.skip("device present: covered by the GPU tests")
    with pytest.raises(RuntimeError):
        kvb.paged_workspace_bytes(c)


def test_available_is_false_without_gpu_or_true_with():
    import torch
    assert kvb.metal_available() == torch.cuda.is_available()


def test_flags_field_and_unknown_flags_refused():
    c = kvb.device_args(kvb.Shape(1, 8, 2, 128), kvb.KvType.f16, 16, 4, 64, q=16, k=16, v=16, block_table=16,
                        seq_lens=16, out=16, num_blocks=4, part_tokens=16, tables_ready=True)
    assert c.flags == kvb.FLAG_TABLES_READY
    c.flags = kvb.FLAG_TABLES_READY | 0x10
    with pytest.raises(ValueError, match="unknown flags"):
        kvb.paged_workspace_bytes(c)
    c.flags = kvb.FLAG_INPUTS_READY  # says more than FLAG_TABLES_READY, so needs it
    with pytest.raises(ValueError, match="needs KVB_FLAG_TABLES_READY"):
        kvb.paged_workspace_bytes(c)
    c = kvb.device_args(kvb.Shape(1, 8, 2, 128), kvb.KvType.f16, 16, 4, 64, q=16, k=16, v=16, block_table=16,
                        seq_lens=16, out=16, num_blocks=4, part_tokens=16, inputs_ready=True)
    assert c.flags == kvb.FLAG_TABLES_READY | kvb.FLAG_INPUTS_READY
    c.flags = kvb.FLAG_TABLES_READY | kvb.FLAG_STEP_STREAM  # a step stream is a stream of ready inputs
    with pytest.raises(ValueError, match="needs KVB_FLAG_INPUTS_READY"):
        kvb.paged_workspace_bytes(c)
    c = kvb.device_args(kvb.Shape(1, 8, 2, 128), kvb.KvType.f16, 16, 4, 64, q=16, k=16, v=16, block_table=16,
                        seq_lens=16, out=16, num_blocks=4, part_tokens=16, step_stream=True)
    assert c.flags == kvb.FLAG_TABLES_READY | kvb.FLAG_INPUTS_READY | kvb.FLAG_STEP_STREAM


def _c_layout(struct, fields):
    """sizeof and offsetof of a header struct, from a small C program compiled against the header."""
    import subprocess
    import tempfile
    src = ["#include <stdio.h>", "#include <stddef.h>", '#include "kvb_cuda.h"', "int main(void) {",
           f'  printf("%zu\\n", sizeof({struct}));']
    src += [f'  printf("%zu\\n", offsetof({struct}, {f}));' for f in fields]
    src += ["  return 0;", "}"]
    with tempfile.TemporaryDirectory() as d:
        c, exe = os.path.join(d, "layout.c"), os.path.join(d, "layout")
        with open(c, "w") as fh:
            fh.write("\n".join(src) + "\n")
        subprocess.run(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split()
    return [int(x) for x in out]


@pytest.mark.parametrize("struct,cls", [("kvb_shape", "_CShape"), ("kvb_paged_args", "_CPagedArgs"),
                                        ("kvb_naive_args", "_CNaiveArgs"), ("kvb_page_write_args", "_CPageWriteArgs"),
                                        ("kvb_ipc_handle", "_CIpcHandle"), ("kvb_peer_out", "_CPeerOut"),
                                        ("kvb_peer_barrier_args", "_CPeerBarrierArgs")])
def test_python_structs_match_the_header_layout(struct, cls):
    # the ctypes mirrors must agree with the C header field for field: a field added on one side only
    # would shift every later one
    c = getattr(kvb, cls)
    names = [f[0] for f in c._fields_]
    got = _c_layout(struct, names)
    assert got[0] == ctypes.sizeof(c), (struct, got[0], ctypes.sizeof(c))
    assert got[1:] == [getattr(c, n).offset for n in names], struct


def test_partition_helper_and_gather_refuse_before_any_device_work():
    # arguments are checked before the device is touched: these refusals need no GPU
    c = kvb.device_args(kvb.Shape(2, 32, 8, 128), kvb.KvType.f16, 16, 64, 1024, q=16, k=16, v=16, block_table=16,
                        seq_lens=16, out=16, num_blocks=4)
    with pytest.raises(ValueError):
        kvb.paged_part_tokens_for(c, [])  # no lengths for a batch of two
    with pytest.raises(ValueError):
        kvb.peer_out([], 0, 1, 1)
    bad = kvb.peer_out([16], 1, 2, 32)  # self outside the peer list
    with pytest.raises(ValueError):
        kvb.paged_decode_gather_async(c, bad, 16, 1 << 20, 0)
    with pytest.raises(ValueError):
        kvb.peer_barrier_async(kvb.peer_barrier_args(0, [16], 0), 16, 0)  # no epoch word
