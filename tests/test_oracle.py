"""The C oracle (oracle/kvb_oracle.c) against golden vectors written by the reference's own code.

Pins the oracle: for every golden case, the fp64 two-pass attention restated in C must reproduce the
reference's attention_reference output (src/reference.cpp:65-100) -- bit for bit, since it performs
the same fp64 operations in the same order -- and the int8 quantizer must reproduce the reference's
pools and scales (src/reference.cpp:32-51) exactly. Also checks the reference's known answers
(tests/cpu_tests.cpp:40-63) and storage-error bounds (tests/gpu_tests.cpp:22-62).
"""
import numpy as np
import pytest

import oracle


def _paged(c):
    return [x for x in c if "page_size" in x]


def test_golden_index_is_complete(golden):
    names = {c["name"] for c in golden}
    assert len(golden) >= 90
    for prefix in ("grid_", "naive_", "boundary_", "empty_", "contiguous_", "cfg", "known_"):
        assert any(n.startswith(prefix) for n in names), prefix


def test_oracle_paged_matches_reference_bitwise(golden):
    for c in _paged(golden):
        out = oracle.paged_attention(c["q"], c["k"], c["v"], c["block_table"], c["seq_lens"],
                                     num_kv_heads=c["num_kv_heads"], page=c["page_size"], kv_type=c["kv_type"],
                                     k_scale=c.get("k_scale"), v_scale=c.get("v_scale"), threads=3)
        assert np.array_equal(out.view(np.uint32), c["ref"].view(np.uint32)), c["name"]


def test_oracle_contiguous_matches_reference_bitwise(golden):
    for c in golden:
        if not c["name"].startswith("naive_"):
            continue
        out = oracle.contig_attention(c["q"], c["k"], c["v"], c["seq_lens"], num_kv_heads=c["num_kv_heads"],
                                      max_len=c["max_len"], kv_type=c["kv_type"], threads=2)
        assert np.array_equal(out.view(np.uint32), c["ref"].view(np.uint32)), c["name"]


def test_oracle_scatter_matches_reference(golden):
    """The fp16 pools the reference's scatter_to_paged wrote (src/reference.hpp:60-68) from its
    contiguous cache (the fp16 rounding of k32 / v32) equal oracle.scatter_paged on every live slot."""
    n = 0
    for c in golden:
        if c.get("kv_type") != oracle.F16 or "k32" not in c or "page_size" not in c:
            continue
        for src, pool_key in (("k32", "k"), ("v32", "v")):
            pool = oracle.scatter_paged(c[src].astype(np.float16), c["block_table"], c["seq_lens"],
                                        num_blocks=c["num_blocks"], page=c["page_size"])
            for b, L in enumerate(c["seq_lens"]):
                for t in range(L):
                    blk, r = c["block_table"][b, t // c["page_size"]], t % c["page_size"]
                    assert np.array_equal(pool[blk, :, r].view(np.uint16), c[pool_key][blk, :, r].view(np.uint16))
        n += 1
    assert n >= 4


def test_oracle_quantizer_matches_reference(golden):
    n = 0
    for c in golden:
        if "k_contig_f32" not in c:
            continue
        for src, pool_key, scale_key in (("k_contig_f32", "k", "k_scale"), ("v_contig_f32", "v", "v_scale")):
            pool, scales = oracle.quantize_i8(c[src], c["block_table"], c["seq_lens"], num_blocks=c["num_blocks"],
                                              page=c["page_size"])
            # only live slots are defined by the quantizer
            assert np.array_equal(scales, c[scale_key]), c["name"]
            for b, L in enumerate(c["seq_lens"]):
                for t in range(L):
                    blk = c["block_table"][b, t // c["page_size"]]
                    assert np.array_equal(pool[blk, :, t % c["page_size"]], c[pool_key][blk, :, t % c["page_size"]])
            n += 1
    assert n >= 4


def test_oracle_i8_reference_on_fp32_data_within_bound(golden):
    for c in _paged(golden):
        if c["kv_type"] != oracle.I8 or "ref_fp32_data" not in c:
            continue
        tol = oracle.i8_bound(c["q"], c["block_table"], c["seq_lens"], c["k_scale"], c["v_scale"],
                              num_kv_heads=c["num_kv_heads"], page=c["page_size"])
        assert oracle.max_abs_diff(c["ref"], c["ref_fp32_data"]) <= tol, c["name"]


def test_oracle_f16_reference_on_fp32_data_within_bound(golden):
    n = 0
    for c in _paged(golden):
        if "k32" not in c:
            continue
        tol = oracle.fp16_bound(c["q"], c["k32"], c["v32"], c["seq_lens"], num_kv_heads=c["num_kv_heads"],
                                max_len=c["max_len"])
        assert oracle.max_abs_diff(c["ref"], c["ref_fp32_data"]) <= tol, c["name"]
        n += 1
    assert n >= 2


def test_known_answers(golden):
    by = {c["name"]: c for c in golden}
    zero = by["known_zero_query_mean_of_v"]
    v = zero["v"]  # [2 blocks = sequences][Hkv][37][64]
    want = np.zeros_like(zero["ref"])
    G = zero["num_heads"] // zero["num_kv_heads"]
    for b, L in enumerate(zero["seq_lens"]):
        for h in range(zero["num_heads"]):
            want[b, h] = v[b, h // G, :L].astype(np.float64).mean(axis=0)
    assert oracle.max_abs_diff(zero["ref"], want) < 1e-6
    dom = by["known_dominant_key"]
    hot = [11, 4]
    for b in range(2):
        for h in range(dom["num_heads"]):
            assert np.array_equal(dom["ref"][b, h], dom["v"][b, h // G, hot[b]])


def test_empty_sequences_give_exactly_zero(golden):
    n = 0
    for c in _paged(golden):
        for b, L in enumerate(c["seq_lens"]):
            if L == 0:
                assert not c["ref"][b].any(), c["name"]
                n += 1
    assert n >= 10


def test_max_abs_diff_is_nan_aware():
    a = np.array([1, np.nan, 3], np.float32)
    b = np.array([1, 2, 3], np.float32)
    c = np.array([1, 2, 3.5], np.float32)
    assert oracle.max_abs_diff(a, b) == np.inf
    assert oracle.max_abs_diff(a, a) == np.inf
    assert oracle.max_abs_diff(b, c) == 0.5


@pytest.mark.parametrize("kv_type", [oracle.F32, oracle.F16, oracle.I8])
def test_synthetic_case_layout(kv_type):
    c = oracle.make_case(num_heads=8, num_kv_heads=2, head_dim=64, lens=[0, 5, 33], kv_type=kv_type, page=16,
                         seed=3, pool_slack=2.0)
    assert c.num_blocks == 2 * (0 + 1 + 3)
    used = c.table[c.table >= 0]
    assert len(set(used.tolist())) == used.size == 4
    out = c.reference(threads=2)
    assert not out[0].any() and np.isfinite(out).all()
