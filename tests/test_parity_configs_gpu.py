"""Parity at the configurations bench.py measures, on the very data it measures.

Each test builds the step with kv_cache_bench_b200.workload.DeviceStep (the code path bench.py uses:
fp32 K/V generated on the device, fp16 by rounding, int8 by the device quantizer that is
bit-identical to the reference's quantize_to_paged_i8), runs one decode step through
kvb_paged_decode_async as bench.py does (automatic partition, tables-ready flag), and compares with
the fp64 oracle on the pages the kernel read, copied back per sequence (configs 4 and 5 are checked
one sequence at a time, as the reference's attention_reference cannot hold config 5 whole).

Tolerances (tests/gpu_tests.cpp:16-62): 2e-5 absolute on the stored (fp16) or dequantized (int8)
values; the fp16 / int8 storage bounds against the unrounded fp32 data. BASELINE.json's fp32 bar:
every output vector within 1e-5 relative to its largest element.
"""
import numpy as np
import pytest
import torch

import kv_cache_bench_b200 as kvb
import oracle
from kv_cache_bench_b200.torch_ops import PagedDecoder
from kv_cache_bench_b200.workload import DeviceStep, config

pytestmark = pytest.mark.gpu
TOL = 2e-5      # kernel vs fp64 oracle on the stored / dequantized values
REL32 = 1e-5    # fp32 cache: relative to the largest element of each output vector
KVT = {"f32": oracle.F32, "f16": oracle.F16, "i8": oracle.I8}


def _decode(s: DeviceStep):
    dec = PagedDecoder(s.device)
    k, v, ks, vs = s.pools[0]
    s.out.fill_(float("nan"))
    dec(s.q, k, v, s.table, s.seq_lens, s.max_len, k_scale=ks, v_scale=vs, out=s.out,
        part_tokens=s.w["part"], tables_ready=True)
    torch.cuda.synchronize()
    assert dec.error_flag() == 0
    return dec


def _oracle(s: DeviceStep, i: int):
    q, k, v, table, lens, ks, vs = s.sequence_pages(torch, i)
    return oracle.paged_attention(q, k, v, table, lens, num_kv_heads=s.Hkv, page=s.page, kv_type=KVT[s.kv],
                                  k_scale=ks, v_scale=vs), (q, table, lens, ks, vs)


def _storage_bound_check(s: DeviceStep, i: int, inputs):
    """The step's output for sequence i against the fp64 oracle on the unrounded fp32 data, within
    the reference's derived fp16 / int8 storage bound."""
    q, table, lens, ks, vs = inputs
    k32, v32 = s.sequence_fp32(torch, i)
    L = int(lens[0])
    ref32 = oracle.contig_attention(q, k32, v32, lens, num_kv_heads=s.Hkv, max_len=L, kv_type=oracle.F32)
    if s.kv == "f16":
        bound = oracle.fp16_bound(q, k32, v32, lens, num_kv_heads=s.Hkv, max_len=L)
    else:
        bound = oracle.i8_bound(q, table, lens, ks, vs, num_kv_heads=s.Hkv, page=s.page)
    err = oracle.max_abs_diff(s.out[i:i + 1].cpu().numpy(), ref32)
    assert err <= bound, f"sequence {s.seqs[i]}: {err:.3g} > storage bound {bound:.3g}"
    return err, bound


def _free(s):
    s.pools.clear()
    torch.cuda.empty_cache()


@pytest.mark.parametrize("dtype", ["i8", "f16"])
def test_config3_full_size(dtype):
    """32768 tokens, page 128, 512-page shuffled pool, the automatic B200 partition (1920 tokens: 18
    partitions x 8 KV heads = 144 units on 148 SMs)."""
    s = DeviceStep(torch, config(3, dtype), device=torch.device("cuda", 0))
    assert s.num_blocks == 512 and s.lens == [32768]
    dec = _decode(s)
    k, v, ks, vs = s.pools[0]
    part = dec.part_tokens(s.q, k, v, s.table, s.seq_lens, s.max_len, k_scale=ks, v_scale=vs, tables_ready=True)
    assert part == 1920
    ref, inputs = _oracle(s, 0)
    err = oracle.max_abs_diff(s.out.cpu().numpy(), ref)
    assert err <= TOL, err
    _storage_bound_check(s, 0, inputs)
    # bench.py's timed steps: a step stream (6 partitions of 5504 tokens per KV head, 48 units), its
    # steps back to back on one workspace
    assert dec.part_tokens(s.q, k, v, s.table, s.seq_lens, s.max_len, k_scale=ks, v_scale=vs, step_stream=True) == 5504
    outs = [dec(s.q, k, v, s.table, s.seq_lens, s.max_len, k_scale=ks, v_scale=vs, step_stream=True)
            for _ in range(8)]
    torch.cuda.synchronize()
    assert dec.error_flag() == 0
    err = oracle.max_abs_diff(outs[0].cpu().numpy(), ref)
    assert err <= TOL, err
    assert all(torch.equal(o, outs[0]) for o in outs)
    if dtype == "i8":
        # bench's int8 pool is what the reference's quantizer makes of the same fp32 values
        k32, v32 = s.sequence_fp32(torch, 0)
        table = s.table_host[:1]
        for src, pool, sc in ((k32, k, ks), (v32, v, vs)):
            p8, s8 = oracle.quantize_i8(src, table, s.lens, num_blocks=s.num_blocks, page=s.page)
            live = table[0, :256]
            assert np.array_equal(pool.cpu().numpy()[live], p8[live])
            assert np.array_equal(sc.cpu().numpy()[live], s8[live])
    _free(s)


def test_config4_all_sequences():
    """64 ragged sequences (log-uniform in [512, 32768]), page 16, pool 1.1 x live pages: every
    sequence against the oracle; the storage bound on the shortest and the longest."""
    s = DeviceStep(torch, config(4), device=torch.device("cuda", 0))
    assert len(s.lens) == 64
    _decode(s)
    out = s.out.cpu().numpy()
    worst = 0.0
    for i in range(64):
        ref, inputs = _oracle(s, i)
        err = oracle.max_abs_diff(out[i:i + 1], ref)
        assert err <= TOL, (i, s.lens[i], err)
        worst = max(worst, err)
        if i in (int(np.argmin(s.lens)), int(np.argmax(s.lens))):
            _storage_bound_check(s, i, inputs)
    print(f"config 4: worst |gpu - ref| over 64 sequences = {worst:.3g}")
    _free(s)


@pytest.mark.parametrize("dtype", ["i8", "f16"])
def test_config5_sampled_sequences(dtype):
    """The whole config-5 step (256 sequences of 8192-131072 tokens, 64/8 heads, page 64, about 19 k
    units in 7808/8064-token partitions) decoded in one launch; the shortest, the longest and a
    seeded sample of four sequences checked against the oracle one at a time."""
    s = DeviceStep(torch, config(5, dtype), device=torch.device("cuda", 0))
    dec = _decode(s)
    k, v, ks, vs = s.pools[0]
    part = dec.part_tokens(s.q, k, v, s.table, s.seq_lens, s.max_len, k_scale=ks, v_scale=vs, tables_ready=True)
    assert 4096 < part <= 8064
    lens = np.asarray(s.lens)
    rng = np.random.default_rng(55)
    picks = sorted({int(lens.argmin()), int(lens.argmax())} | set(rng.choice(256, 4, replace=False).tolist()))
    out = s.out.cpu().numpy()
    for i in picks:
        ref, inputs = _oracle(s, i)
        err = oracle.max_abs_diff(out[i:i + 1], ref)
        assert err <= TOL, (i, s.lens[i], err)
    i = int(lens.argmin())
    _, inputs = _oracle(s, i)
    _storage_bound_check(s, i, inputs)
    _free(s)


def _rel_err_per_vector(out, ref):
    """max over (sequence, head) of max_d |out - ref| / max_d |ref| (empty sequences must be exactly
    0 and are skipped)."""
    worst = 0.0
    for b in range(ref.shape[0]):
        for h in range(ref.shape[1]):
            scale = float(np.abs(ref[b, h]).max())
            if scale == 0.0:
                assert (out[b, h] == 0).all()
                continue
            worst = max(worst, float(np.abs(out[b, h].astype(np.float64) - ref[b, h]).max()) / scale)
    return worst


def test_config1_fp32_relative():
    """Config 1 (fp32 cache, 512 tokens, page 16, 64-page pool): within 1e-5 relative."""
    s = DeviceStep(torch, config(1), device=torch.device("cuda", 0))
    _decode(s)
    ref, _ = _oracle(s, 0)
    out = s.out.cpu().numpy()
    assert oracle.max_abs_diff(out, ref) <= TOL
    rel = _rel_err_per_vector(out, ref)
    assert rel <= REL32, rel
    _free(s)


# the reference's grid (tests/gpu_tests.cpp:74-157), fp32 storage: shapes, lengths {L, L/3+1, L+5},
# seeds with (part, q_amp), pages
GRID_SHAPES = [(8, 2, 128), (4, 4, 64)]
GRID_LENS = [1, 7, 100, 513, 2049, 4097]
GRID_SEEDS = [(1, 64, 1.0), (2, 256, 8.0), (3, 512, 3.0)]
GRID_PAGES = [16, 32, 64, 128]


@pytest.mark.parametrize("H,Hkv,D", GRID_SHAPES)
def test_fp32_grid_relative(H, Hkv, D):
    """Every fp32 case of the reference's grid shape x length x seed x page, on every kernel that
    takes fp32, within 1e-5 relative per output vector (and the 2e-5 absolute bar)."""
    worst, n = 0.0, 0
    from tests.cuda_runner import run_case
    for L in GRID_LENS:
        for seed, part, q_amp in GRID_SEEDS:
            for page in GRID_PAGES:
                case = oracle.make_case(num_heads=H, num_kv_heads=Hkv, head_dim=D, lens=[L, L // 3 + 1, L + 5],
                                        kv_type=oracle.F32, page=page, seed=seed * 1000 + page, q_amp=q_amp)
                ref = case.reference()
                for kernel in (kvb.Kernel.simt, kvb.Kernel.auto):
                    out = run_case(case, part=part, kernel=kernel)
                    assert oracle.max_abs_diff(out, ref) <= TOL
                    worst = max(worst, _rel_err_per_vector(out, ref))
                    n += 1
    print(f"{n} fp32 runs, worst relative error {worst:.3g}")
    assert worst <= REL32, worst
