"""The stream-level C ABI (kvb_paged_decode_async) with torch tensors as device buffers: parity,
workspace reuse across calls and shapes, CUDA-graph capture, and the device-side refusal of bad
lengths and block ids (NaN outputs plus an error flag, no out-of-bounds access)."""
import numpy as np
import pytest
import torch

import kv_cache_bench_b200 as kvb
import oracle
from kv_cache_bench_b200.torch_ops import PagedDecoder

pytestmark = pytest.mark.gpu
TOL = 2e-5


def _dev(case, device="cuda"):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)  # noqa: E731
    d = dict(q=t(case.q), k=t(case.k), v=t(case.v), table=t(case.table), lens=t(case.lens.astype(np.int32)))
    if case.k_scale is not None:
        d["ks"], d["vs"] = t(case.k_scale), t(case.v_scale)
    return d


def _call(dec, d, max_len, **kw):
    return dec(d["q"], d["k"], d["v"], d["table"], d["lens"], max_len, k_scale=d.get("ks"), v_scale=d.get("vs"),
               **kw)


@pytest.mark.parametrize("kv_type", [oracle.F32, oracle.F16, oracle.I8])
def test_async_matches_oracle_and_reuses_workspace(kv_type):
    dec = PagedDecoder()
    for seed, lens in enumerate([[3000, 5, 0, 700], [64, 65], [9000]]):
        case = oracle.make_case(num_heads=32, num_kv_heads=8, head_dim=128, lens=lens, kv_type=kv_type, page=64,
                                seed=seed)
        d = _dev(case)
        ref = case.reference()
        for part in (0, 128, 0):  # the same workspace across calls, shapes and partition sizes
            out = _call(dec, d, case.max_len, part_tokens=part)
            torch.cuda.synchronize()
            assert oracle.max_abs_diff(out.cpu().numpy(), ref) <= TOL, (lens, part)
        assert dec.error_flag() == 0


def test_cuda_graph_replay():
    case = oracle.make_case(num_heads=32, num_kv_heads=8, head_dim=128, lens=[5000, 300], kv_type=oracle.I8,
                            page=128, seed=3)
    d = _dev(case)
    dec = PagedDecoder()
    out = torch.empty_like(d["q"])
    _call(dec, d, case.max_len, out=out)  # sizes the workspace outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            _call(dec, d, case.max_len, out=out)
    out.fill_(float("nan"))
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert oracle.max_abs_diff(out.cpu().numpy(), case.reference()) <= TOL
    del g


@pytest.mark.parametrize("kv_type,lens", [(oracle.F16, [8000, 0, 3, 5000, 129] * 8),
                                          (oracle.I8, [8000, 0, 3, 5000, 129] * 8),
                                          (oracle.F16, [(i * 97) % 701 for i in range(300)])])
def test_tables_ready_and_dynamic_units_are_bit_identical(kv_type, lens):
    """FLAG_TABLES_READY (lengths and block ids read while the previous kernel finishes),
    FLAG_INPUTS_READY (pages streamed before it finishes) and the dynamic hand-out of units (far more
    units than CTAs here) change no bit of the output, over
    repeated launches on one workspace (the work counters must come back to zero each time). The
    300-sequence case enumerates units densely (more sequences than the per-CTA prefix holds)."""
    case = oracle.make_case(num_heads=32, num_kv_heads=8, head_dim=128, lens=lens, kv_type=kv_type, page=64,
                            seed=11)
    d = _dev(case)
    dec = PagedDecoder()
    flags = [dict(), dict(tables_ready=True), dict(tables_ready=True, inputs_ready=True), dict(),
             dict(tables_ready=True, inputs_ready=True), dict(tables_ready=True)]
    outs = [_call(dec, d, case.max_len, part_tokens=512, **f).clone() for f in flags]
    torch.cuda.synchronize()
    assert oracle.max_abs_diff(outs[0].cpu().numpy(), case.reference()) <= TOL
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    assert dec.error_flag() == 0


def test_automatic_partitions_grow_with_many_units():
    """With far more units than SMs and pages of 32 tokens or more, the automatic partition exceeds
    4096 tokens (up to 8064); a small batch keeps the one-wave split."""
    mk = lambda B, L, page: kvb.device_args(kvb.Shape(B, 64, 8, 128), kvb.KvType.f16, page, (L + page - 1) // page,  # noqa: E731
                                            L, q=256, k=256, v=256, block_table=256, seq_lens=256, out=256,
                                            num_blocks=B * ((L + page - 1) // page))
    big = kvb.paged_part_tokens(mk(256, 131072, 64))
    assert 4096 < big <= 8064 and big % 128 == 0
    assert kvb.paged_part_tokens(mk(256, 131072, 16)) <= 4096  # 16-token pages: the page table's bound
    assert kvb.paged_part_tokens(mk(1, 32768, 128)) <= 4096


@pytest.mark.parametrize("kernel", [kvb.Kernel.simt, kvb.Kernel.mma, kvb.Kernel.umma])
def test_device_refuses_bad_lengths_with_nan_and_flag(kernel):
    case = oracle.make_case(num_heads=32, num_kv_heads=8, head_dim=128, lens=[300, 200, 100], kv_type=oracle.F16,
                            page=64, seed=4)
    d = _dev(case)
    dec = PagedDecoder()
    ref = case.reference()
    # sequence 1 claims more tokens than max_len (and than its block table holds)
    d["lens"][1] = 10_000
    out = _call(dec, d, case.max_len, kernel=kernel)
    torch.cuda.synchronize()
    o = out.cpu().numpy()
    assert np.isnan(o[1]).all()
    assert oracle.max_abs_diff(o[[0, 2]], ref[[0, 2]]) <= TOL
    assert dec.error_flag() & 1
    assert dec.error_flag() == 0  # reading clears it
    # a negative length
    d["lens"][1] = -5
    o = _call(dec, d, case.max_len, kernel=kernel).cpu().numpy()
    assert np.isnan(o[1]).all() and dec.error_flag() & 1


@pytest.mark.parametrize("kernel", [kvb.Kernel.simt, kvb.Kernel.mma, kvb.Kernel.umma])
def test_device_refuses_bad_block_ids_with_nan_and_flag(kernel):
    case = oracle.make_case(num_heads=32, num_kv_heads=8, head_dim=128, lens=[300, 200], kv_type=oracle.I8,
                            page=64, seed=6)
    d = _dev(case)
    dec = PagedDecoder()
    ref = case.reference()
    for bad in (case.num_blocks, 1 << 30, -7):
        d["table"][0, 2] = bad
        o = _call(dec, d, case.max_len, kernel=kernel).cpu().numpy()
        assert np.isnan(o[0]).all(), bad
        assert oracle.max_abs_diff(o[1], ref[1]) <= TOL
        assert dec.error_flag() & 2


def test_host_path_refuses_bad_block_ids_before_launch():
    case = oracle.make_case(num_heads=8, num_kv_heads=2, head_dim=128, lens=[40], kv_type=oracle.F16, page=16,
                            seed=8)
    case.table[0, 1] = case.num_blocks + 3
    from tests.cuda_runner import run_case
    with pytest.raises(ValueError, match="block"):
        run_case(case)


@pytest.mark.parametrize("kernel", [kvb.Kernel.simt, kvb.Kernel.mma, kvb.Kernel.umma])
def test_stale_arrival_counter_reports_state_and_the_flag_read_resets_it(kernel):
    """A split-K arrival counter left past its partition count (what an aborted launch or two
    launches sharing one workspace leave behind) is planted in the workspace on the host: the next
    launch reports STATE (8) instead of merging, kvb_paged_error_flag resets the counters, and the
    launch after it is correct again."""
    case = oracle.make_case(num_heads=32, num_kv_heads=8, head_dim=128, lens=[3000, 700], kv_type=oracle.F16,
                            page=64, seed=9)
    d = _dev(case)
    dec = PagedDecoder()
    ref = case.reference()
    out = _call(dec, d, case.max_len, part_tokens=512, kernel=kernel)
    torch.cuda.synchronize()
    assert oracle.max_abs_diff(out.cpu().numpy(), ref) <= TOL and dec.error_flag() == 0
    # counter of (sequence 0, head group 0): the clean epoch with 1000 arrivals already counted
    dec.workspace[256:264].view(torch.int64).fill_((0x7FFFFFFF << 32) | 1000)
    _call(dec, d, case.max_len, part_tokens=512, kernel=kernel)
    torch.cuda.synchronize()
    assert dec.error_flag() & 8
    out = torch.full_like(d["q"], float("nan"))
    _call(dec, d, case.max_len, part_tokens=512, kernel=kernel, out=out)
    torch.cuda.synchronize()
    assert oracle.max_abs_diff(out.cpu().numpy(), ref) <= TOL
    assert dec.error_flag() == 0


@pytest.mark.parametrize("kv_type,lens,part", [(oracle.I8, [32768], 0), (oracle.F16, [20000, 3000, 0, 129], 2048),
                                               (oracle.I8, [9000, 9000, 4000], 0)])
def test_single_wave_launches_with_inputs_ready_are_bit_identical(kv_type, lens, part):
    """With FLAG_INPUTS_READY the pages stream before the previous kernel's end: back-to-back
    launches on one workspace, each with one unit per CTA, give the oracle's result, bit-identical to
    the launch without the flags."""
    case = oracle.make_case(num_heads=32, num_kv_heads=8, head_dim=128, lens=lens, kv_type=kv_type, page=128,
                            seed=13)
    d = _dev(case)
    dec = PagedDecoder()
    base = _call(dec, d, case.max_len, part_tokens=part).clone()
    outs = [_call(dec, d, case.max_len, part_tokens=part, tables_ready=True, inputs_ready=True) for _ in range(6)]
    torch.cuda.synchronize()
    assert oracle.max_abs_diff(base.cpu().numpy(), case.reference()) <= TOL
    for o in outs:
        assert torch.equal(o, base)
    assert dec.error_flag() == 0


@pytest.mark.parametrize("kv_type,lens", [(oracle.I8, [32768]), (oracle.F16, [32768]), (oracle.I8, [9000, 20000, 700]),
                                           (oracle.F16, [5000, 0, 129])])
def test_step_stream_steps_overlap_and_match_a_lone_launch(kv_type, lens):
    """FLAG_STEP_STREAM: longer partitions for few (sequence, head group) pairs, and back-to-back
    steps on one workspace with several of them streaming at once: each step gives the oracle's
    result, bit-identical to a lone launch (no flags) with the same partition size."""
    case = oracle.make_case(num_heads=32, num_kv_heads=8, head_dim=128, lens=lens, kv_type=kv_type, page=128,
                            seed=19)
    d = _dev(case)
    dec = PagedDecoder()
    kw = dict(k_scale=d.get("ks"), v_scale=d.get("vs"))
    part_one = dec.part_tokens(d["q"], d["k"], d["v"], d["table"], d["lens"], case.max_len, inputs_ready=True, **kw)
    part = dec.part_tokens(d["q"], d["k"], d["v"], d["table"], d["lens"], case.max_len, step_stream=True, **kw)
    assert part > part_one
    base = _call(dec, d, case.max_len, part_tokens=part).clone()
    outs = [_call(dec, d, case.max_len, step_stream=True) for _ in range(12)]
    torch.cuda.synchronize()
    assert oracle.max_abs_diff(base.cpu().numpy(), case.reference()) <= TOL
    for o in outs:
        assert torch.equal(o, base)
    assert dec.error_flag() == 0


@pytest.mark.parametrize("kv_type,page,lens", [(oracle.F32, 16, [512]), (oracle.F32, 7, [3000, 0, 130, 65]),
                                               (oracle.I8, 48, [2000, 1, 700])])
def test_cuda_core_kernel_with_inputs_ready_is_bit_identical(kv_type, page, lens):
    """The CUDA-core kernel reads its inputs before the previous kernel ends when both early flags
    are set and waits only before its writes: back-to-back launches give the oracle's result,
    bit-identical to launches without the flags."""
    case = oracle.make_case(num_heads=32, num_kv_heads=8, head_dim=128, lens=lens, kv_type=kv_type, page=page,
                            seed=17)
    d = _dev(case)
    dec = PagedDecoder()
    base = _call(dec, d, case.max_len, kernel=kvb.Kernel.simt).clone()
    outs = [_call(dec, d, case.max_len, kernel=kvb.Kernel.simt, inputs_ready=True).clone() for _ in range(5)]
    torch.cuda.synchronize()
    assert oracle.max_abs_diff(base.cpu().numpy(), case.reference()) <= TOL
    for o in outs:
        assert torch.equal(o, base)
    assert dec.error_flag() == 0


@pytest.mark.parametrize("kv_type,lens,kernel,flags", [
    (oracle.I8, [32768], kvb.Kernel.auto, "stream"), (oracle.F16, [9000, 0, 700], kvb.Kernel.auto, "inputs"),
    (oracle.I8, [5000, 129], kvb.Kernel.auto, ""), (oracle.F32, [3000, 65], kvb.Kernel.simt, "inputs")])
def test_inputs_and_output_in_pinned_host_memory(kv_type, lens, kernel, flags):
    """q, the lengths and the block table read by the kernels from page-locked host memory, the output
    written into page-locked host memory (the device reaches it at the host address): back-to-back
    steps give the result of the same launch on device buffers, bit for bit."""
    case = oracle.make_case(num_heads=32, num_kv_heads=8, head_dim=128, lens=lens, kv_type=kv_type, page=128,
                            seed=23)
    d = _dev(case)
    dec = PagedDecoder()
    kw = dict(inputs_ready=flags in ("inputs", "stream"), step_stream=flags == "stream")
    base = _call(dec, d, case.max_len, kernel=kernel, **kw).clone()
    torch.cuda.synchronize()
    assert oracle.max_abs_diff(base.cpu().numpy(), case.reference()) <= TOL
    hq, hl, ht = (d[n].cpu().pin_memory() for n in ("q", "lens", "table"))
    hout = torch.full(tuple(base.shape), float("nan")).pin_memory()
    B, H, D = hq.shape
    num_blocks, Hkv, page, _ = d["k"].shape
    kvt = {oracle.F32: kvb.KvType.f32, oracle.F16: kvb.KvType.f16, oracle.I8: kvb.KvType.i8}[kv_type]
    c = kvb.device_args(kvb.Shape(B, H, Hkv, D), kvt, page, ht.shape[1], case.max_len, q=hq.data_ptr(),
                        k=d["k"].data_ptr(), v=d["v"].data_ptr(), block_table=ht.data_ptr(), seq_lens=hl.data_ptr(),
                        out=hout.data_ptr(), num_blocks=num_blocks,
                        k_scale=d["ks"].data_ptr() if "ks" in d else 0, v_scale=d["vs"].data_ptr() if "vs" in d else 0,
                        kernel=kernel, **kw)
    stream = torch.cuda.current_stream()
    for _ in range(6):
        kvb.paged_decode_async(c, dec.workspace.data_ptr(), dec.workspace.numel(), stream.cuda_stream)
    stream.synchronize()
    assert torch.equal(hout, base.cpu())
    assert dec.error_flag() == 0


def test_partition_from_host_lengths():
    """kvb_paged_part_tokens_for: a ragged batch with a few units per CTA gets smaller partitions
    than the automatic size (at least 1024 tokens), one wave keeps the automatic size, and the
    decode with the chosen size gives the oracle's result."""
    lens = [9000, 30000, 700, 4100, 15000, 2000, 25000, 600]
    case = oracle.make_case(num_heads=32, num_kv_heads=8, head_dim=128, lens=lens, kv_type=oracle.F16, page=16,
                            seed=31)
    d = _dev(case)
    dec = PagedDecoder()
    auto = dec.part_tokens(d["q"], d["k"], d["v"], d["table"], d["lens"], case.max_len, inputs_ready=True)
    out = torch.empty_like(d["q"])
    c = dec.args(d["q"], d["k"], d["v"], d["table"], d["lens"], case.max_len, out=out, inputs_ready=True)
    part = kvb.paged_part_tokens_for(c, lens)
    assert 1024 <= part < auto and part % 128 == 0
    got = _call(dec, d, case.max_len, part_tokens=part, inputs_ready=True)
    torch.cuda.synchronize()
    assert oracle.max_abs_diff(got.cpu().numpy(), case.reference()) <= TOL
    assert dec.error_flag() == 0
    one = oracle.make_case(num_heads=32, num_kv_heads=8, head_dim=128, lens=[32768], kv_type=oracle.I8, page=128,
                           seed=31)
    d1 = _dev(one)
    o1 = torch.empty_like(d1["q"])
    c1 = dec.args(d1["q"], d1["k"], d1["v"], d1["table"], d1["lens"], one.max_len, out=o1, k_scale=d1["ks"],
                  v_scale=d1["vs"], inputs_ready=True)
    assert kvb.paged_part_tokens_for(c1, [32768]) == kvb.paged_part_tokens(c1) == 1920
