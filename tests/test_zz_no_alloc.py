"""kvb_paged_decode_static (the library-owned 16 MiB workspace, no allocation on the call path)
against kvb_paged_decode_async with a caller workspace, through the C ABI. Named to run last: the
static workspace persists for the process, so this also checks that it is ready after whatever the
other tests left behind."""
import numpy as np
import pytest
import torch

import kv_cache_bench_b200 as kvb
import oracle

pytestmark = pytest.mark.gpu
TOL = 2e-5  # the reference's kernel tolerance (tests/gpu_tests.cpp:16)


def _dev(case):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    d = dict(q=t(case.q), k=t(case.k), v=t(case.v), table=t(case.table), lens=t(case.lens.astype(np.int32)))
    d["ks"] = t(case.k_scale) if case.k_scale is not None else None
    d["vs"] = t(case.v_scale) if case.v_scale is not None else None
    return d


def _args(d, max_len, out, **kw):
    B, H, D = d["q"].shape
    num_blocks, Hkv, page, _ = d["k"].shape
    kvt = {torch.float32: kvb.KvType.f32, torch.float16: kvb.KvType.f16, torch.int8: kvb.KvType.i8}[d["k"].dtype]
    return kvb.device_args(kvb.Shape(B, H, Hkv, D), kvt, page, d["table"].shape[1], max_len, q=d["q"].data_ptr(),
                           k=d["k"].data_ptr(), v=d["v"].data_ptr(), block_table=d["table"].data_ptr(),
                           seq_lens=d["lens"].data_ptr(), out=out.data_ptr(), num_blocks=num_blocks,
                           k_scale=d["ks"].data_ptr() if d["ks"] is not None else 0,
                           v_scale=d["vs"].data_ptr() if d["vs"] is not None else 0, **kw)


@pytest.mark.parametrize("kv_type,page,kernel", [(oracle.F32, 16, kvb.Kernel.auto), (oracle.F16, 64, kvb.Kernel.auto),
                                                 (oracle.I8, 128, kvb.Kernel.auto), (oracle.F16, 32, kvb.Kernel.mma),
                                                 (oracle.I8, 16, kvb.Kernel.simt)])
def test_static_workspace_matches_caller_workspace_twice_in_a_row(kv_type, page, kernel):
    case = oracle.make_case(num_heads=32, num_kv_heads=8, head_dim=128, lens=[3000, 0, 777, 129, 8200],
                            kv_type=kv_type, page=page, seed=21)
    d = _dev(case)
    stream = torch.cuda.current_stream().cuda_stream
    ref_out = torch.full_like(d["q"], float("nan"))
    a = _args(d, case.max_len, ref_out, kernel=kernel)
    ws = torch.zeros(kvb.paged_workspace_bytes(a), dtype=torch.uint8, device="cuda")
    kvb.paged_decode_async(a, ws.data_ptr(), ws.numel(), stream)

    outs = []
    for _ in range(2):  # two calls in a row on the same static workspace
        out = torch.full_like(d["q"], float("nan"))
        kvb.paged_decode_static(_args(d, case.max_len, out, kernel=kernel), stream)
        outs.append(out)
    torch.cuda.synchronize()
    ref = ref_out.cpu().numpy()
    assert oracle.max_abs_diff(ref, case.reference()) <= TOL
    for out in outs:
        o = out.cpu().numpy()
        assert not np.isnan(o).any()
        assert oracle.max_abs_diff(o, ref) <= TOL
        assert oracle.max_abs_diff(o, case.reference()) <= TOL
        assert (o[1] == 0).all()  # the empty sequence


def test_static_workspace_refuses_oversize_before_launch():
    # 256 sequences x 64 heads x 32 partitions x 128 dims of fp32 partials: far above 16 MiB
    B, H, Hkv, D, page, max_len = 256, 64, 8, 128, 64, 131072
    q = torch.zeros(B, H, D, device="cuda")
    out = torch.full_like(q, 7.0)
    k = torch.zeros(1, Hkv, page, D, dtype=torch.float16, device="cuda")
    table = torch.zeros(B, max_len // page, dtype=torch.int32, device="cuda")
    lens = torch.zeros(B, dtype=torch.int32, device="cuda")
    a = kvb.device_args(kvb.Shape(B, H, Hkv, D), kvb.KvType.f16, page, table.shape[1], max_len, q=q.data_ptr(),
                        k=k.data_ptr(), v=k.data_ptr(), block_table=table.data_ptr(), seq_lens=lens.data_ptr(),
                        out=out.data_ptr(), num_blocks=1)
    assert kvb.paged_workspace_bytes(a) > kvb.STATIC_WORKSPACE_BYTES
    with pytest.raises(ValueError, match="static workspace holds"):
        kvb.paged_decode_static(a, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert (out == 7.0).all()  # nothing was launched


def test_static_error_word_is_read_and_cleared():
    """kvb_paged_static_error_flag reads the library-owned workspace's error word: a refused length
    (NaN outputs, bit 1) shows once and is cleared by the read; a correct call follows."""
    case = oracle.make_case(num_heads=32, num_kv_heads=8, head_dim=128, lens=[900, 300], kv_type=oracle.I8,
                            page=64, seed=23)
    d = _dev(case)
    stream = torch.cuda.current_stream().cuda_stream
    assert kvb.paged_static_error_flag(stream) == 0
    d["lens"][1] = 100_000  # beyond max_len and the block table
    out = torch.full_like(d["q"], 0.0)
    kvb.paged_decode_static(_args(d, case.max_len, out), stream)
    assert kvb.paged_static_error_flag(stream) & 1
    assert kvb.paged_static_error_flag(stream) == 0
    assert torch.isnan(out[1]).all()
    d["lens"][1] = 300
    out = torch.full_like(d["q"], float("nan"))
    kvb.paged_decode_static(_args(d, case.max_len, out), stream)
    torch.cuda.synchronize()
    assert oracle.max_abs_diff(out.cpu().numpy(), case.reference()) <= TOL
    assert kvb.paged_static_error_flag(stream) == 0
