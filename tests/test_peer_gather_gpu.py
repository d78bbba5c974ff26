"""The in-kernel gather of sharded steps on one GPU (kvb_paged_decode_gather_async,
kvb_peer_barrier_async): output rows land at their global position (row map, head offset) in every
buffer of the peer list, bit-identical to a plain launch, on every kernel; a bad global row is
refused; and a step barrier whose peer never signals gives up after its limit with the TIMEOUT bit,
leaving the context usable. The two-rank path runs in tests/test_sharded_nccl_gpu.py."""
import numpy as np
import pytest
import torch

import kv_cache_bench_b200 as kvb
import oracle
from kv_cache_bench_b200.torch_ops import PagedDecoder

pytestmark = pytest.mark.gpu
TOL = 2e-5


def _case(kv_type, lens, seed=29):
    case = oracle.make_case(num_heads=32, num_kv_heads=8, head_dim=128, lens=lens, kv_type=kv_type, page=16,
                            seed=seed)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    d = dict(q=t(case.q), k=t(case.k), v=t(case.v), table=t(case.table), lens=t(case.lens.astype(np.int32)))
    if case.k_scale is not None:
        d["ks"], d["vs"] = t(case.k_scale), t(case.v_scale)
    return case, d


def _args(dec, d, max_len, kernel):
    out = torch.empty_like(d["q"])
    return dec.args(d["q"], d["k"], d["v"], d["table"], d["lens"], max_len, out=out, k_scale=d.get("ks"),
                    v_scale=d.get("vs"), kernel=kernel), out


def _workspace(dec, c):
    need = kvb.paged_workspace_bytes(c)
    if need > dec.workspace.numel():
        dec.workspace = torch.zeros(need, dtype=torch.uint8, device="cuda")
    return dec.workspace.data_ptr(), dec.workspace.numel()


@pytest.mark.parametrize("kv_type,lens,kernel", [
    (oracle.F16, [3000, 0, 700, 129], kvb.Kernel.auto), (oracle.I8, [5000, 17, 2100], kvb.Kernel.auto),
    (oracle.F16, [900, 2200, 0], kvb.Kernel.mma), (oracle.F32, [1500, 64], kvb.Kernel.simt)])
def test_rows_land_at_their_global_position_in_every_buffer(kv_type, lens, kernel):
    case, d = _case(kv_type, lens)
    dec = PagedDecoder()
    c, out = _args(dec, d, case.max_len, kernel)
    ws, wsn = _workspace(dec, c)
    stream = torch.cuda.current_stream()
    kvb.paged_decode_async(c, ws, wsn, stream.cuda_stream)
    B, H, D = d["q"].shape
    rows_g, heads_g, head0 = 2 * B + 1, 2 * H, H  # this "rank" holds the second half of the heads
    rows = torch.tensor([2 * b + 1 for b in range(B)][::-1], dtype=torch.int32, device="cuda")
    bufs = [torch.full((rows_g, heads_g, D), -7.0, device="cuda") for _ in range(3)]
    peers = kvb.peer_out([b.data_ptr() for b in bufs], 1, rows_g, heads_g, head0, rows.data_ptr())
    for _ in range(3):
        kvb.paged_decode_gather_async(c, peers, ws, wsn, stream.cuda_stream)
    torch.cuda.synchronize()
    assert dec.error_flag() == 0
    assert oracle.max_abs_diff(out.cpu().numpy(), case.reference()) <= TOL
    expect = torch.full((rows_g, heads_g, D), -7.0, device="cuda")
    expect[rows.long(), head0:] = out
    for b in bufs:
        assert torch.equal(b, expect)


def test_a_global_row_out_of_range_is_refused():
    case, d = _case(oracle.F16, [800, 300])
    dec = PagedDecoder()
    c, out = _args(dec, d, case.max_len, kvb.Kernel.auto)
    ws, wsn = _workspace(dec, c)
    B, H, D = d["q"].shape
    buf = torch.full((B, H, D), -7.0, device="cuda")
    rows = torch.tensor([0, B], dtype=torch.int32, device="cuda")  # the second row is past the buffer
    peers = kvb.peer_out([buf.data_ptr()], 0, B, H, 0, rows.data_ptr())
    kvb.paged_decode_gather_async(c, peers, ws, wsn, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert dec.error_flag() == 2
    assert torch.all(buf[1] == -7.0)


def test_peer_arguments_are_checked_before_launch():
    case, d = _case(oracle.F16, [100])
    dec = PagedDecoder()
    c, out = _args(dec, d, case.max_len, kvb.Kernel.auto)
    ws, wsn = _workspace(dec, c)
    B, H, D = d["q"].shape
    buf = torch.zeros((B, H, D), device="cuda")
    for peers in (kvb.peer_out([buf.data_ptr()], 1, B, H),  # self out of range
                  kvb.peer_out([buf.data_ptr()], 0, B, H - 1),  # heads do not fit
                  kvb.peer_out([buf.data_ptr() + 4], 0, B, H)):  # misaligned
        with pytest.raises(ValueError):
            kvb.paged_decode_gather_async(c, peers, ws, wsn, 0)
    sig = torch.zeros(kvb.MAX_PEERS, dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError):
        kvb.peer_barrier_async(kvb.peer_barrier_args(2, [sig.data_ptr()] * 2, sig.data_ptr()), ws, 0)


def test_barrier_passes_alone_and_times_out_without_its_peer():
    """One rank alone passes at once. With a second rank that never signals (its word in this rank's
    signal array stays 0), the wait gives up after its limit, sets the TIMEOUT bit, and the stream
    stays usable: a decode after it gives the oracle's result."""
    case, d = _case(oracle.I8, [2000, 300])
    dec = PagedDecoder()
    c, out = _args(dec, d, case.max_len, kvb.Kernel.auto)
    ws, wsn = _workspace(dec, c)
    stream = torch.cuda.current_stream().cuda_stream
    mine = torch.zeros(kvb.MAX_PEERS, dtype=torch.int32, device="cuda")
    other = torch.zeros(kvb.MAX_PEERS, dtype=torch.int32, device="cuda")
    epoch = torch.zeros(4, dtype=torch.int32, device="cuda")
    alone = kvb.peer_barrier_args(0, [mine.data_ptr()], epoch.data_ptr(), timeout_us=20000)
    for _ in range(3):
        kvb.peer_barrier_async(alone, ws, stream)
    torch.cuda.synchronize()
    assert dec.error_flag() == 0
    assert int(epoch[0]) == 3 and int(mine[0]) == 3
    pair = kvb.peer_barrier_args(0, [mine.data_ptr(), other.data_ptr()], epoch.data_ptr(), timeout_us=20000)
    kvb.peer_barrier_async(pair, ws, stream)
    kvb.paged_decode_async(c, ws, wsn, stream)
    torch.cuda.synchronize()
    assert dec.error_flag() == 4  # TIMEOUT, read and cleared
    assert int(other[0]) == 4  # this rank's signal reached the silent peer's array
    assert oracle.max_abs_diff(out.cpu().numpy(), case.reference()) <= TOL
    kvb.paged_decode_async(c, ws, wsn, stream)
    torch.cuda.synchronize()
    assert dec.error_flag() == 0
