"""One process, two GPUs: kernel attributes, occupancy, the static workspace's address and the
reference-facing state are per device, so decoding on device 1 after device 0 works through every
entry point (kvb_paged_decode_async, kvb_paged_decode_static, kvb_run_paged). Needs two GPUs; skipped
on one."""
import numpy as np
import pytest
import torch

import kv_cache_bench_b200 as kvb
import oracle
from kv_cache_bench_b200.torch_ops import PagedDecoder
from tests.cuda_runner import run_case

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")]
TOL = 2e-5


def _dev(case, device):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)  # noqa: E731
    d = dict(q=t(case.q), k=t(case.k), v=t(case.v), table=t(case.table), lens=t(case.lens.astype(np.int32)))
    d["ks"] = t(case.k_scale) if case.k_scale is not None else None
    d["vs"] = t(case.v_scale) if case.v_scale is not None else None
    return d


@pytest.mark.parametrize("kv_type,page,kernel", [(oracle.I8, 128, kvb.Kernel.umma), (oracle.F16, 64, kvb.Kernel.mma),
                                                 (oracle.F32, 16, kvb.Kernel.simt)])
def test_device1_after_device0(kv_type, page, kernel):
    case = oracle.make_case(num_heads=32, num_kv_heads=8, head_dim=128, lens=[2500, 0, 700], kv_type=kv_type,
                            page=page, seed=31)
    ref = case.reference()
    for dev in (0, 1, 0, 1):
        torch.cuda.set_device(dev)
        device = torch.device("cuda", dev)
        d = _dev(case, device)
        dec = PagedDecoder(device)
        out = dec(d["q"], d["k"], d["v"], d["table"], d["lens"], case.max_len, k_scale=d["ks"], v_scale=d["vs"],
                  kernel=kernel)
        torch.cuda.synchronize(device)
        assert oracle.max_abs_diff(out.cpu().numpy(), ref) <= TOL, ("async", dev)
        assert dec.error_flag() == 0
        # the library-owned workspace of this device
        a = kvb.device_args(kvb.Shape(3, 32, 8, 128), kvb.KvType(kv_type), page, d["table"].shape[1], case.max_len,
                            q=d["q"].data_ptr(), k=d["k"].data_ptr(), v=d["v"].data_ptr(),
                            block_table=d["table"].data_ptr(), seq_lens=d["lens"].data_ptr(),
                            out=out.data_ptr(), num_blocks=case.num_blocks,
                            k_scale=d["ks"].data_ptr() if d["ks"] is not None else 0,
                            v_scale=d["vs"].data_ptr() if d["vs"] is not None else 0, kernel=kernel)
        out.fill_(float("nan"))
        stream = torch.cuda.current_stream(device).cuda_stream
        kvb.paged_decode_static(a, stream)
        torch.cuda.synchronize(device)
        assert oracle.max_abs_diff(out.cpu().numpy(), ref) <= TOL, ("static", dev)
        assert kvb.paged_static_error_flag(stream) == 0
        # the reference-facing API (managed buffers, the library's own stream for this device)
        assert oracle.max_abs_diff(run_case(case, kernel=kernel), ref) <= TOL, ("run_paged", dev)
    torch.cuda.set_device(0)
