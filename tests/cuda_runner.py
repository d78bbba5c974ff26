"""Drives the CUDA path through the reference-facing C ABI (kvb_run_paged / kvb_run_naive with
managed Buffers), the way the reference's tests drive run_paged (tests/gpu_tests.cpp:120-131):
the output is poisoned with NaN first, so an element the kernel fails to write shows up."""
import numpy as np

import kv_cache_bench_b200 as kvb


def _buf(a):
    return kvb.Buffer.from_array(np.ascontiguousarray(a))


def run_paged(q, k, v, table, lens, *, num_kv_heads, page, kv_type, max_len=None, k_scale=None, v_scale=None,
              part=0, share_kv=True, kernel=kvb.Kernel.auto, steps=1):
    q = np.ascontiguousarray(q, np.float32)
    B, H, D = q.shape
    lens = np.ascontiguousarray(lens, np.int32)
    table = np.ascontiguousarray(table, np.int32)
    max_blocks = table.shape[1] if table.ndim == 2 else 0
    if max_len is None:
        max_len = int(lens.max()) if lens.size else 0
    out = kvb.Buffer(q.nbytes)
    out.as_array(np.float32)[:] = np.nan
    bufs = dict(q=_buf(q), k=_buf(k), v=_buf(v), block_table=_buf(table), seq_lens=_buf(lens), out=out)
    if k_scale is not None:
        bufs["k_scale"], bufs["v_scale"] = _buf(k_scale), _buf(v_scale)
    a = kvb.PagedArgs(kvb.Shape(B, H, num_kv_heads, D), kvb.KvType(kv_type), page, max_blocks, max_len, part,
                      share_kv=share_kv, num_blocks=int(k.shape[0]), kernel=kernel, **bufs)
    kvb.run_paged_steps(a, steps)
    return out.as_array(np.float32, q.size).reshape(B, H, D).copy()


def run_case(case, **kw):
    """A golden-vector dict or an oracle.PagedCase through run_paged."""
    if isinstance(case, dict):
        return run_paged(case["q"], case["k"], case["v"], case["block_table"], case["seq_lens"],
                         num_kv_heads=case["num_kv_heads"], page=case["page_size"], kv_type=case["kv_type"],
                         max_len=case["max_len"], k_scale=case.get("k_scale"), v_scale=case.get("v_scale"), **kw)
    return run_paged(case.q, case.k, case.v, case.table, case.lens, num_kv_heads=case.num_kv_heads, page=case.page,
                     kv_type=case.kv_type, k_scale=case.k_scale, v_scale=case.v_scale, **kw)


def run_naive(case):
    q = np.ascontiguousarray(case["q"], np.float32)
    B, H, D = q.shape
    out = kvb.Buffer(q.nbytes)
    out.as_array(np.float32)[:] = np.nan
    a = kvb.NaiveArgs(kvb.Shape(B, H, case["num_kv_heads"], D), kvb.KvType(case["kv_type"]), case["max_len"],
                      _buf(q), _buf(case["k"]), _buf(case["v"]), _buf(np.asarray(case["seq_lens"], np.int32)), out)
    kvb.run_naive(a)
    return out.as_array(np.float32, q.size).reshape(B, H, D).copy()


def mma_ok(kv_type, head_dim, page, group, share_kv=True):
    qg = min(group, 8) if share_kv else 1
    row = head_dim * (2 if kv_type == 1 else 1)
    return kv_type in (1, 2) and row in (128, 256) and page in (8, 16, 32, 64, 128, 256) and 1 <= qg <= 8


def umma_ok(kv_type, head_dim, page, group, share_kv=True):
    qg = min(group, 8) if share_kv else 1
    return kv_type in (1, 2) and head_dim == 128 and page in (8, 16, 32, 64, 128, 256) and 1 <= qg <= 8


def kernels_for(kv_type, head_dim, page, group, share_kv=True):
    """Every kernel that supports the shape, plus the automatic choice."""
    ks = [kvb.Kernel.simt, kvb.Kernel.auto]
    if mma_ok(kv_type, head_dim, page, group, share_kv):
        ks.append(kvb.Kernel.mma)
    if umma_ok(kv_type, head_dim, page, group, share_kv):
        ks.append(kvb.Kernel.umma)
    return ks
