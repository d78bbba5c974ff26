"""CPU oracle for the paged decode path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this package, always
as the checker (or the timed CPU baseline), never as part of the product path; the product
(kv_cache_bench_b200) neither imports nor calls it.

``liboracle.so`` (kvb_oracle.c) restates the reference's fp64 oracle (src/reference.cpp:65-100),
its int8 quantizer (src/reference.cpp:32-62) and the storage error bounds of its GPU tests
(tests/gpu_tests.cpp:22-62); tests/test_oracle.py pins it to golden vectors written by the
reference's own code (tests/golden/). The numpy helpers below build seeded synthetic workloads in
the reference's layouts: pool [blocks][Hkv][page][D], block table [B][max_blocks] with -1 for unused
entries, physical blocks assigned in sequence order from a shuffled pool (src/reference.cpp:11-30).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
F32, F16, I8 = 0, 1, 2
NP_DTYPE = {F32: np.float32, F16: np.float16, I8: np.int8}


def _load() -> ctypes.CDLL:
    path = os.path.join(HERE, "liboracle.so")
    if not os.path.exists(path):
        subprocess.run(["make", "-C", HERE, "liboracle.so"], check=True, capture_output=True)
    return ctypes.CDLL(path)


_P = ctypes.c_void_p


def _declare(lib: ctypes.CDLL) -> ctypes.CDLL:
    lib.kvb_oracle_paged_attention.argtypes = [ctypes.c_int] * 7 + [_P] * 8 + [ctypes.c_int]
    lib.kvb_oracle_paged_attention.restype = None
    lib.kvb_oracle_contig_attention.argtypes = [ctypes.c_int] * 6 + [_P] * 5 + [ctypes.c_int]
    lib.kvb_oracle_contig_attention.restype = None
    lib.kvb_oracle_quantize_i8.argtypes = [ctypes.c_int] * 6 + [_P] * 5
    lib.kvb_oracle_quantize_i8.restype = None
    lib.kvb_oracle_dequantize_i8.argtypes = [ctypes.c_int] * 6 + [_P] * 5
    lib.kvb_oracle_dequantize_i8.restype = None
    lib.kvb_oracle_fp16_bound.argtypes = [ctypes.c_int] * 5 + [_P] * 4
    lib.kvb_oracle_fp16_bound.restype = ctypes.c_double
    lib.kvb_oracle_i8_bound.argtypes = [ctypes.c_int] * 6 + [_P] * 5
    lib.kvb_oracle_i8_bound.restype = ctypes.c_double
    lib.kvb_oracle_max_abs_diff.argtypes = [_P, _P, ctypes.c_size_t]
    lib.kvb_oracle_max_abs_diff.restype = ctypes.c_double
    return lib


_lib = _declare(_load())


class use_library:
    """Context manager: the functions of this module call the oracle built at `path` instead (the
    mutation tests load deliberately broken builds of kvb_oracle.c this way)."""

    def __init__(self, path: str):
        self.lib = _declare(ctypes.CDLL(path))

    def __enter__(self):
        global _lib
        self.saved, _lib = _lib, self.lib
        return self

    def __exit__(self, *exc):
        global _lib
        _lib = self.saved
        return False


def _p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def paged_attention(q, k, v, table, lens, *, num_kv_heads, page, kv_type, k_scale=None, v_scale=None,
                    threads: int = os.cpu_count() or 1) -> np.ndarray:
    """fp64 two-pass softmax attention over the paged cache; q [B][H][D] -> out [B][H][D] fp32."""
    q = _c(q, np.float32)
    B, H, D = q.shape
    table = _c(table, np.int32).reshape(B, -1) if B else _c(table, np.int32).reshape(0, 0)
    lens = _c(lens, np.int32)
    k = np.ascontiguousarray(k, dtype=NP_DTYPE[kv_type])
    v = np.ascontiguousarray(v, dtype=NP_DTYPE[kv_type])
    ks = _c(k_scale, np.float32) if k_scale is not None else None
    vs = _c(v_scale, np.float32) if v_scale is not None else None
    out = np.zeros((B, H, D), np.float32)
    _lib.kvb_oracle_paged_attention(B, H, num_kv_heads, D, kv_type, page, table.shape[1] if B else 0, _p(q), _p(k),
                                    _p(v), _p(table), _p(lens), _p(ks), _p(vs), _p(out), int(threads))
    return out


def contig_attention(q, k, v, lens, *, num_kv_heads, max_len, kv_type, threads: int = os.cpu_count() or 1):
    """The same on the contiguous cache [B][Hkv][max_len][D] (fp32 or fp16)."""
    q = _c(q, np.float32)
    B, H, D = q.shape
    k = np.ascontiguousarray(k, dtype=NP_DTYPE[kv_type])
    v = np.ascontiguousarray(v, dtype=NP_DTYPE[kv_type])
    lens = _c(lens, np.int32)
    out = np.zeros((B, H, D), np.float32)
    _lib.kvb_oracle_contig_attention(B, H, num_kv_heads, D, kv_type, max_len, _p(q), _p(k), _p(v), _p(lens),
                                     _p(out), int(threads))
    return out


def quantize_i8(contig, table, lens, *, num_blocks, page):
    """Per (sequence block, KV head) absmax/127 int8 quantization into the paged pool."""
    contig = _c(contig, np.float32)
    B, Hkv, max_len, D = contig.shape
    table = _c(table, np.int32).reshape(B, -1)
    lens = _c(lens, np.int32)
    pool = np.zeros((num_blocks, Hkv, page, D), np.int8)
    scales = np.zeros((num_blocks, Hkv), np.float32)
    _lib.kvb_oracle_quantize_i8(B, Hkv, D, page, table.shape[1], max_len, _p(table), _p(lens), _p(contig), _p(pool),
                                _p(scales))
    return pool, scales


def scatter_paged(contig, table, lens, *, num_blocks, page, fill=0):
    """The live tokens of a contiguous cache [B][Hkv][max_len][D] copied into a pool
    [num_blocks][Hkv][page][D] through the block table (src/reference.hpp:60-68 scatter_to_paged);
    slots holding no live token keep `fill`."""
    contig = np.ascontiguousarray(contig)
    B, Hkv, max_len, D = contig.shape
    table = _c(table, np.int32).reshape(B, -1)
    pool = np.full((num_blocks, Hkv, page, D), fill, contig.dtype)
    for b in range(B):
        L = int(lens[b])
        for i in range((L + page - 1) // page):
            t0, t1 = i * page, min(L, (i + 1) * page)
            pool[table[b, i], :, : t1 - t0] = contig[b, :, t0:t1]
    return pool


def dequantize_i8(pool, scales, table, lens, *, max_len):
    pool = _c(pool, np.int8)
    num_blocks, Hkv, page, D = pool.shape
    lens = _c(lens, np.int32)
    B = lens.shape[0]
    table = _c(table, np.int32).reshape(B, -1)
    contig = np.zeros((B, Hkv, max_len, D), np.float32)
    _lib.kvb_oracle_dequantize_i8(B, Hkv, D, page, table.shape[1], max_len, _p(table), _p(lens), _p(pool),
                                  _p(_c(scales, np.float32)), _p(contig))
    return contig


def fp16_bound(q, k32, v32, lens, *, num_kv_heads, max_len) -> float:
    q = _c(q, np.float32)
    B, H, D = q.shape
    return float(_lib.kvb_oracle_fp16_bound(B, H, num_kv_heads, D, max_len, _p(_c(lens, np.int32)), _p(q),
                                            _p(_c(k32, np.float32)), _p(_c(v32, np.float32))))


def i8_bound(q, table, lens, k_scale, v_scale, *, num_kv_heads, page) -> float:
    q = _c(q, np.float32)
    B, H, D = q.shape
    table = _c(table, np.int32).reshape(B, -1)
    return float(_lib.kvb_oracle_i8_bound(B, H, num_kv_heads, D, page, table.shape[1], _p(table),
                                          _p(_c(lens, np.int32)), _p(q), _p(_c(k_scale, np.float32)),
                                          _p(_c(v_scale, np.float32))))


def max_abs_diff(a, b) -> float:
    """NaN-aware max |a - b| (src/reference.hpp:27-35): any NaN difference is infinite."""
    a = _c(a, np.float32).reshape(-1)
    b = _c(b, np.float32).reshape(-1)
    assert a.size == b.size
    return float(_lib.kvb_oracle_max_abs_diff(_p(a), _p(b), a.size))


# ---- seeded synthetic workloads --------------------------------------------------------------------

def layout_from_perm(lens, page: int, perm: np.ndarray):
    """Block table of src/reference.cpp:11-30 with the shuffle given by `perm` (physical block ids in
    assignment order; len(perm) >= live blocks leaves pool slack). Returns (table, max_blocks)."""
    lens = np.asarray(lens, np.int64)
    nblk = (lens + page - 1) // page
    max_blocks = int(nblk.max()) if lens.size else 0
    table = np.full((lens.size, max_blocks), -1, np.int32)
    nxt = 0
    for b, n in enumerate(nblk):
        table[b, :n] = perm[nxt:nxt + n]
        nxt += int(n)
    return table, max_blocks


@dataclass
class PagedCase:
    """One synthetic decode step in the reference's layouts."""
    num_heads: int
    num_kv_heads: int
    head_dim: int
    kv_type: int
    page: int
    lens: np.ndarray
    q: np.ndarray                # [B][H][D] fp32
    k: np.ndarray                # pool [num_blocks][Hkv][page][D]
    v: np.ndarray
    table: np.ndarray            # [B][max_blocks] int32
    k_scale: Optional[np.ndarray] = None
    v_scale: Optional[np.ndarray] = None
    extras: dict = field(default_factory=dict)

    @property
    def batch(self):
        return int(self.lens.size)

    @property
    def max_len(self):
        return int(self.lens.max()) if self.lens.size else 0

    @property
    def num_blocks(self):
        return int(self.k.shape[0])

    def reference(self, threads: int = os.cpu_count() or 1) -> np.ndarray:
        return paged_attention(self.q, self.k, self.v, self.table, self.lens, num_kv_heads=self.num_kv_heads,
                               page=self.page, kv_type=self.kv_type, k_scale=self.k_scale, v_scale=self.v_scale,
                               threads=threads)

    def min_bytes(self) -> float:
        """Bytes a step must move: K and V of every live token, q and out (src/workload.hpp:69-74)."""
        elem = {F32: 4, F16: 2, I8: 1}[self.kv_type]
        toks = float(self.lens.sum())
        return toks * self.num_kv_heads * self.head_dim * 2 * elem + self.batch * self.num_heads * self.head_dim * 8


def make_case(*, num_heads: int, num_kv_heads: int, head_dim: int, lens, kv_type: int, page: int, seed: int,
              q_amp: float = 1.0, pool_slack: float = 1.0, varied: bool = False, dead_fill: float = 0.0) -> PagedCase:
    """q ~ U(-q_amp, q_amp), K, V ~ U(-1, 1) (src/workload.hpp:26-64), written straight into a
    shuffled pool of ceil(live_blocks * pool_slack) blocks; int8 is quantized per (block, KV head)
    from the fp32 values exactly as the reference's quantizer does. With `varied`, every 16-token
    chunk of K and V gets its own magnitude 2^-U(0,3). Pool slots not holding a live token are
    filled with `dead_fill` (NaN tests that the kernels never let them leak)."""
    rng = np.random.default_rng(seed)
    lens = np.asarray(lens, np.int32)
    B = lens.size
    nblk = (lens.astype(np.int64) + page - 1) // page
    live = int(nblk.sum())
    num_blocks = max(int(np.ceil(live * pool_slack)), live, 1)
    perm = rng.permutation(num_blocks).astype(np.int32)
    table, max_blocks = layout_from_perm(lens, page, perm)
    q = (rng.uniform(-1, 1, (B, num_heads, head_dim)) * q_amp).astype(np.float32)
    pool_shape = (num_blocks, num_kv_heads, page, head_dim)
    k32 = rng.uniform(-1, 1, pool_shape).astype(np.float32)
    v32 = rng.uniform(-1, 1, pool_shape).astype(np.float32)
    if varied:
        chunks = max(1, page // 16) if page >= 16 else 1
        amp = np.exp2(-rng.uniform(0, 3, (2, num_blocks, num_kv_heads, chunks))).astype(np.float32)
        rep = page // chunks
        k32 *= np.repeat(amp[0], rep, axis=2)[:, :, :page, None]
        v32 *= np.repeat(amp[1], rep, axis=2)[:, :, :page, None]
    # mark slots that hold no live token
    live_mask = np.zeros(pool_shape[:3], bool)
    for b in range(B):
        for i in range(int(nblk[b])):
            n = min(page, int(lens[b]) - i * page)
            live_mask[table[b, i], :, :n] = True
    case = PagedCase(num_heads, num_kv_heads, head_dim, kv_type, page, lens, q, None, None, table)
    if kv_type == I8:
        k8 = np.zeros(pool_shape, np.int8)
        v8 = np.zeros(pool_shape, np.int8)
        ks = np.zeros(pool_shape[:2], np.float32)
        vs = np.zeros(pool_shape[:2], np.float32)
        for src, dst, sc in ((k32, k8, ks), (v32, v8, vs)):
            masked = np.where(live_mask[..., None], np.abs(src), 0.0)
            amax = masked.max(axis=(2, 3)).astype(np.float32)
            scale = (amax / np.float32(127.0)).astype(np.float32)
            sc[:] = scale
            with np.errstate(divide="ignore", invalid="ignore"):
                r = np.where(scale[:, :, None, None] > 0, np.rint(src / scale[:, :, None, None]), 0.0)
            dst[:] = np.where(live_mask[..., None], np.clip(r, -127, 127), 0).astype(np.int8)
        case.k, case.v, case.k_scale, case.v_scale = k8, v8, ks, vs
    else:
        dt = NP_DTYPE[kv_type]
        case.k, case.v = k32.astype(dt), v32.astype(dt)
        if dead_fill != 0.0:
            case.k[~live_mask] = dead_fill
            case.v[~live_mask] = dead_fill
    case.extras["k32"], case.extras["v32"] = k32, v32
    return case
