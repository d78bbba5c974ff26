"""B200-native paged decode attention: Python host mirror of kv-cache-bench's C++ host API.

The functions and types below mirror ``src/metal_attn.hpp`` of the reference (same names,
argument meaning and error behaviour: ``ValueError`` where the reference throws
``std::invalid_argument``, ``RuntimeError`` where it throws ``std::runtime_error``). They call the
C ABI of ``libkvbcuda.so`` (``include/kvb_cuda.h``) through ctypes; the CUDA kernels behind it are
the only implementation. Importing this package fails if the library has not been built.

Reference API (``src/metal_attn.hpp`` line):
    metal_available (13), device_name (14), Buffer (18-33), KvType/name/elem_size (37-39),
    kSimdGroups (41), auto_part_tokens (47-51), PagedArgs (53-69), NaiveArgs (71-80),
    run_paged (86), run_naive (87), run_paged_steps (91), begin_pipelined/end_pipelined (98-99),
    run_read_bandwidth (102), flush_gpu_caches (106).
Shape is ``src/reference.hpp:17-23``.

Stream-level API (device pointers, no host reads, no allocation): ``paged_workspace_bytes``,
``paged_part_tokens``, ``paged_decode_async``, ``paged_error_flag``; torch conveniences are in
``kv_cache_bench_b200.torch_ops``.
"""
from __future__ import annotations

import ctypes
import enum
import os
from dataclasses import dataclass
from typing import Optional

import numpy as np

__all__ = [
    "Shape", "KvType", "name", "elem_size", "kSimdGroups", "auto_part_tokens", "Buffer", "PagedArgs",
    "NaiveArgs", "metal_available", "device_name", "run_paged", "run_paged_steps", "run_naive",
    "begin_pipelined", "end_pipelined", "run_read_bandwidth", "flush_gpu_caches", "Kernel",
    "paged_workspace_bytes", "paged_part_tokens", "paged_part_tokens_for", "paged_decode_async", "paged_error_flag",
    "paged_decode_static", "paged_static_error_flag", "library_path", "lib", "MAX_PEERS", "ipc_alloc", "ipc_free",
    "ipc_open", "ipc_close", "peer_out", "paged_decode_gather_async", "peer_barrier_args", "peer_barrier_async",
]

_HERE = os.path.dirname(os.path.abspath(__file__))


def library_path() -> str:
    """Path of the in-tree libkvbcuda.so."""
    return os.path.join(_HERE, "libkvbcuda.so")


def _load() -> ctypes.CDLL:
    path = library_path()
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build it with `make -C {_HERE}` (or __graft_entry__.build()); "
            "this package has no fallback implementation")
    return ctypes.CDLL(path)


lib = _load()

# ---- C ABI declarations (include/kvb_cuda.h) ----------------------------------------------------

KVB_OK, KVB_ERR_INVALID, KVB_ERR_DEVICE, KVB_ERR_NO_DEVICE, KVB_ERR_STATE = 0, 1, 2, 3, 4


class _CShape(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int), ("num_heads", ctypes.c_int), ("num_kv_heads", ctypes.c_int),
                ("head_dim", ctypes.c_int)]


class _CPagedArgs(ctypes.Structure):
    _fields_ = [("shape", _CShape), ("kv_type", ctypes.c_int), ("page_size", ctypes.c_int),
                ("max_blocks", ctypes.c_int), ("max_len", ctypes.c_int), ("part_tokens", ctypes.c_int),
                ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
                ("block_table", ctypes.c_void_p), ("seq_lens", ctypes.c_void_p), ("out", ctypes.c_void_p),
                ("share_kv", ctypes.c_int), ("k_scale", ctypes.c_void_p), ("v_scale", ctypes.c_void_p),
                ("num_blocks", ctypes.c_int64), ("kernel", ctypes.c_int), ("flags", ctypes.c_int)]


# kvb_paged_args.flags (include/kvb_cuda.h): the lengths and block table are not written by the kernel
# launched right before the call on its stream, so the tensor-core kernel may read them early.
FLAG_TABLES_READY = 1
# ... and q, the pools and the scales are not written by it either (needs FLAG_TABLES_READY): the
# tensor-core kernel streams the pages while that kernel finishes.
FLAG_INPUTS_READY = 2
# ... and the call is one of a stream of independent steps launched back to back (needs
# FLAG_INPUTS_READY): with few (sequence, head group) pairs, partitions sized for throughput.
FLAG_STEP_STREAM = 4


class _CPageWriteArgs(ctypes.Structure):
    _fields_ = [("shape", _CShape), ("kv_type", ctypes.c_int), ("page_size", ctypes.c_int),
                ("max_blocks", ctypes.c_int), ("max_len", ctypes.c_int), ("contig", ctypes.c_void_p),
                ("block_table", ctypes.c_void_p), ("seq_lens", ctypes.c_void_p), ("pool", ctypes.c_void_p),
                ("scales", ctypes.c_void_p), ("num_blocks", ctypes.c_int64), ("error_word", ctypes.c_void_p)]


class _CNaiveArgs(ctypes.Structure):
    _fields_ = [("shape", _CShape), ("kv_type", ctypes.c_int), ("max_len", ctypes.c_int),
                ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
                ("seq_lens", ctypes.c_void_p), ("out", ctypes.c_void_p)]


def _sig(fn, restype, *argtypes):
    f = getattr(lib, fn)
    f.restype = restype
    f.argtypes = list(argtypes)
    return f


_c_available = _sig("kvb_available", ctypes.c_int)
_c_device_name = _sig("kvb_device_name", ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t)
_c_buffer_alloc = _sig("kvb_buffer_alloc", ctypes.c_int, ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p))
_c_buffer_free = _sig("kvb_buffer_free", ctypes.c_int, ctypes.c_void_p)
_c_run_paged = _sig("kvb_run_paged", ctypes.c_int, ctypes.POINTER(_CPagedArgs), ctypes.c_int,
                    ctypes.POINTER(ctypes.c_double))
_c_run_naive = _sig("kvb_run_naive", ctypes.c_int, ctypes.POINTER(_CNaiveArgs), ctypes.POINTER(ctypes.c_double))
_c_begin_pipelined = _sig("kvb_begin_pipelined", ctypes.c_int)
_c_pipelined_runs = _sig("kvb_pipelined_runs", ctypes.c_int, ctypes.POINTER(ctypes.c_size_t))
_c_end_pipelined = _sig("kvb_end_pipelined", ctypes.c_int, ctypes.POINTER(ctypes.c_double), ctypes.c_size_t,
                        ctypes.POINTER(ctypes.c_size_t))
_c_read_bw = _sig("kvb_read_bandwidth", ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
                  ctypes.POINTER(ctypes.c_double))
_c_flush = _sig("kvb_flush_caches", ctypes.c_int)
_c_auto_part = _sig("kvb_auto_part_tokens", ctypes.c_int, _CShape, ctypes.c_int)
_c_last_error = _sig("kvb_last_error", ctypes.c_char_p)
_c_part_tokens = _sig("kvb_paged_part_tokens", ctypes.c_int, ctypes.POINTER(_CPagedArgs))
_c_part_tokens_for = _sig("kvb_paged_part_tokens_for", ctypes.c_int, ctypes.POINTER(_CPagedArgs),
                          ctypes.POINTER(ctypes.c_int32))
_c_ws_bytes = _sig("kvb_paged_workspace_bytes", ctypes.c_int, ctypes.POINTER(_CPagedArgs),
                   ctypes.POINTER(ctypes.c_size_t))
_c_decode_async = _sig("kvb_paged_decode_async", ctypes.c_int, ctypes.POINTER(_CPagedArgs), ctypes.c_void_p,
                       ctypes.c_size_t, ctypes.c_void_p)
_c_quantize = _sig("kvb_quantize_paged_i8", ctypes.c_int, ctypes.POINTER(_CPageWriteArgs), ctypes.c_void_p)
_c_scatter = _sig("kvb_scatter_paged", ctypes.c_int, ctypes.POINTER(_CPageWriteArgs), ctypes.c_void_p)
_c_decode_static = _sig("kvb_paged_decode_static", ctypes.c_int, ctypes.POINTER(_CPagedArgs), ctypes.c_void_p)
_c_error_flag = _sig("kvb_paged_error_flag", ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                     ctypes.POINTER(ctypes.c_int))
_c_static_error_flag = _sig("kvb_paged_static_error_flag", ctypes.c_int, ctypes.c_void_p,
                            ctypes.POINTER(ctypes.c_int))


def _check(rc: int, what: str) -> None:
    if rc == KVB_OK:
        return
    msg = f"{what}: {_c_last_error().decode(errors='replace')}"
    if rc == KVB_ERR_INVALID:
        raise ValueError(msg)
    raise RuntimeError(msg)


# ---- reference types ------------------------------------------------------------------------------

@dataclass
class Shape:
    """One decode step's shape (src/reference.hpp:17-23)."""
    batch: int = 1
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128

    def group(self) -> int:
        return self.num_heads // self.num_kv_heads

    def _c(self) -> _CShape:
        return _CShape(self.batch, self.num_heads, self.num_kv_heads, self.head_dim)


class KvType(enum.IntEnum):
    """Storage type of the cache (src/metal_attn.hpp:37)."""
    f32 = 0
    f16 = 1
    i8 = 2


class Kernel(enum.IntEnum):
    """Kernel choice of kvb_paged_args.kernel (include/kvb_cuda.h)."""
    auto = 0
    simt = 1
    mma = 2
    umma = 3


def name(t: KvType) -> str:
    return {KvType.f32: "f32", KvType.f16: "f16", KvType.i8: "i8"}[KvType(t)]


def elem_size(t: KvType) -> int:
    return {KvType.f32: 4, KvType.f16: 2, KvType.i8: 1}[KvType(t)]


kSimdGroups = 4  # the reference kernel's simdgroups per threadgroup (src/metal_attn.hpp:41)


def auto_part_tokens(s: Shape, max_len: int) -> int:
    """The reference's split-K rule (src/metal_attn.hpp:47-51), computed by the library."""
    return int(_c_auto_part(s._c(), int(max_len)))


def metal_available() -> bool:
    """True when a CUDA device is usable (src/metal_attn.hpp:13)."""
    return _c_available() == 1


def device_name() -> str:
    buf = ctypes.create_string_buffer(256)
    return buf.value.decode() if _c_device_name(buf, 256) == KVB_OK else ""


class Buffer:
    """Host-visible, device-usable memory (src/metal_attn.hpp:18-33): CUDA managed memory.

    ``data()`` is the pointer, ``as_array(dtype)`` a numpy view the host fills in place, as the
    reference fills its shared-storage MTLBuffers.
    """

    def __init__(self, nbytes: int):
        self._bytes = int(nbytes)
        ptr = ctypes.c_void_p()
        _check(_c_buffer_alloc(self._bytes, ctypes.byref(ptr)), "Buffer")
        self._ptr = ptr.value

    def __del__(self):
        if getattr(self, "_ptr", None):
            _c_buffer_free(self._ptr)
            self._ptr = None

    def data(self) -> int:
        return self._ptr

    def handle(self) -> int:
        return self._ptr

    def size(self) -> int:
        return self._bytes

    def as_array(self, dtype, count: Optional[int] = None) -> np.ndarray:
        dt = np.dtype(dtype)
        n = self._bytes // dt.itemsize if count is None else int(count)
        raw = (ctypes.c_uint8 * max(n * dt.itemsize, 1)).from_address(self._ptr)
        return np.frombuffer(raw, dtype=dt, count=n)

    @classmethod
    def from_array(cls, a: np.ndarray) -> "Buffer":
        a = np.ascontiguousarray(a)
        b = cls(a.nbytes)
        if a.nbytes:
            b.as_array(a.dtype, a.size)[:] = a.reshape(-1)
        return b


@dataclass
class PagedArgs:
    """Arguments of one paged decode step (src/metal_attn.hpp:53-69), same field order.

    ``num_blocks`` (pool size) defaults to what the K buffer holds; ``kernel`` selects the kernel.
    """
    shape: Shape
    type: KvType = KvType.f32
    page_size: int = 16
    max_blocks: int = 0
    max_len: int = 0
    part_tokens: int = 0
    q: Optional[Buffer] = None
    k: Optional[Buffer] = None
    v: Optional[Buffer] = None
    block_table: Optional[Buffer] = None
    seq_lens: Optional[Buffer] = None
    out: Optional[Buffer] = None
    share_kv: bool = True
    k_scale: Optional[Buffer] = None
    v_scale: Optional[Buffer] = None
    num_blocks: Optional[int] = None
    kernel: Kernel = Kernel.auto

    def _c(self) -> _CPagedArgs:
        s = self.shape
        nb = self.num_blocks
        if nb is None:
            per = max(self.page_size, 0) * max(s.num_kv_heads, 0) * max(s.head_dim, 0) * elem_size(self.type)
            nb = (self.k.size() // per) if (self.k is not None and per) else 0
        ptr = lambda b: b.handle() if b is not None else None  # noqa: E731
        return _CPagedArgs(s._c(), int(self.type), self.page_size, self.max_blocks, self.max_len, self.part_tokens,
                           ptr(self.q), ptr(self.k), ptr(self.v), ptr(self.block_table), ptr(self.seq_lens),
                           ptr(self.out), 1 if self.share_kv else 0, ptr(self.k_scale), ptr(self.v_scale),
                           int(nb), int(self.kernel))


@dataclass
class NaiveArgs:
    """Arguments of the naive baseline (src/metal_attn.hpp:71-80): contiguous [B][Hkv][max_len][D]."""
    shape: Shape
    type: KvType = KvType.f32
    max_len: int = 0
    q: Optional[Buffer] = None
    k: Optional[Buffer] = None
    v: Optional[Buffer] = None
    seq_lens: Optional[Buffer] = None
    out: Optional[Buffer] = None

    def _c(self) -> _CNaiveArgs:
        ptr = lambda b: b.handle() if b is not None else None  # noqa: E731
        return _CNaiveArgs(self.shape._c(), int(self.type), self.max_len, ptr(self.q), ptr(self.k), ptr(self.v),
                           ptr(self.seq_lens), ptr(self.out))


def run_paged_steps(a: PagedArgs, steps: int) -> float:
    """``steps`` decode steps back to back; device milliseconds (0 in pipelined mode)."""
    ms = ctypes.c_double()
    c = a._c()
    _check(_c_run_paged(ctypes.byref(c), int(steps), ctypes.byref(ms)), "run_paged")
    return ms.value


def run_paged(a: PagedArgs) -> float:
    return run_paged_steps(a, 1)


def run_naive(a: NaiveArgs) -> float:
    ms = ctypes.c_double()
    c = a._c()
    _check(_c_run_naive(ctypes.byref(c), ctypes.byref(ms)), "run_naive")
    return ms.value


def begin_pipelined() -> None:
    _check(_c_begin_pipelined(), "begin_pipelined")


def end_pipelined() -> list:
    n = ctypes.c_size_t()
    _check(_c_pipelined_runs(ctypes.byref(n)), "end_pipelined")
    arr = (ctypes.c_double * max(n.value, 1))()
    _check(_c_end_pipelined(arr, n.value, ctypes.byref(n)), "end_pipelined")
    return [arr[i] for i in range(n.value)]


def run_read_bandwidth(src: Buffer) -> float:
    ms = ctypes.c_double()
    _check(_c_read_bw(src.handle(), src.size(), ctypes.byref(ms)), "run_read_bandwidth")
    return ms.value


def flush_gpu_caches() -> None:
    _check(_c_flush(), "flush_gpu_caches")


# ---- stream level ---------------------------------------------------------------------------------

def device_args(shape: Shape, kv_type: KvType, page_size: int, max_blocks: int, max_len: int, *, q: int, k: int,
                v: int, block_table: int, seq_lens: int, out: int, num_blocks: int, part_tokens: int = 0,
                share_kv: bool = True, k_scale: int = 0, v_scale: int = 0,
                kernel: Kernel = Kernel.auto, tables_ready: bool = False, inputs_ready: bool = False,
                step_stream: bool = False) -> _CPagedArgs:
    """kvb_paged_args over raw device pointers (ints). tables_ready sets FLAG_TABLES_READY;
    inputs_ready sets FLAG_INPUTS_READY as well; step_stream sets FLAG_STEP_STREAM and both others."""
    return _CPagedArgs(shape._c(), int(kv_type), page_size, max_blocks, max_len, part_tokens, q or None, k or None,
                       v or None, block_table or None, seq_lens or None, out or None, 1 if share_kv else 0,
                       k_scale or None, v_scale or None, int(num_blocks), int(kernel),
                       (FLAG_TABLES_READY if tables_ready or inputs_ready or step_stream else 0)
                       | (FLAG_INPUTS_READY if inputs_ready or step_stream else 0)
                       | (FLAG_STEP_STREAM if step_stream else 0))


def paged_workspace_bytes(c: _CPagedArgs) -> int:
    n = ctypes.c_size_t()
    _check(_c_ws_bytes(ctypes.byref(c), ctypes.byref(n)), "paged_workspace_bytes")
    return n.value


def paged_part_tokens(c: _CPagedArgs) -> int:
    r = _c_part_tokens(ctypes.byref(c))
    if r < 0:
        _check(-r, "paged_part_tokens")
    return r


def paged_part_tokens_for(c: _CPagedArgs, lens) -> int:
    """kvb_paged_part_tokens_for: the partition size for these host-side sequence lengths."""
    if len(lens) < c.shape.batch:
        raise ValueError(f"paged_part_tokens_for: {len(lens)} lengths for a batch of {c.shape.batch}")
    arr = (ctypes.c_int32 * max(1, len(lens)))(*[int(x) for x in lens])
    r = _c_part_tokens_for(ctypes.byref(c), arr)
    if r < 0:
        _check(-r, "paged_part_tokens_for")
    return r


def paged_decode_async(c: _CPagedArgs, workspace: int, workspace_bytes: int, stream: int = 0) -> None:
    _check(_c_decode_async(ctypes.byref(c), workspace or None, int(workspace_bytes), stream or None),
           "paged_decode_async")


def paged_decode_static(c: _CPagedArgs, stream: int = 0) -> None:
    """kvb_paged_decode_static: one decode step with the library-owned workspace (no allocation)."""
    _check(_c_decode_static(ctypes.byref(c), stream or None), "paged_decode_static")


def paged_static_error_flag(stream: int = 0) -> int:
    """kvb_paged_static_error_flag: reads and clears the library-owned workspace's error word on the
    current device (and resets its counters after a TIMEOUT or STATE bit)."""
    f = ctypes.c_int()
    _check(_c_static_error_flag(stream or None, ctypes.byref(f)), "paged_static_error_flag")
    return f.value


STATIC_WORKSPACE_BYTES = 16 << 20


# ---- page write path (src/reference.cpp:32-51, src/reference.hpp:60-68) ----------------------------

def page_write_args(batch: int, num_kv_heads: int, head_dim: int, kv_type: KvType, page_size: int, max_blocks: int,
                    max_len: int, *, contig: int, block_table: int, seq_lens: int, pool: int, num_blocks: int,
                    scales: int = 0, error_word: int = 0) -> _CPageWriteArgs:
    """kvb_page_write_args over raw device pointers (ints)."""
    return _CPageWriteArgs(_CShape(batch, num_kv_heads, num_kv_heads, head_dim), int(kv_type), page_size, max_blocks,
                           max_len, contig or None, block_table or None, seq_lens or None, pool or None,
                           scales or None, int(num_blocks), error_word or None)


def quantize_paged_i8(a: _CPageWriteArgs, stream: int = 0) -> None:
    """kvb_quantize_paged_i8: the reference's per-(page, KV head) absmax/127 quantizer on the device."""
    _check(_c_quantize(ctypes.byref(a), stream or None), "quantize_paged_i8")


def scatter_paged(a: _CPageWriteArgs, stream: int = 0) -> None:
    """kvb_scatter_paged: the reference's scatter_to_paged on the device (fp32 / fp16)."""
    _check(_c_scatter(ctypes.byref(a), stream or None), "scatter_paged")


def paged_error_flag(workspace: int, stream: int = 0) -> int:
    f = ctypes.c_int()
    _check(_c_error_flag(workspace or None, stream or None, ctypes.byref(f)), "paged_error_flag")
    return f.value


# ---- sharded steps gathered in the kernel (include/kvb_cuda.h, "sharded steps") ---------------------

MAX_PEERS = 8


class _CIpcHandle(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


class _CPeerOut(ctypes.Structure):
    _fields_ = [("n_peers", ctypes.c_int), ("self", ctypes.c_int), ("rows", ctypes.c_int),
                ("out_heads", ctypes.c_int), ("out_head0", ctypes.c_int), ("out_rows", ctypes.c_void_p),
                ("peer_out", ctypes.c_void_p * MAX_PEERS)]


class _CPeerBarrierArgs(ctypes.Structure):
    _fields_ = [("n_peers", ctypes.c_int), ("rank", ctypes.c_int), ("timeout_us", ctypes.c_uint),
                ("epoch", ctypes.c_void_p), ("signal", ctypes.c_void_p * MAX_PEERS)]


_c_ipc_alloc = _sig("kvb_ipc_alloc", ctypes.c_int, ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p),
                    ctypes.POINTER(_CIpcHandle))
_c_ipc_free = _sig("kvb_ipc_free", ctypes.c_int, ctypes.c_void_p)
_c_ipc_open = _sig("kvb_ipc_open", ctypes.c_int, ctypes.POINTER(_CIpcHandle), ctypes.POINTER(ctypes.c_void_p))
_c_ipc_close = _sig("kvb_ipc_close", ctypes.c_int, ctypes.c_void_p)
_c_decode_gather = _sig("kvb_paged_decode_gather_async", ctypes.c_int, ctypes.POINTER(_CPagedArgs),
                        ctypes.POINTER(_CPeerOut), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p)
_c_peer_barrier = _sig("kvb_peer_barrier_async", ctypes.c_int, ctypes.POINTER(_CPeerBarrierArgs), ctypes.c_void_p,
                       ctypes.c_void_p)


def ipc_alloc(nbytes: int):
    """kvb_ipc_alloc: zero-filled device memory another process can map. Returns (pointer, handle
    bytes)."""
    p, h = ctypes.c_void_p(), _CIpcHandle()
    _check(_c_ipc_alloc(int(nbytes), ctypes.byref(p), ctypes.byref(h)), "ipc_alloc")
    return p.value, bytes(h.bytes)


def ipc_free(ptr: int) -> None:
    _check(_c_ipc_free(ptr or None), "ipc_free")


def ipc_open(handle: bytes) -> int:
    """kvb_ipc_open: maps another process's ipc_alloc memory on the current device."""
    h = _CIpcHandle()
    if len(handle) != 64:
        raise ValueError("an IPC handle has 64 bytes")
    ctypes.memmove(h.bytes, handle, 64)
    p = ctypes.c_void_p()
    _check(_c_ipc_open(ctypes.byref(h), ctypes.byref(p)), "ipc_open")
    return p.value


def ipc_close(ptr: int) -> None:
    _check(_c_ipc_close(ptr or None), "ipc_close")


def peer_out(peers, self_index: int, rows: int, out_heads: int, out_head0: int = 0, out_rows: int = 0) -> _CPeerOut:
    """kvb_peer_out: every rank's global output buffer (device pointers, this rank's own at
    self_index), the global rows and heads, and the device array of global rows of the local
    sequences (0: local index = global row)."""
    if not 1 <= len(peers) <= MAX_PEERS:
        raise ValueError(f"1..{MAX_PEERS} peers")
    arr = (ctypes.c_void_p * MAX_PEERS)(*([int(x) for x in peers] + [None] * (MAX_PEERS - len(peers))))
    return _CPeerOut(len(peers), int(self_index), int(rows), int(out_heads), int(out_head0), out_rows or None, arr)


def paged_decode_gather_async(c: _CPagedArgs, peers: _CPeerOut, workspace: int, workspace_bytes: int,
                              stream: int = 0) -> None:
    """kvb_paged_decode_gather_async: a decode step whose outputs the kernel writes into every rank's
    global output buffer."""
    _check(_c_decode_gather(ctypes.byref(c), ctypes.byref(peers), workspace or None, int(workspace_bytes),
                            stream or None), "paged_decode_gather_async")


def peer_barrier_args(rank: int, signals, epoch: int, timeout_us: int = 0) -> _CPeerBarrierArgs:
    """kvb_peer_barrier_args: every rank's signal array (device pointers, in rank order) and this
    rank's epoch word."""
    if not 1 <= len(signals) <= MAX_PEERS:
        raise ValueError(f"1..{MAX_PEERS} peers")
    arr = (ctypes.c_void_p * MAX_PEERS)(*([int(x) for x in signals] + [None] * (MAX_PEERS - len(signals))))
    return _CPeerBarrierArgs(len(signals), int(rank), int(timeout_us), epoch or None, arr)


def peer_barrier_async(b: _CPeerBarrierArgs, workspace: int, stream: int = 0) -> None:
    """kvb_peer_barrier_async: the step barrier after paged_decode_gather_async on every rank; a wait
    that runs out sets bit 4 of the workspace's error word."""
    _check(_c_peer_barrier(ctypes.byref(b), workspace or None, stream or None), "peer_barrier_async")
