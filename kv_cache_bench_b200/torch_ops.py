"""Torch-facing convenience over the stream-level C ABI.

``PagedDecoder`` launches ``kvb_paged_decode_async`` on torch's current CUDA stream with torch
tensors as device buffers; torch is only the allocator and stream here, the work is the library's
CUDA kernels.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import Kernel, KvType, Shape, device_args, paged_decode_async, paged_error_flag, paged_part_tokens, \
    paged_workspace_bytes

_KV_DTYPE = {KvType.f32: torch.float32, KvType.f16: torch.float16, KvType.i8: torch.int8}


def kv_type_of(t: torch.Tensor) -> KvType:
    for k, v in _KV_DTYPE.items():
        if t.dtype == v:
            return k
    raise ValueError(f"unsupported cache dtype {t.dtype}")


class PagedDecoder:
    """One decode step per call over a paged cache held in torch tensors.

    q: float32 [B][H][D]; k_pool, v_pool: [num_blocks][Hkv][page][D] (float32, float16 or int8);
    block_table: int32 [B][max_blocks]; seq_lens: int32 [B]; k_scale, v_scale: float32
    [num_blocks][Hkv] for int8. The workspace is owned by the decoder (grown and zeroed on demand);
    calls on one decoder must not overlap on the device.
    """

    def __init__(self, device: Optional[torch.device] = None):
        self.device = torch.device(device or torch.device("cuda", torch.cuda.current_device()))
        self.workspace = torch.zeros(256, dtype=torch.uint8, device=self.device)

    def args(self, q, k_pool, v_pool, block_table, seq_lens, max_len, *, out, k_scale=None, v_scale=None,
             part_tokens=0, share_kv=True, kernel=Kernel.auto, tables_ready=False, inputs_ready=False,
             step_stream=False):
        B, H, D = q.shape
        num_blocks, Hkv, page, D2 = k_pool.shape
        if D2 != D or v_pool.shape != k_pool.shape:
            raise ValueError("pool shapes do not match q")
        for t in (q, k_pool, v_pool, block_table, seq_lens, out):
            if not t.is_contiguous() or t.device != self.device:
                raise ValueError("tensors must be contiguous and on the decoder's device")
        kvt = kv_type_of(k_pool)
        return device_args(Shape(B, H, Hkv, D), kvt, page, block_table.shape[1], int(max_len), q=q.data_ptr(),
                           k=k_pool.data_ptr(), v=v_pool.data_ptr(), block_table=block_table.data_ptr(),
                           seq_lens=seq_lens.data_ptr(), out=out.data_ptr(), num_blocks=num_blocks,
                           part_tokens=part_tokens, share_kv=share_kv,
                           k_scale=k_scale.data_ptr() if k_scale is not None else 0,
                           v_scale=v_scale.data_ptr() if v_scale is not None else 0, kernel=kernel,
                           tables_ready=tables_ready, inputs_ready=inputs_ready, step_stream=step_stream)

    def __call__(self, q, k_pool, v_pool, block_table, seq_lens, max_len, *, k_scale=None, v_scale=None,
                 part_tokens=0, share_kv=True, kernel=Kernel.auto, out=None, stream=None, tables_ready=False,
                 inputs_ready=False, step_stream=False):
        if out is None:
            out = torch.empty_like(q)
        c = self.args(q, k_pool, v_pool, block_table, seq_lens, max_len, out=out, k_scale=k_scale,
                      v_scale=v_scale, part_tokens=part_tokens, share_kv=share_kv, kernel=kernel,
                      tables_ready=tables_ready, inputs_ready=inputs_ready, step_stream=step_stream)
        need = paged_workspace_bytes(c)
        if need > self.workspace.numel():
            self.workspace = torch.zeros(need, dtype=torch.uint8, device=self.device)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        paged_decode_async(c, self.workspace.data_ptr(), self.workspace.numel(), s.cuda_stream)
        return out

    def part_tokens(self, q, k_pool, v_pool, block_table, seq_lens, max_len, **kw) -> int:
        out = torch.empty_like(q)
        return paged_part_tokens(self.args(q, k_pool, v_pool, block_table, seq_lens, max_len, out=out, **kw))

    def error_flag(self, stream=None) -> int:
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        return paged_error_flag(self.workspace.data_ptr(), s.cuda_stream)
