"""Seeded synthetic decode steps of BASELINE.json's five configs, built on the device.

The device counterpart of the reference's ``src/workload.hpp`` (``Workload`` + ``PagedCache``):
q ~ U(-1, 1); K and V ~ U(-1, 1) generated in fp32; an fp16 cache holds their round-to-nearest
halves; an int8 cache is quantized per (page, KV head) from the fp32 values by
``kvb_quantize_paged_i8``, which is bit-identical to the reference's ``quantize_to_paged_i8``
(``src/reference.cpp:32-51``); fp32 and fp16 pages are written by ``kvb_scatter_paged``
(``src/reference.hpp:60-68``). Block tables are seeded shuffles of a pool with slack
(``src/reference.cpp:11-30``, plus the configs' 2x / 1.1x pools).

The values are keyed by the logical position, not by where they are stored: the K (V) rows of
sequence b, KV head h come from their own Philox stream seeded by (config seed, b, h, K/V), and q
from one stream over the whole batch. So a rank that holds some of the sequences (sharding by
sequence) or some of the KV heads (sharding by KV head) holds exactly its slice of the one-GPU
step's data, whatever its physical page layout; the outputs of the shards can be compared with the
unsharded reference.

``torch`` is only the allocator and random-number source here; the pages are written by the
library's own CUDA kernels.
"""
from __future__ import annotations

import math
from typing import List, Optional, Sequence

import numpy as np

ELEM = {"f32": 4, "f16": 2, "i8": 1}


# ---- the configs --------------------------------------------------------------------------------

def config(cfg: int, dtype: Optional[str] = None) -> dict:
    """BASELINE.json config `cfg` (1-5): shape, storage type, lengths, page, pool, partition, seed and
    how it shards across GPUs ("replica": every rank runs the whole step)."""
    if cfg == 1:
        w = dict(H=32, Hkv=8, D=128, kv="f32", lens=[512], page=16, pool_blocks=64, part=0, seed=1,
                 shard="replica")
    elif cfg == 2:
        w = dict(H=32, Hkv=8, D=128, kv="f16", lens=[4096], page=32, pool_blocks=256, part=512, seed=2,
                 shard="replica")
    elif cfg == 3:
        w = dict(H=32, Hkv=8, D=128, kv="i8", lens=[32768], page=128, pool_blocks=512, part=0, seed=3,
                 shard="replica")
    elif cfg == 4:
        rng = np.random.default_rng(4)
        lens = np.rint(np.exp(rng.uniform(math.log(512), math.log(32768), 64))).astype(int).tolist()
        w = dict(H=32, Hkv=8, D=128, kv="f16", lens=lens, page=16, pool_slack=1.1, part=0, seed=4,
                 shard="sequence")
    elif cfg == 5:
        rng = np.random.default_rng(5)
        lens = rng.integers(8192, 131072, 256, endpoint=True).tolist()
        w = dict(H=64, Hkv=8, D=128, kv="f16", lens=lens, page=64, pool_slack=1.0, part=0, seed=5,
                 shard="kv_head")
    else:
        raise ValueError(f"unknown config {cfg}")
    if dtype:
        w["kv"] = dtype
    w["cfg"] = cfg
    return w


def min_bytes(w: dict, lens: Sequence[int], Hkv: int, H: int) -> float:
    """Bytes a step must move (src/workload.hpp:69-74): K and V of every live token, q and out."""
    return float(sum(lens)) * Hkv * w["D"] * 2 * ELEM[w["kv"]] + float(len(lens)) * H * w["D"] * 8


def build_layout(lens: Sequence[int], page: int, slack: float, pool_blocks: Optional[int], rng):
    """Block table [B][max_blocks] (-1 unused) over a shuffled pool: `pool_blocks` blocks, or
    ceil(live * slack); physical blocks handed out in sequence order (src/reference.cpp:11-30)."""
    nblk = [(int(l) + page - 1) // page for l in lens]
    live = sum(nblk)
    num_blocks = pool_blocks if pool_blocks else max(live, int(math.ceil(live * slack)))
    num_blocks = max(num_blocks, live, 1)
    perm = rng.permutation(num_blocks).astype(np.int32)
    max_blocks = max(nblk) if nblk else 0
    table = np.full((len(lens), max(max_blocks, 1)), -1, np.int32)
    nxt = 0
    for b, n in enumerate(nblk):
        table[b, :n] = perm[nxt:nxt + n]
        nxt += n
    return table, num_blocks


def kv_seed(w: dict, which: int, b: int, h: int) -> int:
    """Philox seed of the K (which 0) or V (which 1) rows of global sequence b, KV head h."""
    return (((w["seed"] * 1_000_003 + b) * 1031 + h) * 2 + which) & 0x7FFF_FFFF_FFFF_FFFF


def q_seed(w: dict) -> int:
    return (w["seed"] * 7919 + 17) & 0x7FFF_FFFF_FFFF_FFFF


def fp32_rows(torch, w: dict, which: int, b: int, heads: Sequence[int], length: int, device, out=None):
    """The fp32 K or V values of sequence b for KV heads `heads`: [len(heads)][length][D] on the
    device (written into `out`'s storage when given)."""
    D = w["D"]
    n = len(heads) * length * D
    buf = out[:n] if out is not None else torch.empty(n, dtype=torch.float32, device=device)
    rows = buf.view(len(heads), length, D)
    g = torch.Generator(device=device)
    for j, h in enumerate(heads):
        g.manual_seed(kv_seed(w, which, b, h))
        rows[j].view(-1).uniform_(-1.0, 1.0, generator=g)
    return rows


def full_q(torch, w: dict, device):
    """q [B][H][D] of the whole (unsharded) step."""
    g = torch.Generator(device=device)
    g.manual_seed(q_seed(w))
    return torch.empty((len(w["lens"]), w["H"], w["D"]), dtype=torch.float32, device=device).uniform_(
        -1.0, 1.0, generator=g)


# ---- one rank's share of a step -------------------------------------------------------------------

class DeviceStep:
    """What one rank holds and computes for config `w`, on `device`.

    seqs: global ids of the sequences this rank decodes (ascending); kv_heads: the global KV heads it
    holds. q [B_r][H_r][D], table [B_r][max_blocks], seq_lens [B_r], out [B_r][H_r][D]; `pools`
    holds `copies` copies of (k, v, k_scale, v_scale) with identical contents (steps rotate through
    them so that their reads miss L2).
    """

    def __init__(self, torch, w: dict, *, device, rank: int = 0, world: int = 1, copies: int = 1):
        from . import KvType, page_write_args, quantize_paged_i8, scatter_paged
        from . import shard as sh

        self.w, self.rank, self.world, self.device = w, rank, world, device
        lens_all = [int(x) for x in w["lens"]]
        H, Hkv, D, page = w["H"], w["Hkv"], w["D"], w["page"]
        G = H // Hkv
        self.seqs: List[int] = list(range(len(lens_all)))
        self.kv_heads: List[int] = list(range(Hkv))
        self.owned = None
        layout_seed = w["seed"] * 1000
        if w["shard"] == "sequence" and world > 1:
            self.owned = sh.lpt_assign(lens_all, world)
            self.seqs = self.owned[rank]
            layout_seed += rank + 1
        if w["shard"] == "kv_head" and world > 1:
            self.kv_heads = list(sh.kv_head_ranges(Hkv, world)[rank])
        self.Hkv = len(self.kv_heads)
        self.H = self.Hkv * G
        self.D, self.page, self.kv = D, page, w["kv"]
        self.lens = [lens_all[b] for b in self.seqs]
        self.max_len = max(self.lens) if self.lens else 0
        table, self.num_blocks = build_layout(self.lens, page, w.get("pool_slack", 1.0), w.get("pool_blocks"),
                                              np.random.default_rng(layout_seed))
        self.table_host = table
        q = full_q(torch, w, device)
        h0 = self.kv_heads[0] * G if self.kv_heads else 0
        self.q = q[self.seqs][:, h0:h0 + self.H].contiguous() if self.seqs else q[:0, :self.H].contiguous()
        del q
        self.table = torch.from_numpy(table).to(device)
        self.seq_lens = torch.tensor(self.lens, dtype=torch.int32, device=device)
        self.out = torch.zeros_like(self.q)
        self.bytes = min_bytes(w, self.lens, self.Hkv, self.H)
        self.live_pool_bytes = float(sum(self.lens)) * self.Hkv * D * 2 * ELEM[self.kv]

        pdt = {"f32": torch.float32, "f16": torch.float16, "i8": torch.int8}[self.kv]
        shape = (self.num_blocks, self.Hkv, page, D)
        k = torch.zeros(shape, dtype=pdt, device=device)
        v = torch.zeros(shape, dtype=pdt, device=device)
        ks = vs = None
        if self.kv == "i8":
            ks = torch.zeros((self.num_blocks, self.Hkv), dtype=torch.float32, device=device)
            vs = torch.zeros_like(ks)
        longest = self.max_len * self.Hkv * D
        scratch = torch.empty(max(longest, 1), dtype=torch.float32, device=device)
        half = torch.empty(max(longest, 1), dtype=torch.float16, device=device) if self.kv == "f16" else None
        kvt = KvType[self.kv]
        stream = torch.cuda.current_stream(device).cuda_stream
        for i, b in enumerate(self.seqs):
            L = self.lens[i]
            if L == 0:
                continue
            for which, pool, sc in ((0, k, ks), (1, v, vs)):
                rows = fp32_rows(torch, w, which, b, self.kv_heads, L, device, out=scratch)
                src = rows
                if self.kv == "f16":
                    src = half[:rows.numel()].view(rows.shape)
                    src.copy_(rows)  # round to nearest even, as the reference's fp32 -> half
                a = page_write_args(1, self.Hkv, D, kvt, page, table.shape[1], L, contig=src.data_ptr(),
                                    block_table=self.table[i].data_ptr(), seq_lens=self.seq_lens[i].data_ptr(),
                                    pool=pool.data_ptr(), num_blocks=self.num_blocks,
                                    scales=sc.data_ptr() if sc is not None else 0)
                (quantize_paged_i8 if self.kv == "i8" else scatter_paged)(a, stream)
        del scratch, half
        self.pools = [(k, v, ks, vs)]
        for _ in range(1, copies):
            self.pools.append(tuple(t.clone() if t is not None else None for t in (k, v, ks, vs)))
        torch.cuda.synchronize(device)

    # -- host copies of one sequence, for checking against the fp64 oracle ---------------------------

    def sequence_pages(self, torch, i: int, copy: int = 0):
        """Sequence i's live pages as a compact host step: (q [1][H_r][D], k, v, table [1][n], lens [1],
        k_scale, v_scale), pages renumbered 0..n-1 in table order."""
        L = self.lens[i]
        n = (L + self.page - 1) // self.page
        ids = self.table[i, :n].long()
        k, v, ks, vs = self.pools[copy]
        host = lambda t: t.index_select(0, ids).cpu().numpy() if t is not None else None  # noqa: E731
        return (self.q[i:i + 1].cpu().numpy(), host(k), host(v), np.arange(n, dtype=np.int32)[None, :],
                np.asarray([L], np.int32), host(ks), host(vs))

    def sequence_fp32(self, torch, i: int):
        """The unrounded fp32 K and V of sequence i: [1][Hkv_r][len][D] each, on the host."""
        b, L = self.seqs[i], self.lens[i]
        kr = fp32_rows(torch, self.w, 0, b, self.kv_heads, L, self.device).cpu().numpy()[None]
        vr = fp32_rows(torch, self.w, 1, b, self.kv_heads, L, self.device).cpu().numpy()[None]
        return kr, vr
