"""Host-side sharding of batched decode (kv_cache_bench_b200/shard.py) and the gather that puts the
per-rank outputs back in global order, checked against the unsharded fp64 oracle. The world-size-2
tests run two gloo ranks on the CPU; each rank decodes its shard with the oracle standing in for the
GPU kernel, so what is tested is the partitioning and the all-gather/permutation logic."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from kv_cache_bench_b200 import shard as sh


def test_lpt_assign_balances_and_covers_every_sequence():
    rng = np.random.default_rng(4)
    lens = np.rint(np.exp(rng.uniform(np.log(512), np.log(32768), 64))).astype(int)
    for n in (1, 2, 4, 8):
        owned = sh.lpt_assign(lens, n)
        assert sorted(b for o in owned for b in o) == list(range(64))
        assert all(o == sorted(o) for o in owned)
        # LPT bound: max load <= mean + longest item
        loads = [int(lens[o].sum()) for o in owned]
        assert max(loads) <= lens.sum() / n + lens.max()
        assert sh.imbalance(lens, owned) < (1.02 if n <= 4 else 1.1)


def test_lpt_assign_ties_and_edges():
    assert sh.lpt_assign([5, 5, 5, 5], 2) == [[0, 2], [1, 3]]
    assert sh.lpt_assign([], 3) == [[], [], []]
    assert sh.lpt_assign([7], 4) == [[0], [], [], []]
    with pytest.raises(ValueError):
        sh.lpt_assign([1], 0)


def test_kv_head_ranges():
    assert sh.kv_head_ranges(8, 8) == [range(r, r + 1) for r in range(8)]
    assert sh.kv_head_ranges(8, 2) == [range(0, 4), range(4, 8)]
    with pytest.raises(ValueError):
        sh.kv_head_ranges(8, 3)


def test_sequence_gather_index_inverts_the_assignment():
    owned = [[1, 4], [0], [2, 3, 5]]
    pad = 3
    idx = sh.sequence_gather_index(owned, pad)
    rows = np.full(len(owned) * pad, -1)
    for r, o in enumerate(owned):
        rows[r * pad: r * pad + len(o)] = o
    assert (rows[idx] == np.arange(6)).all()


def _shard_outputs(case, mode, rank, world):
    """Decode rank `rank`'s shard of `case` with the oracle: [B_r][H][D] (sequence) or
    [B][H/world][D] (KV head)."""
    if mode == "sequence":
        o = sh.lpt_assign(case.lens, world)[rank]
        return oracle.paged_attention(case.q[o], case.k, case.v, case.table[o], case.lens[o],
                                      num_kv_heads=case.num_kv_heads, page=case.page, kv_type=case.kv_type,
                                      k_scale=case.k_scale, v_scale=case.v_scale, threads=1)
    heads = sh.kv_head_ranges(case.num_kv_heads, world)[rank]
    G = case.q.shape[1] // case.num_kv_heads
    qh = slice(heads.start * G, heads.stop * G)
    ks = case.k_scale[:, heads.start:heads.stop] if case.k_scale is not None else None
    vs = case.v_scale[:, heads.start:heads.stop] if case.v_scale is not None else None
    return oracle.paged_attention(case.q[:, qh], case.k[:, heads.start:heads.stop],
                                  case.v[:, heads.start:heads.stop], case.table, case.lens,
                                  num_kv_heads=len(heads), page=case.page, kv_type=case.kv_type,
                                  k_scale=ks, v_scale=vs, threads=1)


def _make(kv_type):
    return oracle.make_case(num_heads=16, num_kv_heads=4, head_dim=64, lens=[300, 0, 41, 1000, 64, 7, 513],
                            kv_type=kv_type, page=16, seed=11)


def _worker(rank, world, port, mode, kv_type, result_path):
    import torch
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = _make(kv_type)
        out = torch.from_numpy(_shard_outputs(case, mode, rank, world))
        if mode == "sequence":
            owned = sh.lpt_assign(case.lens, world)
            pad = max(len(o) for o in owned)
            local = torch.zeros((pad,) + tuple(out.shape[1:]))
            local[: out.shape[0]] = out
            parts = [torch.empty_like(local) for _ in range(world)]
            dist.all_gather(parts, local)
            full = torch.cat(parts)[torch.from_numpy(sh.sequence_gather_index(owned, pad))]
        else:
            parts = [torch.empty_like(out) for _ in range(world)]
            dist.all_gather(parts, out.contiguous())
            full = torch.from_numpy(sh.merge_kv_head_shards(torch.stack(parts).numpy()))
        if rank == 0:
            np.save(result_path, full.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("mode,kv_type", [("sequence", oracle.F16), ("kv_head", oracle.I8), ("kv_head", oracle.F32)])
def test_two_rank_gloo_gather_matches_unsharded(tmp_path, mode, kv_type):
    path = str(tmp_path / "out.npy")
    mp.start_processes(_worker, args=(2, _free_port(), mode, kv_type, path), nprocs=2, join=True,
                       start_method="spawn")
    case = _make(kv_type)
    full = np.load(path)
    assert full.shape == case.q.shape
    # sharding changes only which rank computes a (sequence, head); the oracle is deterministic
    assert np.array_equal(full, case.reference(threads=1))
