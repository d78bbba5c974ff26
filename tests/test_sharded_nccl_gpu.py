"""Sharded decode on two GPUs, through bench.py's own measured path: each rank builds its shard of
the step (kv_cache_bench_b200.workload.DeviceStep: sequences by LPT bin packing, or KV heads) and
replays CUDA graphs that hold the step, with either gather: the decode kernel writing every output
row into both ranks' global buffers over peer memory plus the step barrier (the default), or the
NCCL all-gather and the reorder into global order. Rank 0 saves both gathered outputs. Every
sequence is then compared with the fp64 oracle on the unsharded data (the values are keyed by
sequence and head, so the shards are slices of the one-GPU step), and the two gathers must agree
bit for bit. Needs two GPUs; skipped on one."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

import oracle
from kv_cache_bench_b200.workload import DeviceStep, config

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")]
TOL = 2e-5
CASES = [(4, "f16", 16), (5, "i8", 6), (5, "f16", 4)]  # config, storage, first N sequences


def _reduced(cfg, dtype, nseq):
    w = config(cfg, dtype)
    w["lens"], w["cut"] = w["lens"][:nseq], True
    return w


def _worker(rank, world, port, out_dir):
    import sys
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import bench
    import kv_cache_bench_b200 as kvb
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=device)
    try:
        ctx = bench.Ctx(torch, dist, rank, world, device)
        for how in ("nccl", "kernel"):
            args = bench.parse_args(["--gpus", str(world), "--steps", "3", "--warmup", "3", "--gather", how])
            for cfg, dtype, nseq in CASES:
                m = bench.measure(ctx, _reduced(cfg, dtype, nseq), args, part=0, kernel=kvb.Kernel.auto, copies=1)
                assert m["flag"] == 0
                assert m["gather"].fused == (how == "kernel")
                final = m["gather"].final.cpu().numpy()
                if rank == 0:
                    np.save(os.path.join(out_dir, f"{cfg}_{dtype}_{how}.npy"), final)
                m["gather"].close()
                del m
                torch.cuda.empty_cache()
    finally:
        dist.barrier()
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(900)
def test_two_gpu_sharded_steps_match_the_unsharded_oracle(tmp_path):
    import torch.multiprocessing as mp
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    kvt = {"f16": oracle.F16, "i8": oracle.I8}
    for cfg, dtype, nseq in CASES:
        final = np.load(tmp_path / f"{cfg}_{dtype}_kernel.npy")
        assert np.array_equal(final, np.load(tmp_path / f"{cfg}_{dtype}_nccl.npy"), equal_nan=True)
        s = DeviceStep(torch, _reduced(cfg, dtype, nseq), device=torch.device("cuda", 0))  # the unsharded step
        assert final.shape == tuple(s.q.shape)
        for i in range(len(s.lens)):
            q, k, v, table, lens, ks, vs = s.sequence_pages(torch, i)
            ref = oracle.paged_attention(q, k, v, table, lens, num_kv_heads=s.Hkv, page=s.page, kv_type=kvt[dtype],
                                         k_scale=ks, v_scale=vs)
            err = oracle.max_abs_diff(final[i:i + 1], ref)
            assert err <= TOL, (cfg, dtype, i, err)
        del s
        torch.cuda.empty_cache()
