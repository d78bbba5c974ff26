"""Host side of the in-kernel gather (kv_cache_bench_b200/peer.py, PeerGather) on two gloo ranks on the
CPU: the IPC calls are replaced by fakes that hand out distinct addresses and handles, so what is
tested is the rendezvous (every rank's handles reach every rank over torch.distributed), the peer
lists in rank order with this rank's own buffer at its index, the barrier arguments, and that
close() unmaps every peer mapping and frees every own allocation."""
import os
import socket
import types

import torch
import torch.multiprocessing as mp

WORLD, NBUF = 2, 2


def _ptr(rank, idx):
    return 0x10000000 * (rank + 1) + 0x100000 * idx


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist
    import kv_cache_bench_b200 as kvb
    from kv_cache_bench_b200 import peer

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    calls = {"alloc": [], "open": [], "close": [], "free": []}

    def ipc_alloc(nbytes):
        idx = len(calls["alloc"])
        calls["alloc"].append(nbytes)
        return _ptr(rank, idx), f"rank{rank}-alloc{idx}".encode().ljust(64, b"\0")

    def ipc_open(handle):
        text = handle.rstrip(b"\0").decode()
        r, i = int(text.split("-")[0][4:]), int(text.split("alloc")[1])
        calls["open"].append((r, i))
        return _ptr(r, i)

    kvb.ipc_alloc, kvb.ipc_open = ipc_alloc, ipc_open
    kvb.ipc_close = lambda p: calls["close"].append(p)
    kvb.ipc_free = lambda p: calls["free"].append(p)
    shim = types.SimpleNamespace(zeros=torch.zeros, int32=torch.int32, as_tensor=torch.as_tensor,
                                 cuda=types.SimpleNamespace(synchronize=lambda: None))
    try:
        rows = torch.arange(3, dtype=torch.int32)
        pg = peer.PeerGather(shim, dist, rank, world, rows=10, heads=32, head_dim=128, device="cpu",
                             out_head0=4 * rank, out_rows=rows, nbuf=NBUF)
        assert calls["alloc"] == [10 * 32 * 128 * 4] * NBUF + [4 * kvb.MAX_PEERS]
        assert sorted(calls["open"]) == sorted((j, i) for j in range(world) if j != rank for i in range(NBUF + 1))
        for b in range(NBUF):
            a = pg.args[b]
            assert (a.n_peers, a.self, a.rows, a.out_heads, a.out_head0) == (world, rank, 10, 32, 4 * rank)
            assert a.out_rows == rows.data_ptr()
            assert [a.peer_out[j] for j in range(world)] == [_ptr(j, b) for j in range(world)]
            assert all(a.peer_out[j] is None for j in range(world, kvb.MAX_PEERS))
        bar = pg.barrier
        assert (bar.n_peers, bar.rank, bar.epoch) == (world, rank, pg.epoch.data_ptr())
        assert [bar.signal[j] for j in range(world)] == [_ptr(j, NBUF) for j in range(world)]
        pg.close()
        assert sorted(calls["close"]) == sorted(_ptr(j, i) for j in range(world) if j != rank for i in range(NBUF + 1))
        assert sorted(calls["free"]) == [_ptr(rank, i) for i in range(NBUF + 1)]
        pg.close()  # a second close does nothing
        assert len(calls["free"]) == NBUF + 1
        with open(os.path.join(out_dir, f"ok{rank}"), "w") as fh:
            fh.write("ok")
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_peer_gather_rendezvous_on_two_gloo_ranks(tmp_path):
    mp.start_processes(_worker, args=(WORLD, _free_port(), str(tmp_path)), nprocs=WORLD, join=True,
                       start_method="spawn")
    assert all((tmp_path / f"ok{r}").exists() for r in range(WORLD))
