"""Multi-rank host logic of bench.py on CPU (gloo, world size 2): batch x head
sharding needs no data exchange, and the job time is the max over ranks."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        from oracle import corope_oracle as O
        # each rank owns whole batch entries of a small global batch
        per_rank, H, S, D = 2, 2, 24, 8
        mine = bench.rank_batches(rank, per_rank)
        g = torch.Generator().manual_seed(7)
        q, k, v = (torch.randn(per_rank * world, H, S, D, generator=g) for _ in range(3))
        r = O.forward_dense(q[mine], k[mine], v[mine], 0.3, 1e4)
        gathered = [torch.empty_like(r["o"]) for _ in range(world)]
        dist.all_gather(gathered, r["o"])
        t = bench.max_over_ranks(float(rank + 1), world, device="cpu")
        if rank == 0:
            full = O.forward_dense(q, k, v, 0.3, 1e4)["o"]
            out["err"] = (torch.cat(gathered) - full).abs().max().item()
            out["max"] = t
            out["owned"] = [bench.rank_batches(i, per_rank) for i in range(world)]
    finally:
        dist.destroy_process_group()


def test_bxh_sharding_and_max_timing_gloo():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
        assert all(p.exitcode == 0 for p in procs)
        assert out["err"] == 0.0
        assert out["max"] == 2.0
        owned = out["owned"]
        assert sorted(sum(owned, [])) == list(range(2 * world)) and not set(owned[0]) & set(owned[1])
