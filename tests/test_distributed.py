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


class _OracleChunks:
    """Test stand-in for the library's chunk calls on CPU: the oracle's
    per-row forward and backward for rows q_row0.. of each (b, h)."""

    @staticmethod
    def _full(x, rows, S):
        f = torch.zeros(S, x.shape[-1], dtype=torch.float64)
        f[rows] = x.double()
        return f

    @staticmethod
    def fwd(q, k, v, o, m, l, a, sm, theta, q_row0, algo):
        from oracle import corope_oracle as O
        B, H, n, _ = q.shape
        g, S = H // k.shape[1], k.shape[2]
        rows = torch.arange(q_row0, q_row0 + n)
        for b in range(B):
            for h in range(H):
                ro, rm, rl, ra = O.forward_rows(_OracleChunks._full(q[b, h], rows, S),
                                                k[b, h // g].double(), v[b, h // g].double(),
                                                rows, sm, theta)
                o[b, h], m[b, h], l[b, h], a[b, h] = ro.to(o.dtype), rm, rl, ra

    @staticmethod
    def bwd(q, k, v, o, do, m, l, a, dq, sm, theta, q_row0, dk_acc, dv_acc, algo,
            accum_chunk_rows):
        from oracle import corope_oracle as O
        from CoROPE.context_parallel import accum_slot
        B, H, n, _ = q.shape
        g, S = H // k.shape[1], k.shape[2]
        C = accum_chunk_rows
        world = S // (2 * C)
        rows = torch.arange(q_row0, q_row0 + n)
        for b in range(B):
            for h in range(H):
                rq, rk, rv = O.backward_rows(_OracleChunks._full(q[b, h], rows, S),
                                             k[b, h // g].double(), v[b, h // g].double(),
                                             _OracleChunks._full(do[b, h], rows, S), rows, sm,
                                             theta)
                dq[b, h] = rq.to(dq.dtype)
                # the owner-major layout [2, world, B, Hkv, C, D]
                for c in range(2 * world):
                    half, r = accum_slot(c, world)
                    dk_acc[half, r, b, h // g] += rk[c * C:(c + 1) * C].float()
                    dv_acc[half, r, b, h // g] += rv[c * C:(c + 1) * C].float()


def _cp_worker(rank, world, port, out):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "corope-jcx_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import corope_oracle as O
        from CoROPE import context_parallel as cp
        B, H, Hkv, S, D, sm, theta = 1, 4, 2, 2 * world * 128, 8, 0.3, 500.0
        g = torch.Generator().manual_seed(11)
        q = torch.randn(B, H, S, D, generator=g, dtype=torch.float64)
        k = torch.randn(B, Hkv, S, D, generator=g, dtype=torch.float64)
        v = torch.randn(B, Hkv, S, D, generator=g, dtype=torch.float64)
        do = torch.randn(B, H, S, D, generator=g, dtype=torch.float64)
        mine = [cp.shard_sequence(x, rank, world) for x in (q, k, v, do)]
        # a budget of one kv head: two kv-head groups in each pass
        one = B * S * D * (2 * 8 + 2 * 4)
        saved, o = cp.co_rope_forward_cp(*mine[:3], sm, theta=theta, kernels=_OracleChunks,
                                         budget=one)
        dq, dk, dv = cp.co_rope_backward_cp(saved, mine[3], sm, theta=theta,
                                            kernels=_OracleChunks, budget=one)
        out["groups"] = len(cp._head_groups(Hkv, B * S * D * (2 * 8 + 2 * 4), one))
        parts = {}
        for name, x in (("o", o), ("a", saved[6]), ("dq", dq), ("dk", dk), ("dv", dv)):
            got = [torch.empty_like(x) for _ in range(world)]
            dist.all_gather(got, x.contiguous())
            parts[name] = cp.unshard_sequence(got)
        if rank == 0:
            ref = O.forward_dense(q, k, v, sm, theta)
            rq, rk, rv = O.backward_dense(q, k, v, do, sm, theta)
            out["o"] = (parts["o"] - ref["o"]).abs().max().item()
            # m, l, a are fp32 by contract (the kernels' saved state)
            out["a"] = ((parts["a"] - ref["a"]).abs().max() / ref["a"].abs().max()).item()
            out["dq"] = (parts["dq"] - rq).abs().max().item()
            out["dk"] = ((parts["dk"] - rk).abs().max() / rk.abs().max()).item()
            out["dv"] = ((parts["dv"] - rv).abs().max() / rv.abs().max()).item()
            x = torch.arange(S).view(1, 1, S, 1).float()
            out["roundtrip"] = torch.equal(
                cp.unshard_sequence([cp.shard_sequence(x, r, world) for r in range(world)]), x)
    finally:
        dist.destroy_process_group()


def test_sequence_sharded_forward_backward_gloo():
    """Zig-zag sequence sharding over 2 ranks (gloo): K/V all-gather, per-rank
    query chunks, owner-major dk/dv accumulators and their reduce-scatter, in
    two kv-head groups -- with the oracle standing in for the chunk kernels --
    reproduces the whole-sequence forward and gradients."""
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        procs = [ctx.Process(target=_cp_worker, args=(r, world, port, out)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
        assert all(p.exitcode == 0 for p in procs)
        assert out["roundtrip"] and out["groups"] == 2
        assert out["o"] < 1e-12 and out["a"] < 1e-6 and out["dq"] < 1e-12
        assert out["dk"] < 1e-6 and out["dv"] < 1e-6


def test_sequence_sharded_backward_refuses_deterministic_mode():
    """co_rope_backward_cp sums key gradients with fp32 atomics: under
    torch.use_deterministic_algorithms(True) it raises before any collective,
    and with warn_only=True it warns and goes on."""
    from CoROPE import context_parallel as cp
    was, only = (torch.are_deterministic_algorithms_enabled(),
                 torch.is_deterministic_algorithms_warn_only_enabled())
    try:
        torch.use_deterministic_algorithms(True)
        with pytest.raises(RuntimeError, match="deterministic"):
            cp.co_rope_backward_cp((None,) * 7, None)
        torch.use_deterministic_algorithms(True, warn_only=True)
        with pytest.warns(UserWarning, match="deterministic"):
            with pytest.raises(Exception):  # no process group: fails after the warning
                cp.co_rope_backward_cp((None,) * 7, None)
    finally:
        torch.use_deterministic_algorithms(was, warn_only=only)
