"""CoRoPE attention forward+backward throughput on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1)

One step = CoRoPE forward + backward (dq, dk, dv) over one batch of the
workload B=4, H=32, S=4096, D=128, bf16, causal, theta=1e4 (synthetic
N(0,1) inputs, per-rank seed).  Multi-GPU runs are weak scaling: every rank
owns its own batch of 4 x 32 (b, h) units (batch x head sharding, no
collective on the data path); the barrier and the max-over-ranks timing
reduction are the only NCCL calls.

Metric: TFLOP/s in the FlashAttention convention over the causal pairs
P = B*H*S*(S+1)/2 (fwd 4*D*P, bwd 10*D*P), whole job (all ranks).

Prints one JSON line (rank 0).  ``--impl reference`` instead times the
reference's own CPU path (the oracle's restatement of check.py's
forward_reference plus autograd) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "corope-jcx_b200"))

import torch  # noqa: E402

WORKLOAD = dict(B=4, H=32, S=4096, D=128, theta=1e4)
METRIC = "CoRoPE attn fwd+bwd TFLOP/s (bf16,S=4096,D=128) at 1/2/4/8 B200; % of peak"
UNIT = "TFLOP/s"
# reference CPU sample: the last ROWS query rows of one (b, h) slice at the
# full S=4096, D=128 (each row attends to every earlier key), fwd + autograd bwd
CPU_SAMPLE_ROWS = 48

# DRAM traffic of one backward call (dram__bytes_read.sum + dram__bytes_write.sum
# summed over its kernels) from ncu captures of B=1,H=8,S=2048,D=128, scaled to
# this workload.  Exact kernel: by query rows x heads (x32),
# profiles/exact_bwd_b1h8s2048d128.md.  Tensor-core kernels: dominated by the
# dQ -> dK hand-off and the dQ kernel's panel reads, 411.9 MB over 8 x 1088
# (b, h, query tile, window) blocks, i.e. 47.3 KB per block, times the
# 128 x 4224 blocks of this workload;
# profiles/tc_bwd_b1h8s2048d128.md.
NCU_TRAFFIC_BYTES = {"exact": 33.78e6 * 32, "tensor": 411.9e6 / (8 * 1088) * (128 * 4224)}


def causal_pairs(B, H, S):
    return B * H * S * (S + 1) / 2


def flops(B, H, S, D):
    P = causal_pairs(B, H, S)
    return 4 * D * P, 10 * D * P


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            j = json.load(f)
        return j["bf16_tflops"], j["bf16_tflops_sustained"], j["hbm_gbs"], "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "100"], stdout=self.out, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.out.flush()
        self.out.seek(0)
        rows = [r.split(",") for r in self.out.read().strip().splitlines() if r.strip()]
        os.unlink(self.out.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, val in zip(names, r[5:9]):
                    if val.strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world, device="cuda"):
    """Max of a per-rank float over all ranks (the job time is the slowest rank)."""
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def rank_batches(rank, per_rank=WORKLOAD["B"]):
    """Global batch indices owned by `rank` (batch x head sharding: each rank
    owns whole batch entries, all heads, so no data crosses ranks)."""
    return list(range(rank * per_rank, (rank + 1) * per_rank))


def rank_seed(rank):
    return 1 + 1000 * rank


def make_inputs(rank, dev, dtype=torch.bfloat16):
    B, H, S, D = (WORKLOAD[k] for k in "BHSD")
    g = torch.Generator(device=dev).manual_seed(rank_seed(rank))
    return [torch.randn(B, H, S, D, device=dev, generator=g, dtype=torch.float32).to(dtype)
            for _ in range(4)]


def cpu_reference_sample(rows=CPU_SAMPLE_ROWS, threads=None):
    """Time the reference's CPU path (loop restatement of check.py:44-103 +
    autograd) on the last ``rows`` query rows of one (b, h) slice of the
    workload.  Returns (TFLOP/s, seconds, threads, description)."""
    from oracle import corope_oracle as O
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    S, D = WORKLOAD["S"], WORKLOAD["D"]
    g = torch.Generator().manual_seed(1)
    q, k, v, do = (torch.randn(1, 1, S, D, generator=g) for _ in range(4))
    rows = torch.arange(S - rows, S)
    do_mask = torch.zeros(1, 1, S, 1)
    do_mask[..., rows, :] = 1
    for t in (q, k, v):
        t.requires_grad_(True)
    t0 = time.perf_counter()
    o, _ = O.forward_reference_loop(q, k, v, 1 / math.sqrt(D), WORKLOAD["theta"], rows=rows)
    o.backward(do * do_mask)
    dt = time.perf_counter() - t0
    pairs = float(sum(int(r) + 1 for r in rows))
    fl = 14 * D * pairs
    desc = (f"last {len(rows)} query rows of one (b,h) slice at S={S}, D={D}, fp32: "
            f"check.py forward_reference loop restated + autograd; {int(pairs)} causal pairs")
    return fl / dt / 1e12, dt, threads, desc


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    vals = []
    for _ in range(args.warmup):
        cpu_reference_sample()
    for _ in range(args.steps):
        v, dt, threads, desc = cpu_reference_sample()
        vals.append((v, dt))
    value = statistics.median(v for v, _ in vals)
    ms = statistics.median(dt for _, dt in vals) * 1e3
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "CoRoPE MHA fwd+bwd causal B=4 H=32 S=4096 D=128 theta=1e4",
                   "sample": desc, "world_size": world},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args):
    world, rank, local = dist_setup()
    import CoROPE  # noqa: F401
    from CoROPE.co_rope_backward import co_rope_backward
    from CoROPE.forward import co_rope_forward
    from CoROPE import _lib

    dev = torch.device("cuda", local)
    B, H, S, D, theta = (WORKLOAD[k] for k in ("B", "H", "S", "D", "theta"))
    sm = 1 / math.sqrt(D)
    q, k, v, do = make_inputs(rank, dev)
    stream = torch.cuda.current_stream(dev)
    algo = args.algo

    def step():
        saved, o = co_rope_forward(q, k, v, sm, theta=theta, algo=algo)
        return co_rope_backward(saved, do, sm, theta, algo=algo)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    f_ev = [(ev(), ev()) for _ in range(args.steps)]
    b_ev = [(ev(), ev()) for _ in range(args.steps)]
    start, end = ev(), ev()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    start.record(stream)
    for i in range(args.steps):
        f_ev[i][0].record(stream)
        saved, o = co_rope_forward(q, k, v, sm, theta=theta, algo=algo)
        f_ev[i][1].record(stream)
        b_ev[i][0].record(stream)
        co_rope_backward(saved, do, sm, theta, algo=algo)
        b_ev[i][1].record(stream)
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    ms_total = max_over_ranks(start.elapsed_time(end), world)
    ms_step = ms_total / args.steps
    fwd_ms = statistics.mean(a.elapsed_time(b) for a, b in f_ev)
    bwd_ms = statistics.mean(a.elapsed_time(b) for a, b in b_ev)
    fl_fwd, fl_bwd = flops(B, H, S, D)
    value = world * (fl_fwd + fl_bwd) / (ms_step * 1e-3) / 1e12

    # ---- end to end through the public API with host buffers -------------
    # Every step copies its q, k, v, dO from pinned host memory and reads o,
    # dq, dk, dv back, all inside the timed region.  As a training loader
    # would, the copies run on their own streams: step i+1's inputs go up
    # (into the other of two device slots) and step i's results come down
    # while the kernels of step i run; within a step the forward needs only
    # q, k, v and o comes down during the backward, so only the first
    # step's q, k, v and the last step's gradients are not overlapped.
    host = [t.cpu().pin_memory() for t in (q, k, v, do)]
    outs = [torch.empty(q.shape, dtype=q.dtype).pin_memory() for _ in range(4)]
    slots = [[torch.empty_like(t) for t in (q, k, v, do)] for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = sum(t.numel() * t.element_size() for t in outs)
    s_up, s_down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    qkv_up = [torch.cuda.Event() for _ in range(2)]   # q, k, v of a slot are on the device
    do_up = [torch.cuda.Event() for _ in range(2)]    # and its dO
    slot_free = [torch.cuda.Event() for _ in range(2)]
    fwd_done = torch.cuda.Event()

    def upload(i):
        with torch.cuda.stream(s_up):
            if i >= 2:
                s_up.wait_event(slot_free[i % 2])
            for dst, src in zip(slots[i % 2][:3], host[:3]):
                dst.copy_(src, non_blocking=True)
            qkv_up[i % 2].record(s_up)
            slots[i % 2][3].copy_(host[3], non_blocking=True)
            do_up[i % 2].record(s_up)

    def compute_and_download(i):
        # the forward starts once q, k, v are up (dO follows while it runs);
        # o goes down while the backward runs, the gradients after it
        sl = slots[i % 2]
        stream.wait_event(qkv_up[i % 2])
        saved, o = co_rope_forward(sl[0], sl[1], sl[2], sm, theta=theta, algo=algo)
        fwd_done.record(stream)
        with torch.cuda.stream(s_down):
            s_down.wait_event(fwd_done)
            outs[0].copy_(o, non_blocking=True)
            o.record_stream(s_down)
        stream.wait_event(do_up[i % 2])
        g = co_rope_backward(saved, sl[3], sm, theta, algo=algo)
        slot_free[i % 2].record(stream)
        s_down.wait_stream(stream)
        with torch.cuda.stream(s_down):
            for dst, src in zip(outs[1:], g):
                dst.copy_(src, non_blocking=True)
                src.record_stream(s_down)

    def e2e_run(n):
        s_up.wait_stream(stream)
        upload(0)
        for i in range(n):
            if i + 1 < n:
                upload(i + 1)
            compute_and_download(i)
        stream.wait_stream(s_down)

    e2e_run(max(1, args.warmup))
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = ev(), ev()
    e0.record(stream)
    e2e_run(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    e_ms = max_over_ranks(e0.elapsed_time(e1), world) / args.steps
    e2e_value = world * (fl_fwd + fl_bwd) / (e_ms * 1e-3) / 1e12

    burst, sustained, hbm, peak_src = measured_peaks()
    bwd_tflops = fl_bwd / (bwd_ms * 1e-3) / 1e12
    # kernel families actually used: the tensor-core kernels cover bf16/f16
    # (forward: D in {64, 128}; backward: D = 128)
    fwd_used = "exact" if algo == "exact" else "tensor"
    bwd_used = "exact" if algo == "exact" else "tensor"
    used = f"fwd {fwd_used}, bwd {bwd_used}"
    # our kernels per step: forward: the scaled-key panels and the forward
    # kernel (tensor path) or the exact kernel; backward: delta/lse, then
    # either the exact main kernel or the panels and the dQ and dK
    # tensor-core kernels, then the fp32 dk/dv conversion
    launches_per_step = (2 if fwd_used == "tensor" else 1) + (3 if bwd_used == "exact" else 5)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cv, cdt, cthreads, cdesc = cpu_reference_sample()
        cpu = {"value": cv, "unit": UNIT, "cores": cthreads, "kind": "port", "sample": cdesc,
               "seconds": cdt}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "CoRoPE MHA fwd+bwd causal, per GPU B=4 H=32 S=4096 D=128 "
                                   "theta=1e4", "global_batch": B * world, "heads": H,
                       "seq_len": S, "head_dim": D, "parallelism": f"bxh-shard{world}",
                       "algo": used, "l2": "inputs (4 x 128 MiB) exceed L2; no flush",
                       "flop_convention": "FA causal: fwd 4*D*P, bwd 10*D*P"},
            "fwd_ms": fwd_ms, "bwd_ms": bwd_ms,
            "pct_of_peak": 100 * value / world / sustained,
            # the reference benchmark's own convention (benchmark.py:172-176):
            # fwd 4*D*B*H*S^2 and bwd 6*D*B*H*S^2, not halved for causal
            "value_reference_convention": world * (4 + 6) * D * B * H * S * S
                                          / (ms_step * 1e-3) / 1e12,
            "roofline": {"bound": "tensor", "kernel": f"corope_bwd ({bwd_used})",
                         "achieved": bwd_tflops, "peak": sustained, "unit": "TFLOP/s",
                         "frac": bwd_tflops / sustained, "peak_source": f"{peak_src} sustained",
                         "traffic": NCU_TRAFFIC_BYTES.get(bwd_used)},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e_ms,
                    "copies": "pinned host <-> device on two copy streams, overlapping the "
                              "previous/next step's kernels; double-buffered input slots"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--algo", default="auto", choices=["auto", "exact", "tensor"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
