"""CoRoPE attention throughput on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload W] [--impl ...]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1)

Default (``--workload bench``): one step = CoRoPE forward + backward (dq, dk,
dv) over one batch of B=4, H=32, S=4096, D=128, bf16, causal, theta=1e4
(synthetic N(0,1) inputs, per-rank seed).  Multi-GPU runs are weak scaling:
every rank owns its own batch of 4 x 32 (b, h) units (batch x head sharding,
no collective on the data path); the barrier and the max-over-ranks timing
reduction are the only NCCL calls.  The other workloads are the remaining
configurations of the path, one line each:

* ``d64``      B=8, H=16, S=2048, D=64, theta 1e4, forward + backward
* ``mqa``      B=4, Hq=32, Hkv=1, S=8192, D=128, theta 5e5, forward
* ``long``     B=1, H=32, S=32768, D=128, theta 5e5, forward + backward: one
               GPU's share of B=8 under batch x head sharding
* ``plain``    plain causal softmax attention forward (no contextual
               positions) at the bench shape on the same tensor-core pipeline,
               with the CoRoPE forward timed beside it
* ``long-seq`` the same sequences sharded over the ranks of a torchrun job
               (zig-zag query chunks, K/V all-gather, dk/dv reduce-scatter;
               global batch = number of ranks)

``--shape B,H,S,D`` runs a workload's kernels on another shape (a small case
for a profiler capture, with ``--no-e2e --no-cpu-baseline``).

Metric: TFLOP/s in the FlashAttention convention over the causal pairs
P = B*H*S*(S+1)/2 (fwd 4*D*P, bwd 10*D*P), whole job (all ranks).

Prints one JSON line (rank 0).  ``--impl reference`` instead times the
reference's own CPU path (the oracle's restatement of check.py's
forward_reference plus autograd) on a bounded sample of the bench workload;
``--impl reference-triton`` times the reference's Triton kernels (staged
with ``--stage-reference <checkout>``) next to this library's on the GPU.
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
# summed over its kernels).  Exact kernel: an ncu capture of B=1,H=8,S=2048,D=128
# scaled by query rows x heads (x32).  Tensor-core kernels: a capture of half the
# bench workload (B=2,H=32,S=4096,D=128: pre 0.14 GB, panels 0.67 GB, dQ kernel
# 2.62 GB, dK kernel 1.50 GB, conversion 0.37 GB), twice that here.
NCU_TRAFFIC_BYTES = {("bench", "exact"): 33.78e6 * 32,
                     ("bench", "tensor"): 2 * 5.3015e9}
# The pipe that binds the dominant kernel (ncu, B=1,H=8,S=2048,D=128 of the same
# kernel): instruction issue of the CUDA-core work around the tensor-core GEMMs
ROOFLINE_BINDING = {("bench", "tensor"): {"resource": "instruction issue",
                                          "issue_active_pct": 50.4, "tensor_pipe_pct": 15.0,
                                          "kernel": "dQ kernel (52% of the step)"}}


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


def rank_seed(rank, seed=1):
    return seed + 1000 * rank


def make_inputs(rank, dev, dtype=torch.bfloat16, shape_q=None, shape_kv=None, seed=1,
                with_do=True):
    """q, k, v (and dO) of this rank: N(0,1) drawn on the device in that
    order, cast to ``dtype``; by default the bench workload's shapes."""
    if shape_q is None:
        shape_q = tuple(WORKLOAD[k] for k in "BHSD")
    shape_kv = shape_q if shape_kv is None else shape_kv
    g = torch.Generator(device=dev).manual_seed(rank_seed(rank, seed))
    shapes = [shape_q, shape_kv, shape_kv] + ([shape_q] if with_do else [])
    return [torch.randn(*sh, device=dev, generator=g, dtype=torch.float32).to(dtype)
            for sh in shapes]


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


# ---- the reference's own Triton kernels on the same GPU -------------------
REF_DIR = os.path.join(ROOT, "baseline", "_ref", "CoROPE")
REF_FILES = ("forward.py", "co_rope_mqa_forward.py", "co_rope_backward.py")


def stage_reference(src):
    """Copy the reference's Triton kernel modules, unmodified, from its
    checkout ``src`` (the directory holding ``CoROPE/``) into
    baseline/_ref/CoROPE (git-ignored; it travels with the tree to the GPU
    machine).  The reference has no setup.py or pyproject.toml, so pip cannot
    install it; these three files are its whole forward / MQA / backward
    path and import only torch and triton."""
    import shutil
    os.makedirs(REF_DIR, exist_ok=True)
    for f in REF_FILES:
        shutil.copyfile(os.path.join(src, "CoROPE", f), os.path.join(REF_DIR, f))
    print(f"staged {', '.join(REF_FILES)} into {REF_DIR}")


def _load_reference_module(name):
    import importlib.util
    path = os.path.join(REF_DIR, name + ".py")
    if not os.path.exists(path):
        return None
    spec = importlib.util.spec_from_file_location("corope_reference_" + name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _event_ms(fn, steps, warmup, stream):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        fn()
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def run_reference_triton(args):
    """Time the reference's own Triton kernels (staged by --stage-reference)
    against this library's kernels on the same GPU, same inputs, CUDA events:

    * the forward ``co_rope_forward`` (CoROPE/forward.py:123-178) at B=4, H=32,
      S=4096, D=128 bf16, theta 1e4;
    * the MQA forward ``co_rope_mqa_forward`` (CoROPE/co_rope_mqa_forward.py:
      107-176) at Hq=32, Hkv=1, S=8192, D=128 bf16, theta 5e5, one launch per
      batch entry: it offsets K/V by the query batch stride
      (co_rope_mqa_forward.py:26-27) and reads past K/V for any batch entry
      but the first, so it only runs on batch-1 slices;
    * the backward ``co_rope_backward`` (CoROPE/co_rope_backward.py:116-211),
      timed but flagged: its result is not the gradient of the forward.

    Rank 0 only; prints one JSON line ("impl": "reference-triton")."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    fwd_mod = _load_reference_module("forward")
    if fwd_mod is None:
        print(json.dumps({"impl": "reference-triton",
                          "unavailable": "reference Triton modules not staged (run bench.py "
                                         "--stage-reference <checkout>)"}), flush=True)
        return
    mqa_mod = _load_reference_module("co_rope_mqa_forward")
    bwd_mod = _load_reference_module("co_rope_backward")
    from CoROPE.co_rope_backward import co_rope_backward
    from CoROPE.co_rope_mqa_forward import co_rope_mqa_forward
    from CoROPE.forward import co_rope_forward
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    B, H, S, D, theta = (WORKLOAD[k] for k in ("B", "H", "S", "D", "theta"))
    sm = 1 / math.sqrt(D)
    q, k, v, do = make_inputs(0, dev)
    fl_fwd, fl_bwd = flops(B, H, S, D)
    steps, warm = max(1, args.steps), max(1, min(args.warmup, 1))
    clocks = ClockSampler(0)
    clocks.start()
    out = {}
    out["fwd_ms_ref"] = _event_ms(lambda: fwd_mod.co_rope_forward(q, k, v, sm, theta=theta),
                                  steps, warm, stream)
    out["fwd_ms_ours"] = _event_ms(lambda: co_rope_forward(q, k, v, sm, theta=theta),
                                   steps, warm, stream)
    saved_ref, o_ref = fwd_mod.co_rope_forward(q, k, v, sm, theta=theta)
    saved, o = co_rope_forward(q, k, v, sm, theta=theta)
    torch.cuda.synchronize()
    out["fwd_o_maxdiff"] = (o_ref.float() - o.float()).abs().max().item()
    out["bwd_ms_ref"] = _event_ms(lambda: bwd_mod.co_rope_backward(saved_ref, do, sm, theta),
                                  1, 1, stream)
    out["bwd_ms_ours"] = _event_ms(lambda: co_rope_backward(saved, do, sm, theta),
                                   steps, warm, stream)
    del saved_ref, o_ref, saved, o
    # MQA: Hq=32, Hkv=1, S=8192, D=128, theta 5e5
    Bm, Hm, Sm, tm = 4, 32, 8192, 5e5
    g = torch.Generator(device=dev).manual_seed(3)
    qm = torch.randn(Bm, Hm, Sm, D, device=dev, generator=g).bfloat16()
    km = torch.randn(Bm, 1, Sm, D, device=dev, generator=g).bfloat16()
    vm = torch.randn(Bm, 1, Sm, D, device=dev, generator=g).bfloat16()

    def ref_mqa():
        for b in range(Bm):  # batch-1 slices only (see above)
            mqa_mod.co_rope_mqa_forward(qm[b:b + 1], km[b:b + 1], vm[b:b + 1], sm, theta=tm)

    out["mqa_fwd_ms_ref"] = _event_ms(ref_mqa, steps, warm, stream)
    out["mqa_fwd_ms_ours"] = _event_ms(lambda: co_rope_mqa_forward(qm, km, vm, sm, theta=tm),
                                       steps, warm, stream)
    clk = clocks.stop()
    mqa_flops = 4 * D * causal_pairs(Bm, Hm, Sm)
    line = {
        "impl": "reference-triton", "metric": "CoRoPE attn fwd TFLOP/s (bf16,S=4096,D=128)",
        "value": fl_fwd / (out["fwd_ms_ref"] * 1e-3) / 1e12, "unit": UNIT, "n_gpus": 1,
        "steps": steps, "warmup": warm, "ms_per_step": out["fwd_ms_ref"],
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "reference Triton kernels (CoROPE/forward.py, "
                               "co_rope_mqa_forward.py, co_rope_backward.py) vs this library, "
                               "same inputs, same GPU",
                   "fwd": "B=4 H=32 S=4096 D=128 theta=1e4",
                   "mqa": "B=4 (4 batch-1 launches) Hq=32 Hkv=1 S=8192 D=128 theta=5e5",
                   "flop_convention": "FA causal: fwd 4*D*P, bwd 10*D*P",
                   "triton": __import__("triton").__version__},
        "fwd_tflops_ref": fl_fwd / (out["fwd_ms_ref"] * 1e-3) / 1e12,
        "fwd_tflops_ours": fl_fwd / (out["fwd_ms_ours"] * 1e-3) / 1e12,
        "fwd_speedup": out["fwd_ms_ref"] / out["fwd_ms_ours"],
        "mqa_tflops_ref": mqa_flops / (out["mqa_fwd_ms_ref"] * 1e-3) / 1e12,
        "mqa_tflops_ours": mqa_flops / (out["mqa_fwd_ms_ours"] * 1e-3) / 1e12,
        "mqa_speedup": out["mqa_fwd_ms_ref"] / out["mqa_fwd_ms_ours"],
        "bwd_speedup": out["bwd_ms_ref"] / out["bwd_ms_ours"],
        "bwd_note": "the reference backward's output is not the gradient of its forward "
                    "(relative L2 error of dq ~625 against autograd of check.py); timed only",
        **out, "clocks": clk,
    }
    print(json.dumps(line), flush=True)


# Workloads.  "bench" is the headline line (the metric and configuration the
# reference benchmark is quoted on); the others are the remaining
# configurations of the same path, each on one GPU's share (weak scaling under
# torchrun: every rank runs its own copy with its own seed).
WORKLOADS = {
    "bench": dict(B=4, H=32, Hkv=32, S=4096, D=128, theta=1e4, seed=1, bwd=True,
                  name="CoRoPE MHA fwd+bwd causal, per GPU B=4 H=32 S=4096 D=128 theta=1e4"),
    "d64": dict(B=8, H=16, Hkv=16, S=2048, D=64, theta=1e4, seed=2, bwd=True,
                name="CoRoPE MHA fwd+bwd causal, per GPU B=8 H=16 S=2048 D=64 theta=1e4"),
    "mqa": dict(B=4, H=32, Hkv=1, S=8192, D=128, theta=5e5, seed=3, bwd=False,
                name="CoRoPE MQA fwd causal, per GPU B=4 Hq=32 Hkv=1 S=8192 D=128 theta=5e5"),
    "long": dict(B=1, H=32, Hkv=32, S=32768, D=128, theta=5e5, seed=4, bwd=True,
                 name="CoRoPE MHA fwd+bwd causal, per GPU B=1 H=32 S=32768 D=128 theta=5e5 "
                      "(one GPU's share of B=8: batch x head sharding)"),
    "plain": dict(B=4, H=32, Hkv=32, S=4096, D=128, theta=1e4, seed=1, bwd=False, plain=True,
                  name="plain causal softmax attention fwd (no contextual positions), per GPU "
                       "B=4 H=32 S=4096 D=128: the baseline kernel on the same pipeline"),
    "long-seq": dict(B=1, H=32, Hkv=32, S=32768, D=128, theta=5e5, seed=4, bwd=True,
                     name="CoRoPE MHA fwd+bwd causal, B=world H=32 S=32768 D=128 theta=5e5, "
                          "every sequence sharded over all ranks (zig-zag query chunks)"),
}


def workload_metric(name, w):
    if name == "bench":
        return METRIC
    if w.get("plain"):
        return (f"plain causal attention fwd TFLOP/s (bf16,B={w['B']},H={w['H']},S={w['S']},"
                f"D={w['D']}) per GPU x N")
    what = "fwd+bwd" if w["bwd"] else "fwd"
    return (f"CoRoPE attn {what} TFLOP/s (bf16,B={w['B']},H={w['H']},Hkv={w['Hkv']},"
            f"S={w['S']},D={w['D']}) per GPU x N")


def run_ours(args):
    world, rank, local = dist_setup()
    import CoROPE  # noqa: F401
    from CoROPE.co_rope_backward import co_rope_backward
    from CoROPE.co_rope_mqa_forward import co_rope_mqa_forward
    from CoROPE.forward import co_rope_forward
    from CoROPE.flash import flash_attention

    w = dict(WORKLOADS[args.workload])
    plain = bool(w.get("plain"))
    if args.shape:
        w["B"], w["H"], w["S"], w["D"] = (int(x) for x in args.shape.split(","))
        w["Hkv"] = 1 if args.workload == "mqa" else w["H"]
        w["name"] = f"{args.workload} at B={w['B']} H={w['H']} S={w['S']} D={w['D']}"
    seq_sharded = args.workload == "long-seq"
    if seq_sharded and world == 1:
        raise SystemExit("--workload long-seq shards each sequence over the ranks of a "
                         "torchrun job (N > 1)")
    dev = torch.device("cuda", local)
    B, H, Hkv, S, D, theta = (w[k] for k in ("B", "H", "Hkv", "S", "D", "theta"))
    mqa = Hkv != H
    sm = 1 / math.sqrt(D)
    stream = torch.cuda.current_stream(dev)
    algo = args.algo
    if seq_sharded:
        # global batch of `world` sequences; this rank holds its zig-zag
        # chunks (2 of 2 * world) of every sequence
        from CoROPE import context_parallel as cp
        B = world
        L = S // world
        shp_q, shp_kv = (B, H, L, D), (B, Hkv, L, D)
    else:
        shp_q, shp_kv = (B, H, S, D), (B, Hkv, S, D)
    ins = make_inputs(rank, dev, shape_q=shp_q, shape_kv=shp_kv, seed=w["seed"],
                      with_do=w["bwd"])
    q, k, v = ins[:3]
    do = ins[3] if w["bwd"] else None
    del ins

    def forward(q_, k_, v_):
        if plain:
            return None, flash_attention(q_, k_, v_, causal=True, sm_scale=sm)
        if seq_sharded:
            return cp.co_rope_forward_cp(q_, k_, v_, sm, theta=theta, algo=algo)
        if mqa:
            return co_rope_mqa_forward(q_, k_, v_, sm, theta=theta, algo=algo)
        return co_rope_forward(q_, k_, v_, sm, theta=theta, algo=algo)

    def backward(saved, do_):
        if seq_sharded:
            return cp.co_rope_backward_cp(saved, do_, sm, theta=theta, algo=algo)
        return co_rope_backward(saved, do_, sm, theta, algo=algo)

    def step():
        saved, o = forward(q, k, v)
        return backward(saved, do) if w["bwd"] else o

    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    f_ev = [(ev(), ev()) for _ in range(args.steps)]
    b_ev = [(ev(), ev()) for _ in range(args.steps)]
    start, end = ev(), ev()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    # warm-up right before the timed steps: after the sampler's start-up pause
    # the GPU is idle, and a short timed region (the plain-attention workload
    # runs 20 steps of ~1 ms) would otherwise include its clock ramp
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start.record(stream)
    for i in range(args.steps):
        f_ev[i][0].record(stream)
        saved, o = forward(q, k, v)
        f_ev[i][1].record(stream)
        if w["bwd"]:
            b_ev[i][0].record(stream)
            backward(saved, do)
            b_ev[i][1].record(stream)
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    del saved, o
    ms_total = max_over_ranks(start.elapsed_time(end), world)
    ms_step = ms_total / args.steps
    fwd_ms = statistics.mean(a.elapsed_time(b) for a, b in f_ev)
    bwd_ms = statistics.mean(a.elapsed_time(b) for a, b in b_ev) if w["bwd"] else None
    # causal pairs of this rank's share of the job (a sequence-sharded rank
    # holds 1/world of each of `world` sequences: one sequence's worth)
    fl_fwd, fl_bwd = flops(B if not seq_sharded else 1, H, S, D)
    fl_step = fl_fwd + (fl_bwd if w["bwd"] else 0)
    value = world * fl_step / (ms_step * 1e-3) / 1e12

    # ---- end to end through the public API with host buffers -------------
    # Every step copies its inputs (q, k, v and, with a backward, dO) from
    # pinned host memory and reads its results (o, and dq, dk, dv) back, all
    # inside the timed region.  As a training loader would, the copies run on
    # their own streams: step i+1's inputs go up (into the other of two
    # device slots) and step i's results come down while the kernels of step
    # i run; within a step the forward needs only q, k, v and o comes down
    # during the backward, so only the first step's q, k, v and the last
    # step's results are not overlapped.
    e2e = None
    if not args.no_e2e:
        ins = [q, k, v] + ([do] if w["bwd"] else [])
        host = [t.cpu().pin_memory() for t in ins]
        out_shapes = [q.shape] + ([q.shape, k.shape, v.shape] if w["bwd"] else [])
        outs = [torch.empty(sh, dtype=q.dtype).pin_memory() for sh in out_shapes]
        slots = [[torch.empty_like(t) for t in ins] for _ in range(2)]
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
                if w["bwd"]:
                    slots[i % 2][3].copy_(host[3], non_blocking=True)
                do_up[i % 2].record(s_up)

        def compute_and_download(i):
            # the forward starts once q, k, v are up (dO follows while it
            # runs); o goes down while the backward runs, the gradients after
            sl = slots[i % 2]
            stream.wait_event(qkv_up[i % 2])
            saved, o = forward(sl[0], sl[1], sl[2])
            fwd_done.record(stream)
            with torch.cuda.stream(s_down):
                s_down.wait_event(fwd_done)
                outs[0].copy_(o, non_blocking=True)
                o.record_stream(s_down)
            if w["bwd"]:
                stream.wait_event(do_up[i % 2])
                g = backward(saved, sl[3])
            slot_free[i % 2].record(stream)
            if w["bwd"]:
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
        e2e = {"value": world * fl_step / (e_ms * 1e-3) / 1e12, "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e_ms,
               "copies": "pinned host <-> device on two copy streams, overlapping the "
                         "previous/next step's kernels; double-buffered input slots"}

    burst, sustained, hbm, peak_src = measured_peaks()
    used = "exact" if algo == "exact" and not plain else "tensor"
    # our kernels per step: forward: the scaled-key panels and the forward
    # kernel (tensor path) or the exact kernel; backward: delta/lse, then
    # either the exact main kernel or the panels and the dQ and dK
    # tensor-core kernels, then the fp32 dk/dv conversion
    launches_per_step = (2 if used == "tensor" and not plain else 1) * (2 if seq_sharded else 1)
    if w["bwd"]:
        launches_per_step += (3 if used == "exact" else 5) * (2 if seq_sharded else 1)
    if w["bwd"]:
        rk_name, rk_ms, rk_flops = f"corope_bwd ({used})", bwd_ms, fl_bwd
    elif plain:
        rk_name, rk_ms, rk_flops = "corope_flash_fwd (plain attention)", fwd_ms, fl_fwd
    else:
        rk_name, rk_ms, rk_flops = f"corope_mqa_fwd ({used})" if mqa else f"corope_fwd ({used})", \
            fwd_ms, fl_fwd
    rk_tflops = rk_flops / (rk_ms * 1e-3) / 1e12 if not seq_sharded else None
    roofline = None
    if rk_tflops is not None:
        roofline = {"bound": "tensor", "kernel": rk_name, "achieved": rk_tflops,
                    "peak": sustained, "unit": "TFLOP/s", "frac": rk_tflops / sustained,
                    "peak_source": f"{peak_src} sustained bf16",
                    "binding_pipe": ROOFLINE_BINDING.get((args.workload, used)),
                    "traffic": NCU_TRAFFIC_BYTES.get((args.workload, used))}

    extra = {}
    if plain:
        # the CoRoPE forward on the same inputs and GPU: what the contextual
        # positions cost over plain attention
        cf = lambda: co_rope_forward(q, k, v, sm, theta=theta, algo=algo)  # noqa: E731
        for _ in range(max(1, args.warmup)):
            cf()
        torch.cuda.synchronize()
        c0, c1 = ev(), ev()
        c0.record(stream)
        for _ in range(args.steps):
            cf()
        c1.record(stream)
        torch.cuda.synchronize()
        corope_ms = max_over_ranks(c0.elapsed_time(c1), world) / args.steps
        extra = {"corope_fwd_ms": corope_ms,
                 "corope_fwd_tflops": fl_fwd / (corope_ms * 1e-3) / 1e12,
                 "corope_over_plain": corope_ms / fwd_ms}

    cpu = None
    if (rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload == "bench"
            and not args.shape):
        cv, cdt, cthreads, cdesc = cpu_reference_sample()
        cpu = {"value": cv, "unit": UNIT, "cores": cthreads, "kind": "port", "sample": cdesc,
               "seconds": cdt}

    if rank == 0:
        line = {
            "metric": workload_metric(args.workload, w), "value": value, "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": w["name"], "global_batch": B * (world if not seq_sharded else 1),
                       "heads": H, "kv_heads": Hkv, "seq_len": S, "head_dim": D, "theta": theta,
                       "parallelism": (f"seq-shard{world}" if seq_sharded
                                       else f"bxh-shard{world}"),
                       "algo": used, "l2": "inputs exceed L2 (126 MB); no flush",
                       "flop_convention": "FA causal: fwd 4*D*P, bwd 10*D*P"},
            "fwd_ms": fwd_ms, "bwd_ms": bwd_ms, **extra,
            "pct_of_peak": 100 * value / world / sustained,
            # the reference benchmark's own convention (benchmark.py:172-176):
            # fwd 4*D*B*H*S^2 and bwd 6*D*B*H*S^2, not halved for causal
            "value_reference_convention": world * (4 + (6 if w["bwd"] else 0)) * D
                                          * (B if not seq_sharded else 1) * H * S * S
                                          / (ms_step * 1e-3) / 1e12,
            "roofline": roofline,
            "e2e": e2e,
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
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-triton"])
    ap.add_argument("--stage-reference", metavar="CHECKOUT",
                    help="copy the reference's Triton modules into baseline/_ref and exit")
    ap.add_argument("--algo", default="auto", choices=["auto", "exact", "tensor"])
    ap.add_argument("--workload", default="bench", choices=sorted(WORKLOADS))
    ap.add_argument("--shape", metavar="B,H,S,D",
                    help="run the workload's kernels on another shape (e.g. a small case "
                         "for a profiler capture)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true",
                    help="skip the end-to-end leg (host copies), e.g. under a profiler")
    args = ap.parse_args()
    if args.stage_reference:
        stage_reference(args.stage_reference)
    elif args.impl == "reference":
        run_reference(args)
    elif args.impl == "reference-triton":
        run_reference_triton(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
