"""Time the CoRoPE kernels on the workload shapes beyond the bench line.

    python corope-jcx_b200/bench_configs.py [bench|d64|mqa|long|plain|all]
    python -m torch.distributed.run --nproc-per-node N corope-jcx_b200/bench_configs.py long-seq

One line per shape: forward / backward milliseconds (CUDA events, best of
a few after warm-up) and TFLOP/s in the FlashAttention convention over causal
pairs P = B*H*S(S+1)/2 (forward 4*D*P, backward 10*D*P).  Inputs are N(0,1)
bf16 drawn on the device.

* bench    B=4, H=32, S=4096, D=128, theta 1e4, forward + backward
* d64      B=8, H=16, S=2048, D=64, theta 1e4, forward + backward
* mqa      B=4, Hq=32, Hkv=1, S=8192, D=128, theta 5e5, forward
* long     one GPU's share of B=8, H=32, S=32768, D=128, theta 5e5 (B=1, H=32),
           forward + backward with the default workspace and with the minimum
* plain    torch's scaled_dot_product_attention (causal) on the bench shape,
           for the cost of the contextual positions (context, not CoRoPE)
* long-seq B=2, H=32, S=32768, D=128 over the ranks of a torchrun job:
           sequence-sharded (CoROPE.context_parallel) against b x h sharding,
           the max over ranks of each
"""
import math
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import torch  # noqa: E402

from CoROPE import _lib  # noqa: E402
from CoROPE.co_rope_backward import co_rope_backward  # noqa: E402
from CoROPE.co_rope_mqa_forward import co_rope_mqa_forward  # noqa: E402
from CoROPE.forward import co_rope_forward  # noqa: E402


def pairs(B, H, S):
    return B * H * S * (S + 1) / 2


def best_of(fn, reps=3, warmup=2):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ts = []
    for _ in range(reps):
        ev[0].record()
        fn()
        ev[1].record()
        torch.cuda.synchronize()
        ts.append(ev[0].elapsed_time(ev[1]))
    return min(ts)


def inputs(shape_q, shape_kv, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(*shape_q, device="cuda", generator=g).bfloat16()
    k, v = (torch.randn(*shape_kv, device="cuda", generator=g).bfloat16() for _ in range(2))
    do = torch.randn(*shape_q, device="cuda", generator=g).bfloat16()
    return q, k, v, do


def fwd_bwd(name, B, H, S, D, theta, seed, workspace="auto"):
    q, k, v, do = inputs((B, H, S, D), (B, H, S, D), seed)
    sm = 1 / math.sqrt(D)
    state = {}

    def f():
        state["saved"], _ = co_rope_forward(q, k, v, sm, theta=theta)

    def b():
        saved = state["saved"]
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        _lib.bwd(*saved[:4], do, *saved[4:], dq, dk, dv, sm, theta, workspace=workspace)

    tf = best_of(f)
    tb = best_of(b)
    P = pairs(B, H, S)
    print(f"{name}: B={B} H={H} S={S} D={D} theta={theta:g} workspace={workspace}: "
          f"fwd {tf:.2f} ms bwd {tb:.2f} ms -> {14 * D * P / (tf + tb) / 1e9:.1f} TFLOP/s "
          f"(fwd {4 * D * P / tf / 1e9:.1f}, bwd {10 * D * P / tb / 1e9:.1f}); "
          f"device error {_lib.take_device_error()}", flush=True)


def mqa():
    B, H, S, D, theta = 4, 32, 8192, 128, 5e5
    q, k, v, _ = inputs((B, H, S, D), (B, 1, S, D), 3)
    sm = 1 / math.sqrt(D)
    t = best_of(lambda: co_rope_mqa_forward(q, k, v, sm, theta=theta))
    print(f"mqa: B={B} Hq={H} Hkv=1 S={S} D={D} theta={theta:g}: fwd {t:.2f} ms -> "
          f"{4 * D * pairs(B, H, S) / t / 1e9:.1f} TFLOP/s; device error "
          f"{_lib.take_device_error()}", flush=True)


def plain():
    B, H, S, D = 4, 32, 4096, 128
    q, k, v, do = inputs((B, H, S, D), (B, H, S, D), 1)
    qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
    state = {}

    def f():
        state["o"] = torch.nn.functional.scaled_dot_product_attention(qq, kk, vv, is_causal=True)

    def b():
        state["o"].backward(do, retain_graph=True)

    tf = best_of(f)
    f()
    tb = best_of(b)
    P = pairs(B, H, S)
    print(f"plain causal attention (torch SDPA): B={B} H={H} S={S} D={D}: fwd {tf:.3f} ms "
          f"bwd {tb:.3f} ms -> {14 * D * P / (tf + tb) / 1e9:.0f} TFLOP/s", flush=True)


def long_seq():
    import datetime
    import torch.distributed as dist
    from CoROPE import context_parallel as cp
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    B, H, S, D, theta = 2, 32, 32768, 128, 5e5
    sm = 1 / math.sqrt(D)

    def timed(fn):
        t = torch.tensor([best_of(fn, reps=2, warmup=1)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    g = torch.Generator(device=dev).manual_seed(4 + rank)
    L = S // world
    q, k, v, do = (torch.randn(B, H, L, D, device=dev, generator=g).bfloat16() for _ in range(4))

    def seq_step():
        saved, _ = cp.co_rope_forward_cp(q, k, v, sm, theta=theta)
        cp.co_rope_backward_cp(saved, do, sm, theta=theta)

    t_seq = timed(seq_step)
    del q, k, v, do
    torch.cuda.empty_cache()
    q, k, v, do = (torch.randn(B, H // world, S, D, device=dev, generator=g).bfloat16()
                   for _ in range(4))

    def bxh_step():
        saved, _ = co_rope_forward(q, k, v, sm, theta=theta)
        co_rope_backward(saved, do, sm, theta)

    t_bxh = timed(bxh_step)
    P = pairs(B, H, S)
    if rank == 0:
        print(f"long-seq: {world} GPUs, B={B} H={H} S={S} D={D} theta={theta:g}: sequence-sharded "
              f"{t_seq:.1f} ms ({14 * D * P / t_seq / 1e9:.1f} TFLOP/s), b x h-sharded "
              f"{t_bxh:.1f} ms ({14 * D * P / t_bxh / 1e9:.1f} TFLOP/s)", flush=True)
    dist.destroy_process_group()


def main():
    which = sys.argv[1] if len(sys.argv) > 1 else "all"
    if which == "long-seq":
        long_seq()
        return
    if which in ("bench", "all"):
        fwd_bwd("bench", 4, 32, 4096, 128, 1e4, 1)
    if which in ("d64", "all"):
        fwd_bwd("d64", 8, 16, 2048, 64, 1e4, 2)
    if which in ("mqa", "all"):
        mqa()
    if which in ("long", "all"):
        fwd_bwd("long", 1, 32, 32768, 128, 5e5, 4)
        fwd_bwd("long", 1, 32, 32768, 128, 5e5, 4, workspace="min")
    if which in ("plain", "all"):
        plain()


if __name__ == "__main__":
    main()
