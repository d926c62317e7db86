"""Sequence-sharded (context-parallel) CoRoPE attention over a process group.

The reference runs a whole sequence on one device (CoROPE/forward.py:123-178,
CoROPE/co_rope_backward.py:116-211).  For sequences whose work should be split
across the GPUs of a node even when there are few (batch, head) units, each
rank here holds two query chunks of every sequence and runs the chunk entry
points of the library (``corope_fwd_chunk`` / ``corope_bwd_chunk``):

* the sequence is cut into ``2 * world`` chunks of ``C`` rows (``C`` a
  multiple of 128); rank ``r`` holds chunks ``r`` and ``2 * world - 1 - r``
  ("zig-zag"), so every rank gets the same causal work;
* forward: K and V are all-gathered (NCCL over NVLink), and each chunk's rows
  run against every key before them.  A row's gate sums, positions and online
  softmax stay inside the kernel, so no per-row state crosses ranks and the
  results equal the whole-sequence call row for row;
* backward: K and V are all-gathered again, each chunk adds its key gradients
  to fp32 accumulators covering the whole sequence, and a reduce-scatter (sum)
  returns to every rank the dk, dv of its own key chunks.

Tensors are ``[B, H, 2C, D]`` per rank in zig-zag order (``shard_sequence``
cuts a full tensor the same way); m, l, a are ``[B, H, 2C]``.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib


def zigzag_chunks(rank: int, world: int) -> tuple:
    """Sequence chunks (in units of C rows) held by ``rank``, in local order."""
    return (rank, 2 * world - 1 - rank)


def shard_sequence(x: torch.Tensor, rank: int, world: int, dim: int = 2) -> torch.Tensor:
    """This rank's zig-zag shard of a full-sequence tensor (a copy)."""
    S = x.shape[dim]
    if S % (2 * world):
        raise ValueError(f"sequence length {S} is not a multiple of 2 * world ({2 * world})")
    C = S // (2 * world)
    return torch.cat([x.narrow(dim, c * C, C) for c in zigzag_chunks(rank, world)], dim=dim)


def unshard_sequence(shards, dim: int = 2) -> torch.Tensor:
    """Inverse of ``shard_sequence`` given every rank's shard, in rank order."""
    world = len(shards)
    C = shards[0].shape[dim] // 2
    pieces = [None] * (2 * world)
    for r, x in enumerate(shards):
        c0, c1 = zigzag_chunks(r, world)
        pieces[c0] = x.narrow(dim, 0, C)
        pieces[c1] = x.narrow(dim, C, C)
    return torch.cat(pieces, dim=dim)


def _all_gather_sequence(x: torch.Tensor, group, world: int) -> torch.Tensor:
    """[B, H, 2C, D] zig-zag shards of every rank -> [B, H, 2 world C, D]."""
    x = x.contiguous()
    out = torch.empty((world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x, group=group)  # ranks concatenated along dim 0
    return unshard_sequence(list(out.chunk(world, dim=0)))


def _reduce_scatter_sequence(x: torch.Tensor, group, world: int) -> torch.Tensor:
    """Sum [B, H, S, D] over ranks and return this rank's zig-zag shard."""
    src = torch.cat([shard_sequence(x, r, world) for r in range(world)], dim=0)
    out = torch.empty((x.shape[0],) + tuple(src.shape[1:]), dtype=x.dtype, device=x.device)
    dist.reduce_scatter_tensor(out, src, op=dist.ReduceOp.SUM, group=group)
    return out


class _Kernels:
    """The library's chunk entry points (the only implementation shipped)."""

    @staticmethod
    def fwd(q, k, v, o, m, l, a, sm_scale, theta, q_row0, algo):
        _lib.fwd(q, k, v, o, m, l, a, None, sm_scale, theta, algo=algo, mqa=True, q_row0=q_row0)

    @staticmethod
    def bwd(q, k, v, o, do, m, l, a, dq, sm_scale, theta, q_row0, dk_acc, dv_acc, algo):
        _lib.bwd(q, k, v, o, do, m, l, a, dq, None, None, sm_scale, theta, algo=algo,
                 q_row0=q_row0, dk_accum=dk_acc, dv_accum=dv_acc)


def _layout(q, k, world):
    B, H, L, D = q.shape
    if L % 2 or (L // 2) % 128:
        raise ValueError(f"local sequence length {L} must be two chunks of a multiple of 128 rows")
    if k.shape[2] != L or k.shape[0] != B or k.shape[3] != D or H % k.shape[1]:
        raise ValueError("k / v shards must be [B, Hkv, 2C, D] with Hkv dividing H")
    return B, H, L // 2, D


def co_rope_forward_cp(q, k, v, sm_scale=None, causal=True, theta=10000.0, group=None,
                       algo="auto", kernels=None):
    """Forward of this rank's zig-zag shard.  Returns
    ``((q, k, v, o, m, l, a), o)`` like ``co_rope_forward``, for the shard."""
    if not causal:
        raise NotImplementedError("causal=False is not implemented (the reference is causal only)")
    kern = kernels or _Kernels
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    B, H, C, D = _layout(q, k, world)
    sm_scale = _lib.default_scale(D, sm_scale)
    k_all = _all_gather_sequence(k, group, world)
    v_all = _all_gather_sequence(v, group, world)
    o = torch.empty_like(q)
    state = []
    for i, c in enumerate(zigzag_chunks(rank, world)):
        rows = slice(i * C, (i + 1) * C)
        m, l, a = (torch.empty(B, H, C, dtype=torch.float32, device=q.device) for _ in range(3))
        kern.fwd(q[:, :, rows], k_all, v_all, o[:, :, rows], m, l, a, sm_scale, theta, c * C,
                 algo)
        state.append((m, l, a))
    m, l, a = (torch.cat([s[j] for s in state], dim=2) for j in range(3))
    return (q, k, v, o, m, l, a), o


def co_rope_backward_cp(saved, do, sm_scale=None, theta=10000.0, group=None, algo="auto",
                        kernels=None):
    """Backward of this rank's shard: (dq, dk, dv) of the shard's rows and
    key chunks (dk, dv summed over every rank's queries)."""
    kern = kernels or _Kernels
    q, k, v, o, m, l, a = saved
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    B, H, C, D = _layout(q, k, world)
    sm_scale = _lib.default_scale(D, sm_scale)
    k_all = _all_gather_sequence(k, group, world)
    v_all = _all_gather_sequence(v, group, world)
    dk_acc = torch.zeros(k_all.shape, dtype=torch.float32, device=q.device)
    dv_acc = torch.zeros_like(dk_acc)
    dq = torch.empty_like(q)
    for i, c in enumerate(zigzag_chunks(rank, world)):
        rows = slice(i * C, (i + 1) * C)
        mi, li, ai = (x[:, :, rows].contiguous() for x in (m, l, a))
        kern.bwd(q[:, :, rows], k_all, v_all, o[:, :, rows], do[:, :, rows], mi, li, ai,
                 dq[:, :, rows], sm_scale, theta, c * C, dk_acc, dv_acc, algo)
    dk = _reduce_scatter_sequence(dk_acc, group, world).to(k.dtype)
    dv = _reduce_scatter_sequence(dv_acc, group, world).to(v.dtype)
    return dq, dk, dv


class CoRoPEContextParallelFunction(torch.autograd.Function):
    """Autograd wrapper: ``apply(q, k, v, group, sm_scale=None, theta=1e4)``
    on zig-zag shards; gradients of q, k, v are the shard's."""

    @staticmethod
    def forward(ctx, q, k, v, group=None, sm_scale=None, theta=10000.0):
        saved, o = co_rope_forward_cp(q, k, v, sm_scale, True, theta, group)
        ctx.save_for_backward(*saved)
        ctx.group, ctx.sm_scale, ctx.theta = group, sm_scale, theta
        return o

    @staticmethod
    def backward(ctx, do):
        dq, dk, dv = co_rope_backward_cp(tuple(ctx.saved_tensors), do.contiguous(), ctx.sm_scale,
                                         ctx.theta, ctx.group)
        return dq, dk, dv, None, None, None
