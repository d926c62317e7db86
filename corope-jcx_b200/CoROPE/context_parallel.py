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
  to fp32 accumulators covering the whole sequence, laid out owner-major (the
  chunks each rank owns side by side), and two reduce-scatters (sum) return to
  every rank the dk, dv of its own key chunks without a reordering copy;
* both passes run in kv-head groups sized so that the gathered K / V and the
  accumulators of a group stay under ``GROUP_BUDGET`` bytes.

Tensors are ``[B, H, 2C, D]`` per rank in zig-zag order (``shard_sequence``
cuts a full tensor the same way); m, l, a are ``[B, H, 2C]``.
"""
from __future__ import annotations

import warnings

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
    """[B, H, 2C, D] zig-zag shards of every rank -> [B, H, 2 world C, D].

    The gathered shards are put in sequence order by one copy per sequence
    chunk, each moving the chunk's contiguous [C, D] block of every (b, h)
    (about twice as fast as concatenating the narrowed shards)."""
    x = x.contiguous()
    B, H, L, D = x.shape
    C = L // 2
    out = torch.empty((world * B, H, L, D), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x, group=group)  # ranks concatenated along dim 0
    src = out.view(world, B * H, 2, C * D)
    seq = torch.empty((B, H, world * L, D), dtype=x.dtype, device=x.device)
    dst = seq.view(B * H, 2 * world, C * D)
    for r in range(world):
        for i, c in enumerate(zigzag_chunks(r, world)):
            dst[:, c].copy_(src[r, :, i])
    return seq


# Most bytes one kv-head group of the backward may hold at once: its
# all-gathered K and V plus the fp32 key-gradient accumulators over the whole
# sequence (the forward holds only K and V).  Larger problems run in kv-head
# groups, each gathered, computed and reduced before the next.
GROUP_BUDGET = 4 << 30


def _head_groups(hkv: int, per_head_bytes: int, budget: int):
    """kv-head ranges [h0, h1) whose buffers fit `budget` bytes (at least one
    head per group).  Every rank derives the same ranges from the same
    shapes, so all take the same collectives in the same order."""
    n = max(1, min(hkv, budget // max(1, per_head_bytes)))
    return [(h0, min(hkv, h0 + n)) for h0 in range(0, hkv, n)]


def accum_slot(c: int, world: int) -> tuple:
    """(half, rank) of sequence chunk c in the owner-major accumulator layout
    [2, world, B, Hkv, C, D]: chunk r at [0][r], chunk 2 world - 1 - r at
    [1][r] -- the two chunks rank r owns (corope_chunk_t.accum_chunk_rows)."""
    return (0, c) if c < world else (1, 2 * world - 1 - c)


class _Kernels:
    """The library's chunk entry points (the only implementation shipped)."""

    @staticmethod
    def fwd(q, k, v, o, m, l, a, sm_scale, theta, q_row0, algo):
        _lib.fwd(q, k, v, o, m, l, a, None, sm_scale, theta, algo=algo, mqa=True, q_row0=q_row0)

    @staticmethod
    def bwd(q, k, v, o, do, m, l, a, dq, sm_scale, theta, q_row0, dk_acc, dv_acc, algo,
            accum_chunk_rows):
        _lib.bwd(q, k, v, o, do, m, l, a, dq, None, None, sm_scale, theta, algo=algo,
                 q_row0=q_row0, dk_accum=dk_acc, dv_accum=dv_acc,
                 accum_chunk_rows=accum_chunk_rows)


def _layout(q, k, world):
    B, H, L, D = q.shape
    if L % 2 or (L // 2) % 128:
        raise ValueError(f"local sequence length {L} must be two chunks of a multiple of 128 rows")
    if k.shape[2] != L or k.shape[0] != B or k.shape[3] != D or H % k.shape[1]:
        raise ValueError("k / v shards must be [B, Hkv, 2C, D] with Hkv dividing H")
    return B, H, L // 2, D


def co_rope_forward_cp(q, k, v, sm_scale=None, causal=True, theta=10000.0, group=None,
                       algo="auto", kernels=None, budget=None):
    """Forward of this rank's zig-zag shard.  Returns
    ``((q, k, v, o, m, l, a), o)`` like ``co_rope_forward``, for the shard."""
    if not causal:
        raise NotImplementedError("causal=False is not implemented (the reference is causal only)")
    kern = kernels or _Kernels
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    B, H, C, D = _layout(q, k, world)
    hkv = k.shape[1]
    g = H // hkv
    sm_scale = _lib.default_scale(D, sm_scale)
    o = torch.empty_like(q)
    m, l, a = (torch.empty(B, H, 2 * C, dtype=torch.float32, device=q.device) for _ in range(3))
    per_head = 2 * B * (2 * world * C) * D * k.element_size()
    for h0, h1 in _head_groups(hkv, per_head, budget or GROUP_BUDGET):
        hs = slice(h0 * g, h1 * g)
        k_all = _all_gather_sequence(k[:, h0:h1], group, world)
        v_all = _all_gather_sequence(v[:, h0:h1], group, world)
        for i, c in enumerate(zigzag_chunks(rank, world)):
            rows = slice(i * C, (i + 1) * C)
            mi, li, ai = (torch.empty(B, (h1 - h0) * g, C, dtype=torch.float32, device=q.device)
                          for _ in range(3))
            kern.fwd(q[:, hs, rows], k_all, v_all, o[:, hs, rows], mi, li, ai, sm_scale, theta,
                     c * C, algo)
            m[:, hs, rows], l[:, hs, rows], a[:, hs, rows] = mi, li, ai
        del k_all, v_all
    return (q, k, v, o, m, l, a), o


def co_rope_backward_cp(saved, do, sm_scale=None, theta=10000.0, group=None, algo="auto",
                        kernels=None, budget=None):
    """Backward of this rank's shard: (dq, dk, dv) of the shard's rows and
    key chunks (dk, dv summed over every rank's queries).  Per kv-head group:
    K and V all-gathered, every local query chunk adds its key gradients to
    fp32 accumulators over the whole sequence in the owner-major layout, and
    one reduce-scatter per half of that layout hands each rank the sums of its
    own two chunks -- no reordering copy of the accumulators.

    The chunk kernels add key gradients with fp32 atomics, so there is no
    deterministic variant: with ``torch.use_deterministic_algorithms(True)``
    this raises (or warns, with ``warn_only=True``), as torch's own
    nondeterministic operations do."""
    if torch.are_deterministic_algorithms_enabled():
        msg = ("co_rope_backward_cp has no deterministic implementation (its key gradients are "
               "summed with fp32 atomics); use co_rope_backward(deterministic=True) on whole "
               "sequences")
        if torch.is_deterministic_algorithms_warn_only_enabled():
            warnings.warn(msg)
        else:
            raise RuntimeError(msg)
    kern = kernels or _Kernels
    q, k, v, o, m, l, a = saved
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    B, H, C, D = _layout(q, k, world)
    hkv = k.shape[1]
    g = H // hkv
    sm_scale = _lib.default_scale(D, sm_scale)
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    S = 2 * world * C
    per_head = B * S * D * (2 * k.element_size() + 2 * 4)
    for h0, h1 in _head_groups(hkv, per_head, budget or GROUP_BUDGET):
        hs, n = slice(h0 * g, h1 * g), h1 - h0
        k_all = _all_gather_sequence(k[:, h0:h1], group, world)
        v_all = _all_gather_sequence(v[:, h0:h1], group, world)
        dk_acc = torch.zeros(2, world, B, n, C, D, dtype=torch.float32, device=q.device)
        dv_acc = torch.zeros_like(dk_acc)
        for i, c in enumerate(zigzag_chunks(rank, world)):
            rows = slice(i * C, (i + 1) * C)
            mi, li, ai = (x[:, hs, rows].contiguous() for x in (m, l, a))
            kern.bwd(q[:, hs, rows], k_all, v_all, o[:, hs, rows], do[:, hs, rows], mi, li, ai,
                     dq[:, hs, rows], sm_scale, theta, c * C, dk_acc, dv_acc, algo, C)
        del k_all, v_all
        for acc, out in ((dk_acc, dk), (dv_acc, dv)):
            for half in range(2):  # the rank's first and second chunk
                mine = torch.empty(B, n, C, D, dtype=torch.float32, device=q.device)
                src = acc[half].view(world * B, n, C, D)  # ranks along dim 0, no copy
                dist.reduce_scatter_tensor(mine, src, op=dist.ReduceOp.SUM, group=group)
                out[:, h0:h1, half * C:(half + 1) * C] = mine.to(out.dtype)
        del dk_acc, dv_acc
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
