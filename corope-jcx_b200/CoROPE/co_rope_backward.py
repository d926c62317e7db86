"""CoRoPE attention backward -- drop-in for the reference's
``CoROPE/co_rope_backward.py:co_rope_backward``.

Two calling conventions exist in the reference and both are accepted:

* ``co_rope_backward(saved, do, sm_scale=None, theta=10000.0) -> (dq, dk, dv)``
  (co_rope_backward.py:116-211, used by check.py:134);
* ``co_rope_backward(q, k, v, o, m, l, a, do, thetas, causal, sm_scale)
  -> (dq, dk, dv, dthetas)`` (co_rope_attn.py:45-47, benchmark.py:46-48) where
  ``thetas`` is the repeat-interleaved [H, D] or [D] frequency table and
  ``dthetas`` is always None (the reference never produces it).

The gradients are those of the reference definition (autograd through
check.py:44-103); the reference's own Triton backward does not compute them
(its loop skips the diagonal, uses a block-local cumsum and rotates in the
opposite direction), so parity is with the definition, not with that kernel.
K/V with fewer heads than Q (MQA/GQA, from ``co_rope_mqa_forward``) are
accepted: their gradients are summed over each head group.

``deterministic=True`` (default: ``torch.are_deterministic_algorithms_enabled()``)
sums dk and dv in 64-bit fixed point instead of with fp32 atomics, so repeated
calls give bit-identical gradients (dq is deterministic either way).
"""
from __future__ import annotations

import torch

from . import _lib
from .forward import _check_causal

__all__ = ["co_rope_backward"]


def _run(q, k, v, o, m, l, a, do, sm_scale, theta, thetas, bias, algo, deterministic=False):
    B, H, S, D = q.shape
    assert q.is_cuda and k.is_cuda and v.is_cuda, "Inputs must be CUDA tensors"
    assert k.shape[0] == B and k.shape[2:] == q.shape[2:] and v.shape == k.shape
    assert do.shape == q.shape and o.shape == q.shape
    sm_scale = _lib.default_scale(D, sm_scale)
    q, k, v, o = (_lib._rowmajor(x) for x in (q, k, v, o))
    do = _lib._rowmajor(do.to(q.dtype))
    m, l, a = (x.contiguous().float() for x in (m, l, a))
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    for t in (dq, dk, dv):
        assert t.stride(-1) == 1
    _lib.bwd(q, k, v, o, do, m, l, a, dq, dk, dv, sm_scale, theta, bias=bias, algo=algo,
             thetas=thetas, deterministic=deterministic)
    return dq, dk, dv


def _table_theta(table, D, theta, algo):
    """(theta, algo) for a caller-supplied [D/2] frequency table.

    The tensor-core kernels derive their expansion coefficients and term counts
    from the scalar ``theta`` while the rotation reads the table, so the two
    must describe the same base.  The reference's callers pass only the table
    (co_rope_attn.py:35-47 rebuilds it from ``ctx.theta``), so a table that is
    not ``theta`` 's has its base recovered from its last entry
    (theta_{D/2-1} = base ** (-(D-2) / D), where fp32 rounding moves the base
    least) and checked entry by entry.  A table of no
    base >= 1 runs the exact kernels under "auto" and raises under "tensor".
    The check reads the table back, which is not allowed while a CUDA graph
    is being captured: there "auto" runs the exact kernels and "tensor"
    trusts ``theta``."""
    if torch.cuda.is_available() and table.is_cuda and torch.cuda.is_current_stream_capturing():
        return theta, ("exact" if algo == "auto" else algo)

    def matches(base):
        ref = _lib.theta_table(D, base, table.device)
        return table.shape == ref.shape and torch.allclose(table, ref, rtol=1e-6, atol=0.0)

    if matches(theta):
        return theta, algo
    if table.numel() > 1:
        t = float(table[-1])
        if 0.0 < t < 1.0:
            base = t ** (-D / (D - 2.0))
            for cand in (float(round(base)), base):
                if cand >= 1.0 and matches(cand):
                    return cand, algo
    if algo == "tensor":
        raise ValueError("thetas is not base ** (-2p / D) for any base >= 1 (or not for the "
                         "given theta); the tensor-core kernels cannot run it, use algo='exact'")
    return theta, "exact"


def co_rope_backward(*args, sm_scale=None, theta=10000.0, thetas=None, causal=True,
                     contextual_bias=None, algo="auto", deterministic=None, **kwargs):
    if deterministic is None:
        deterministic = torch.are_deterministic_algorithms_enabled()
    if args and isinstance(args[0], (tuple, list)):
        # (saved, do, sm_scale=None, theta=10000.0)
        saved, do = args[0], args[1] if len(args) > 1 else kwargs.pop("do")
        if len(args) > 2:
            sm_scale = args[2]
        if len(args) > 3:
            theta = args[3]
        q, k, v, o, m, l, a = saved
        _check_causal(causal)
        return _run(q, k, v, o, m, l, a, do, sm_scale, theta, None, contextual_bias, algo,
                    deterministic)
    # (q, k, v, o, m, l, a, do, thetas, causal, sm_scale)
    names = ["q", "k", "v", "o", "m", "l", "a", "do", "thetas", "causal", "sm_scale"]
    vals = dict(zip(names, args))
    for n in names:
        if n not in vals and n in kwargs:
            vals[n] = kwargs.pop(n)
    if "thetas" not in vals:
        vals["thetas"] = thetas
    if "causal" not in vals:
        vals["causal"] = causal
    if "sm_scale" not in vals:
        vals["sm_scale"] = sm_scale
    _check_causal(vals["causal"])
    th = vals["thetas"]
    table = None
    if th is not None:
        th = th.reshape(-1, th.shape[-1])[0] if th.dim() > 1 else th
        # repeat-interleaved [D] -> one entry per pair
        table = th[0::2].float().contiguous() if th.numel() == vals["q"].shape[-1] else th.float().contiguous()
        if algo != "exact":
            theta, algo = _table_theta(table, vals["q"].shape[-1], theta, algo)
    dq, dk, dv = _run(vals["q"], vals["k"], vals["v"], vals["o"], vals["m"], vals["l"], vals["a"],
                      vals["do"], vals["sm_scale"], theta, table, contextual_bias, algo,
                      deterministic)
    return dq, dk, dv, None
