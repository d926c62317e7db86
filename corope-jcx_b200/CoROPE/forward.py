"""CoRoPE attention forward -- drop-in for the reference's
``CoROPE/forward.py:co_rope_forward`` (CoROPE/forward.py:123-178).

Same signature and return value, ``((q, k, v, o, m, l, a), o)``; the work runs
in the sm_100a kernels of libcorope_b200.so.  Additions that the reference's
own callers rely on: ``sm_scale=None`` means ``1/sqrt(D)`` and ``a_k_out``
(CoROPE/co_rope_attn.py:16-18, benchmark.py:131-133) receives ``A``.
"""
from __future__ import annotations

import torch

from . import _lib

__all__ = ["co_rope_forward"]


def _check_causal(causal):
    if not causal:
        # The reference accepts the flag but always computes the causal form
        # (CAUSAL is unused in CoROPE/forward.py:7-120); a silent causal result
        # for causal=False would be wrong, so refuse instead.
        raise NotImplementedError("CoRoPE attention is causal only (causal=False unsupported)")


def co_rope_forward(q, k, v, sm_scale=None, causal=True, theta=10000.0, a_k_out=None, *,
                    algo="auto", return_lse=False):
    """CoRoPE forward.  q, k, v: [B, H, S, D] CUDA tensors (fp32/fp16/bf16).

    Returns ``((q, k, v, o, m, l, a), o)`` where ``o`` is [B, H, S, D] in the
    input dtype and ``m``, ``l``, ``a`` are fp32 [B, H, S]: the running max of
    the logits, the sum of ``exp(logit - m)`` and the total gate sum of each
    query row (CoROPE/forward.py:110-120).  ``algo`` selects the kernel family
    ("auto", "tensor", "exact").  With ``return_lse=True`` the log-sum-exp
    ``m + log(l)`` is appended as a third element."""
    _check_causal(causal)
    batch_size, num_heads, seq_len, head_dim = q.shape
    assert k.shape == q.shape
    assert v.shape == q.shape
    assert q.is_cuda and k.is_cuda and v.is_cuda, "Inputs must be CUDA tensors"
    assert q.dtype == k.dtype == v.dtype, "q, k, v must share a dtype"
    sm_scale = _lib.default_scale(head_dim, sm_scale)
    q, k, v = _lib._rowmajor(q), _lib._rowmajor(k), _lib._rowmajor(v)
    o = torch.empty_like(q)
    if o.stride(-1) != 1:
        o = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    shape = (batch_size, num_heads, seq_len)
    m = torch.empty(shape, device=q.device, dtype=torch.float32)
    l = torch.empty(shape, device=q.device, dtype=torch.float32)
    if a_k_out is not None:
        assert a_k_out.shape == shape and a_k_out.dtype == torch.float32 and a_k_out.is_contiguous()
        a = a_k_out
    else:
        a = torch.empty(shape, device=q.device, dtype=torch.float32)
    lse = torch.empty(shape, device=q.device, dtype=torch.float32) if return_lse else None
    _lib.fwd(q, k, v, o, m, l, a, lse, sm_scale, theta, algo=algo)
    if return_lse:
        return (q, k, v, o, m, l, a), o, lse
    return (q, k, v, o, m, l, a), o
