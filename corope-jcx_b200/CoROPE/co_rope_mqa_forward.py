"""CoRoPE multi-query attention forward -- drop-in for the reference's
``CoROPE/co_rope_mqa_forward.py:co_rope_mqa_forward`` (:107-176).

K and V carry one head shared by all query heads of the batch entry.  Each
CTA runs 128 query rows of one query head; the CTAs of a head group read the
same K/V tiles and the same scaled-key operands (written once per call into
the workspace), which stay resident in L2 across the group.  The reference
adds a fresh random bias ``tril(randn(S, S) * 0.02)``
to the logits on every call (co_rope_mqa_forward.py:146, :72-75).  Here the
bias is an explicit keyword:

* ``contextual_bias=None`` (default): no bias -- plain CoRoPE MQA, equal to
  the MHA definition with K/V broadcast over heads;
* a [S, S] fp32 tensor: added to the scaled logits as the reference does;
* ``"reference"``: draw ``torch.tril(torch.randn(S, S, device=q.device) * 0.02)``
  from torch's global RNG exactly like the reference, so the same RNG state
  gives the same result.

The reference kernel offsets K/V by the query batch stride
(co_rope_mqa_forward.py:26-27,161) and is only correct for batch 1; this one
uses K/V's own strides for every batch entry.
"""
from __future__ import annotations

import torch

from . import _lib
from .forward import _check_causal

__all__ = ["co_rope_mqa_forward"]


def co_rope_mqa_forward(q, k, v, sm_scale=None, causal=True, theta=10000.0, *,
                        contextual_bias=None, algo="auto", return_bias=False):
    _check_causal(causal)
    batch_size, num_heads, seq_len, head_dim = q.shape
    if k.shape[1] != 1 or v.shape[1] != 1:
        raise ValueError("In MQA, K and V should have shape [batch_size, 1, seq_len, head_dim]")
    assert k.shape == (batch_size, 1, seq_len, head_dim) and v.shape == k.shape
    assert q.is_cuda and k.is_cuda and v.is_cuda, "Inputs must be CUDA tensors"
    assert q.dtype == k.dtype == v.dtype, "q, k, v must share a dtype"
    sm_scale = _lib.default_scale(head_dim, sm_scale)
    bias = contextual_bias
    if isinstance(bias, str):
        if bias != "reference":
            raise ValueError("contextual_bias must be None, a tensor or 'reference'")
        bias = torch.tril(torch.randn(seq_len, seq_len, device=q.device) * 0.02)
    if bias is not None:
        assert bias.shape == (seq_len, seq_len), "contextual_bias must be [S, S]"
        bias = bias.to(device=q.device, dtype=torch.float32)
        if bias.stride(-1) != 1:
            bias = bias.contiguous()
    q, k, v = _lib._rowmajor(q), _lib._rowmajor(k), _lib._rowmajor(v)
    o = torch.empty_like(q)
    if o.stride(-1) != 1:
        o = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    shape = (batch_size, num_heads, seq_len)
    m = torch.empty(shape, device=q.device, dtype=torch.float32)
    l = torch.empty(shape, device=q.device, dtype=torch.float32)
    a = torch.empty(shape, device=q.device, dtype=torch.float32)
    _lib.fwd(q, k, v, o, m, l, a, None, sm_scale, theta, bias=bias, algo=algo, mqa=True)
    if return_bias:
        return (q, k, v, o, m, l, a), o, bias
    return (q, k, v, o, m, l, a), o
