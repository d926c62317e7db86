"""Plain (softmax) attention forward -- drop-in for the reference's
``CoROPE/flash.py`` (``flash_attention`` :305, ``FlashAttention`` :205-302),
run by the tensor-core kernel of libcorope_b200.so that shares the CoRoPE
kernels' pipeline (corope_flash_fwd).  It is the baseline that measures what
CoRoPE's contextual positions cost on the same hardware path.

Same call surface: ``flash_attention(q, k, v, causal=True, sm_scale=None)``
returns ``o`` like q; ``FlashAttention.apply(q, k, v, causal, sm_scale)``
saves ``(q, k, v, o, M)`` with ``M`` the row max of the scaled logits
(flash.py:239, :287-289).  Documented divergences:

* bf16 / f16 inputs and head_dim 64 or 128 (the reference accepts 16..256 and
  fp32 through Triton's ``tl.dot``); other cases raise NotImplementedError;
* keys past the sequence never enter the softmax: with ``causal=False`` and a
  length that is not a multiple of 64 the reference counts the zero-filled
  keys of its last block (flash.py:149-160 load them with ``other=0`` and
  nothing masks them);
* the backward raises NotImplementedError instead of returning zero
  gradients as the reference's placeholder does (flash.py:294-302), so that
  a training loop cannot silently learn nothing.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib

__all__ = ["flash_attention", "FlashAttention"]


def _forward(q, k, v, causal, sm_scale, return_lse=False):
    B, H, S, D = q.shape
    assert k.shape == v.shape and k.shape[0] == B and k.shape[2:] == q.shape[2:], \
        "Q, K, V must have the same shape (K/V may have fewer heads dividing Q's)"
    assert q.is_cuda and k.is_cuda and v.is_cuda, "Inputs must be CUDA tensors"
    assert q.dtype == k.dtype == v.dtype, "q, k, v must share a dtype"
    if q.dtype not in (torch.bfloat16, torch.float16) or D not in (64, 128):
        raise NotImplementedError("plain attention kernel: bf16/f16 with head_dim 64 or 128")
    sm_scale = _lib.default_scale(D, sm_scale)
    q, k, v = _lib._rowmajor(q), _lib._rowmajor(k), _lib._rowmajor(v)
    o = torch.empty_like(q)
    if o.stride(-1) != 1:
        o = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    m = torch.empty((B, H, S), device=q.device, dtype=torch.float32)
    lse = torch.empty((B, H, S), device=q.device, dtype=torch.float32) if return_lse else None
    _lib.flash_fwd(q, k, v, o, m, lse, sm_scale, causal)
    return (o, m, lse) if return_lse else (o, m)


class FlashAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal=True, sm_scale=None):
        o, m = _forward(q, k, v, causal, sm_scale)
        ctx.save_for_backward(q, k, v, o, m)
        ctx.sm_scale = sm_scale
        ctx.causal = causal
        return o

    @staticmethod
    def backward(ctx, grad_output):
        raise NotImplementedError(
            "plain attention has a forward kernel only (the reference's backward returns "
            "zero gradients as a placeholder)")


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
                    sm_scale: Optional[float] = None) -> torch.Tensor:
    """softmax(sm_scale q k^T) v over [batch, heads, seq_len, head_dim]
    tensors, causal by default; ``sm_scale`` defaults to 1/sqrt(head_dim)."""
    return FlashAttention.apply(q, k, v, causal, sm_scale)
