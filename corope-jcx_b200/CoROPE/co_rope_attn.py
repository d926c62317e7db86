"""Autograd function and attention module -- drop-in for the reference's
``CoROPE/co_rope_attn.py`` (CoRoPEAttentionFunction :5-48, CoRoPEAttention
:52-84).  Same signatures, saved tensors and gradient tuple; the projection
outputs are passed to the kernels as strided [B, H, S, D] views (no
transpose copies)."""
from __future__ import annotations

import torch
import torch.nn as nn

from .co_rope_backward import co_rope_backward
from .forward import co_rope_forward

__all__ = ["CoRoPEAttentionFunction", "CoRoPEAttention"]


class CoRoPEAttentionFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal=True, sm_scale=None, theta=10000.0):
        batch_size, num_heads, seq_len, head_dim = q.shape
        a_k_out = torch.empty((batch_size, num_heads, seq_len), device=q.device,
                              dtype=torch.float32)
        (q_out, k_out, v_out, o_out, m_out, l_out, a_k_out), output = co_rope_forward(
            q, k, v, causal=causal, sm_scale=sm_scale, theta=theta, a_k_out=a_k_out)
        ctx.save_for_backward(q_out, k_out, v_out, o_out, m_out, l_out, a_k_out)
        ctx.causal = causal
        ctx.sm_scale = sm_scale
        ctx.theta = theta
        return output

    @staticmethod
    def backward(ctx, grad_output):
        # the (saved, do, sm_scale, theta) convention: the library builds its
        # own frequency table from theta (the reference's [H, D] table at
        # co_rope_attn.py:38-42 only feeds its 11-argument backward)
        dq, dk, dv = co_rope_backward(tuple(ctx.saved_tensors), grad_output, ctx.sm_scale,
                                      ctx.theta, causal=ctx.causal)
        return dq, dk, dv, None, None, None


class CoRoPEAttention(nn.Module):
    def __init__(self, embed_dim, num_heads, theta=10000.0, causal=True):
        super().__init__()
        self.embed_dim = embed_dim
        self.num_heads = num_heads
        self.head_dim = embed_dim // num_heads
        assert self.head_dim * num_heads == embed_dim, "embed_dim must be divisible by num_heads"
        self.q_proj = nn.Linear(embed_dim, embed_dim)
        self.k_proj = nn.Linear(embed_dim, embed_dim)
        self.v_proj = nn.Linear(embed_dim, embed_dim)
        self.out_proj = nn.Linear(embed_dim, embed_dim)
        self.theta = theta
        self.causal = causal

    def forward(self, x):
        B, S, E = x.shape
        H, D = self.num_heads, self.head_dim
        q = self.q_proj(x).view(B, S, H, D).transpose(1, 2)
        k = self.k_proj(x).view(B, S, H, D).transpose(1, 2)
        v = self.v_proj(x).view(B, S, H, D).transpose(1, 2)
        sm_scale = 1.0 / (D ** 0.5)
        attn_out = CoRoPEAttentionFunction.apply(q, k, v, self.causal, sm_scale, self.theta)
        attn_out = attn_out.transpose(1, 2).contiguous().view(B, S, E)
        return self.out_proj(attn_out)
