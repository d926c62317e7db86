"""CPU oracle for CoRoPE attention -- TEST INFRASTRUCTURE ONLY.

This module is the reference the CUDA kernels of this repository are tested
against.  Only the
tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
import it.  The product path (the ``CoROPE`` package and the C-ABI library)
never calls into it and fails loudly when the CUDA library is missing.

It restates, in plain PyTorch on the CPU, the pure-PyTorch CoRoPE definition of
the reference (N1-research/CoRoPE-jcx ``check.py:44-103``, ``forward_reference``):

* gate          ``z[t,i] = sigmoid(q_t . k_i)`` (no ``sm_scale``), zero for
                ``i > t``                                   (check.py:48-56)
* position      ``c[t,j] = sum_{i<=j} z[t,i]``              (check.py:58)
* frequencies   ``theta_p = theta ** (-2p/D)``              (check.py:61-63)
* rotation      interleaved pairs ``(2p, 2p+1)``:
                ``even' = e cos - o sin``, ``odd' = e sin + o cos``
                                                            (check.py:65-81)
* logits        ``sm_scale * <R(c[t,t] theta) q_t, R(c[t,j] theta) k_j>``
                with a causal ``-inf`` mask                 (check.py:88-95)
* softmax, ``O = W V``                                      (check.py:98-101)

Gradients are those of PyTorch autograd through that definition, which is how
the reference checks its own backward (check.py:138-148).  ``backward_dense``
gives the same gradients in closed form (validated against autograd in the
tests) so that larger shapes fit in memory.

The forward also reports the running-max ``M``, the sum of exponentials ``L``
and the total gate sum ``A`` exactly as the reference's forward kernel stores
them (CoROPE/forward.py:96-120): ``M_t = max_j logit_tj``,
``L_t = sum_j exp(logit_tj - M_t)``, ``A_t = sum_{i<=t} z_ti``.

The MQA variant (CoROPE/co_rope_mqa_forward.py:7-104) is the same computation
with the single K/V head shared by every query head plus an optional additive
``bias[t, j]`` applied after the scaling (co_rope_mqa_forward.py:72-75).

Parity of this restatement is pinned by ``tests/golden/`` (fixtures produced by
running the reference's own ``check.forward_reference``, its autograd
gradients and its Triton kernels in interpreter mode; see
``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

__all__ = [
    "thetas_for",
    "forward_reference_loop",
    "forward_dense",
    "backward_dense",
    "forward_rows",
    "expand_kv",
]


def thetas_for(head_dim: int, theta: float, dtype=torch.float32) -> torch.Tensor:
    """``theta_p = 1 / theta ** (2p / D)`` for p = 0..D/2-1 (check.py:61-63).

    Computed in fp32 exactly as the reference does, then cast."""
    th = 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))
    return th.to(dtype)


def expand_kv(x: torch.Tensor, num_q_heads: int) -> torch.Tensor:
    """Broadcast K/V heads over their query-head group (MQA/GQA)."""
    B, Hkv, S, D = x.shape
    if Hkv == num_q_heads:
        return x
    g = num_q_heads // Hkv
    return x[:, :, None].expand(B, Hkv, g, S, D).reshape(B, num_q_heads, S, D)


def _rotate(d: torch.Tensor, ang: torch.Tensor) -> torch.Tensor:
    """Interleaved pair rotation of ``d[..., D]`` by ``ang[..., D/2]``
    (check.py:65-81; rope_utils.py:68-82 pairing)."""
    c, s = torch.cos(ang), torch.sin(ang)
    e, o = d[..., 0::2], d[..., 1::2]
    out = torch.stack((e * c - o * s, e * s + o * c), dim=-1)
    return out.reshape(*out.shape[:-2], d.shape[-1])


def forward_reference_loop(q, k, v, sm_scale, theta=10000.0, rows=None):
    """Row-by-row restatement of check.py:44-103 (same loop structure: a dense
    gate matrix, then one Python iteration per (b, h, t) that rotates q_t and
    all keys).  Returns ``(o, w)`` like the reference.  This is the form timed
    as the CPU baseline; it is slow by construction.  ``rows`` restricts the
    loop to a subset of query rows (the other rows of ``o`` and ``w`` stay 0),
    which bounds a timing sample of a long sequence."""
    B, H, S, D = q.shape
    qk = torch.matmul(q, k.transpose(-2, -1))
    mask = torch.triu(torch.ones(S, S, dtype=torch.bool), diagonal=1)
    z = torch.sigmoid(qk).masked_fill(mask, 0)
    a = torch.cumsum(z, dim=-1)
    th = thetas_for(D, theta, q.dtype)
    w = torch.zeros(B, H, S, S, dtype=q.dtype)
    ar = torch.arange(S)
    row_list = range(S) if rows is None else [int(r) for r in rows]
    for b in range(B):
        for h in range(H):
            for t in row_list:
                q_rot = _rotate(q[b, h, t], a[b, h, t, t] * th)
                k_rot = _rotate(k[b, h], torch.outer(a[b, h, t], th))
                logits = torch.where(ar <= t, (k_rot * q_rot).sum(-1) * sm_scale,
                                     torch.tensor(float("-inf"), dtype=q.dtype))
                w[b, h, t] = torch.softmax(logits, dim=0)
    return torch.matmul(w, v), w


def _gate_positions(q, k):
    """Gate matrix z (masked) and inclusive positions c = cumsum(z)."""
    S = q.shape[-2]
    s = torch.matmul(q, k.transpose(-2, -1))
    mask = torch.triu(torch.ones(S, S, dtype=torch.bool), diagonal=1)
    z = torch.sigmoid(s).masked_fill(mask, 0)
    c = torch.cumsum(z, dim=-1)
    return s, z, c, mask


def _logits_rows(q, k, c, rows, th, sm_scale):
    """Logits for query rows ``rows`` of one (b, h): absolute rotations
    ``R(c[t,t] th) q_t`` and ``R(c[t,j] th) k_j`` as check.py:90-95 does."""
    ct = c[rows]                                   # [T, S]
    ctt = ct[torch.arange(len(rows)), rows]        # [T]
    q_rot = _rotate(q[rows], ctt[:, None] * th)    # [T, D]
    k_rot = _rotate(k[None, :, :], ct[:, :, None] * th)   # [T, S, D]
    return (k_rot * q_rot[:, None, :]).sum(-1) * sm_scale


def forward_dense(q, k, v, sm_scale, theta=10000.0, bias=None, row_chunk=64):
    """Vectorised forward.  q: [B,H,S,D]; k, v: [B,Hkv,S,D] (Hkv divides H).

    Returns dict with ``o`` [B,H,S,D], ``m``, ``l``, ``a`` [B,H,S] (the
    reference's saved state, CoROPE/forward.py:110-120) and ``lse``.
    Computation dtype is the dtype of ``q`` (fp32 or fp64)."""
    B, H, S, D = q.shape
    k = expand_kv(k, H)
    v = expand_kv(v, H)
    th = thetas_for(D, theta, q.dtype)
    o = torch.empty_like(q)
    m = torch.empty(B, H, S, dtype=q.dtype)
    l = torch.empty_like(m)
    a = torch.empty_like(m)
    causal = torch.tril(torch.ones(S, S, dtype=torch.bool))
    for b in range(B):
        for h in range(H):
            _, z, c, _ = _gate_positions(q[b, h], k[b, h])
            a[b, h] = torch.diagonal(c)
            for r0 in range(0, S, row_chunk):
                rows = torch.arange(r0, min(S, r0 + row_chunk))
                lg = _logits_rows(q[b, h], k[b, h], c, rows, th, sm_scale)
                if bias is not None:
                    lg = lg + bias[rows].to(q.dtype)
                lg = lg.masked_fill(~causal[rows], float("-inf"))
                mx = lg.max(-1).values
                e = torch.exp(lg - mx[:, None])
                se = e.sum(-1)
                m[b, h, rows] = mx
                l[b, h, rows] = se
                o[b, h, rows] = (e / se[:, None]) @ v[b, h]
    return {"o": o, "m": m, "l": l, "a": a, "lse": m + torch.log(l)}


def forward_rows(q, k, v, rows, sm_scale, theta=10000.0, bias=None):
    """Forward for a subset of query rows of one (b, h) slice.

    q: [S, D], k, v: [S, D]; rows: 1-D LongTensor.  Row t only needs keys
    0..t, so sampled rows of a long sequence are cheap.  Returns o [T,D],
    m, l, a [T]."""
    S, D = q.shape
    th = thetas_for(D, theta, q.dtype)
    outs_o, outs_m, outs_l, outs_a = [], [], [], []
    for t in rows.tolist():
        kk = k[: t + 1]
        z = torch.sigmoid(kk @ q[t])
        c = torch.cumsum(z, 0)
        q_rot = _rotate(q[t], c[t] * th)
        k_rot = _rotate(kk, c[:, None] * th)
        lg = (k_rot * q_rot).sum(-1) * sm_scale
        if bias is not None:
            lg = lg + bias[t, : t + 1].to(q.dtype)
        mx = lg.max()
        e = torch.exp(lg - mx)
        se = e.sum()
        outs_o.append((e / se) @ v[: t + 1])
        outs_m.append(mx)
        outs_l.append(se)
        outs_a.append(c[t])
    return (torch.stack(outs_o), torch.stack(outs_m), torch.stack(outs_l),
            torch.stack(outs_a))


def backward_dense(q, k, v, do, sm_scale, theta=10000.0, bias=None, row_chunk=64):
    """Closed-form gradients of ``forward_dense`` (equal to autograd through
    check.py:44-103).  q, do: [B,H,S,D]; k, v: [B,Hkv,S,D].

    With ``a_tj = c_tt - c_tj`` and ``phi = a theta_p`` the logit is
    ``sm * sum_p cos(phi) C_p + sin(phi) S_p`` where ``C_p = q_e k_e + q_o k_o``
    and ``S_p = q_e k_o - q_o k_e``.  The chain rule runs through the softmax,
    the rotation (direct q/k terms), the position ``a`` (d logit / d a), the
    gate cumsum (exclusive prefix sum of ``da`` along keys) and the sigmoid.
    Returns (dq, dk, dv) with k/v gradients summed over each head group."""
    B, H, S, D = q.shape
    Hkv = k.shape[1]
    ke = expand_kv(k, H)
    ve = expand_kv(v, H)
    th = thetas_for(D, theta, q.dtype)
    dq = torch.zeros_like(q)
    dk = torch.zeros(B, H, S, D, dtype=q.dtype)
    dv = torch.zeros(B, H, S, D, dtype=q.dtype)
    causal = torch.tril(torch.ones(S, S, dtype=torch.bool))
    for b in range(B):
        for h in range(H):
            qq, kk, vv, dd = q[b, h], ke[b, h], ve[b, h], do[b, h]
            s, z, c, _ = _gate_positions(qq, kk)
            ds_full = torch.zeros(S, S, dtype=q.dtype)
            qe, qo = qq[:, 0::2], qq[:, 1::2]
            kev, kov = kk[:, 0::2], kk[:, 1::2]
            for r0 in range(0, S, row_chunk):
                rows = torch.arange(r0, min(S, r0 + row_chunk))
                T = len(rows)
                cm = causal[rows]
                ar = (c[rows, rows][:, None] - c[rows]).masked_fill(~cm, 0)
                phi = ar[:, :, None] * th                      # [T,S,P]
                cs, sn = torch.cos(phi), torch.sin(phi)
                Cp = qe[rows][:, None, :] * kev[None] + qo[rows][:, None, :] * kov[None]
                Sp = qe[rows][:, None, :] * kov[None] - qo[rows][:, None, :] * kev[None]
                lg = (cs * Cp + sn * Sp).sum(-1) * sm_scale
                if bias is not None:
                    lg = lg + bias[rows].to(q.dtype)
                lg = lg.masked_fill(~cm, float("-inf"))
                P = torch.softmax(lg, -1)
                o_rows = P @ vv
                dv[b, h] += P.transpose(0, 1) @ dd[rows]
                dP = dd[rows] @ vv.transpose(0, 1)
                delta = (dd[rows] * o_rows).sum(-1, keepdim=True)
                dl = P * (dP - delta)                         # d logit
                dlp = (th * (cs * Sp - sn * Cp)).sum(-1)      # (d logit / d a) / sm
                da = (dl * sm_scale * dlp).masked_fill(~cm, 0)
                dz = torch.cumsum(da, -1) - da                # sum_{j<i} da_tj
                zr = z[rows]
                ds = (dz * zr * (1 - zr)).masked_fill(~cm, 0)
                ds_full[rows] = ds
                w = (dl * sm_scale)[:, :, None]
                # direct rotation terms
                dqe = (w * (kev[None] * cs + kov[None] * sn)).sum(1)
                dqo = (w * (-kev[None] * sn + kov[None] * cs)).sum(1)
                dq[b, h, rows, 0::2] += dqe
                dq[b, h, rows, 1::2] += dqo
                dke = (w * (qe[rows][:, None, :] * cs - qo[rows][:, None, :] * sn)).sum(0)
                dko = (w * (qe[rows][:, None, :] * sn + qo[rows][:, None, :] * cs)).sum(0)
                dk[b, h, :, 0::2] += dke
                dk[b, h, :, 1::2] += dko
            dq[b, h] += ds_full @ kk
            dk[b, h] += ds_full.transpose(0, 1) @ qq
    if Hkv != H:
        g = H // Hkv
        dk = dk.reshape(B, Hkv, g, S, D).sum(2)
        dv = dv.reshape(B, Hkv, g, S, D).sum(2)
    return dq, dk, dv


def backward_rows(q, k, v, do, rows, sm_scale, theta=10000.0, row_chunk=16):
    """The part of ``backward_dense`` that query rows ``rows`` of one (b, h)
    slice contribute, for long sequences.  q, k, v, do: [S, D].

    Row t only involves keys 0..t, so this costs O(T S D).  Returns
    ``dq`` of those rows [T, D] (complete: a row's dq depends on that row
    alone) and their summed contributions ``dk_part``, ``dv_part`` [S, D] to
    every key.  The gradient of key j is complete once every row t >= j is
    among ``rows``: with rows = S-n..S-1 the last n keys' dk, dv are exact."""
    S, D = q.shape
    th = thetas_for(D, theta, q.dtype)
    rows = rows.to(torch.long)
    dq = torch.zeros(len(rows), D, dtype=q.dtype)
    dk = torch.zeros(S, D, dtype=q.dtype)
    dv = torch.zeros(S, D, dtype=q.dtype)
    for r0 in range(0, len(rows), row_chunk):
        rr = rows[r0:r0 + row_chunk]
        n = int(rr.max()) + 1                             # keys any of these rows sees
        kk, vv = k[:n], v[:n]
        qt, dot = q[rr], do[rr]                           # [T, D]
        cm = torch.arange(n)[None, :] <= rr[:, None]      # causal mask [T, n]
        z = torch.sigmoid(qt @ kk.T).masked_fill(~cm, 0)
        c = torch.cumsum(z, 1)
        ctt = c.gather(1, rr[:, None])                    # c[t, t]
        phi = ((ctt - c).masked_fill(~cm, 0))[:, :, None] * th   # [T, n, P]
        cs, sn = torch.cos(phi), torch.sin(phi)
        qe, qo = qt[:, None, 0::2], qt[:, None, 1::2]
        ke, ko = kk[None, :, 0::2], kk[None, :, 1::2]
        Cp = qe * ke + qo * ko
        Sp = qe * ko - qo * ke
        lg = ((cs * Cp + sn * Sp).sum(-1) * sm_scale).masked_fill(~cm, float("-inf"))
        P = torch.softmax(lg, 1)
        o = P @ vv
        dv[:n] += P.T @ dot
        dl = P * (dot @ vv.T - (dot * o).sum(-1, keepdim=True))
        da = (dl * sm_scale * (th * (cs * Sp - sn * Cp)).sum(-1)).masked_fill(~cm, 0)
        dz = torch.cumsum(da, 1) - da                     # sum_{j<i} da_tj
        ds = (dz * z * (1 - z)).masked_fill(~cm, 0)
        w = (dl * sm_scale)[:, :, None]
        dq[r0:r0 + len(rr), 0::2] = (w * (ke * cs + ko * sn)).sum(1)
        dq[r0:r0 + len(rr), 1::2] = (w * (-ke * sn + ko * cs)).sum(1)
        dq[r0:r0 + len(rr)] += ds @ kk
        dk[:n, 0::2] += (w * (qe * cs - qo * sn)).sum(0)
        dk[:n, 1::2] += (w * (qe * sn + qo * cs)).sum(0)
        dk[:n] += ds.T @ qt
    return dq, dk, dv


def autograd_reference(q, k, v, do, sm_scale, theta=10000.0, bias=None):
    """Gradients by autograd through ``forward_dense`` (small shapes only)."""
    qq = q.detach().clone().requires_grad_(True)
    kk = k.detach().clone().requires_grad_(True)
    vv = v.detach().clone().requires_grad_(True)
    B, H, S, D = qq.shape
    ke, ve = expand_kv(kk, H), expand_kv(vv, H)
    th = thetas_for(D, theta, qq.dtype)
    outs = []
    causal = torch.tril(torch.ones(S, S, dtype=torch.bool))
    for b in range(B):
        hs = []
        for h in range(H):
            _, z, c, _ = _gate_positions(qq[b, h], ke[b, h])
            lg = _logits_rows(qq[b, h], ke[b, h], c, torch.arange(S), th, sm_scale)
            if bias is not None:
                lg = lg + bias.to(qq.dtype)
            lg = lg.masked_fill(~causal, float("-inf"))
            hs.append(torch.softmax(lg, -1) @ ve[b, h])
        outs.append(torch.stack(hs))
    o = torch.stack(outs)
    o.backward(do)
    return o.detach(), qq.grad, kk.grad, vv.grad


def flops(B, H, S, D, kind="fwd+bwd"):
    """FlashAttention flop convention over the causal pairs
    ``P = B*H*S*(S+1)/2``: fwd ``4*D*P``, bwd ``10*D*P``."""
    P = B * H * S * (S + 1) / 2
    return {"fwd": 4 * D * P, "bwd": 10 * D * P, "fwd+bwd": 14 * D * P}[kind]
