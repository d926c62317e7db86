"""The plain attention kernel (corope_flash_fwd, CoROPE.flash) against a
dense softmax reference in fp64 on the CPU: O = softmax(sm_scale q k^T) v,
causal or not, and the row max M of the scaled logits that the reference's
FlashAttention saves (CoROPE/flash.py:239).  Tolerance for bf16/f16 inputs
with fp32 accumulation: max-abs <= 2e-2 on O, relative L2 <= 1e-2."""
import math

import pytest
import torch

from CoROPE import _lib
from CoROPE.flash import FlashAttention, flash_attention, _forward

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
O_MAXABS, REL_L2 = 2e-2, 1e-2


def dense(q, k, v, sm, causal):
    """fp64 softmax attention of one (b, h): q, k, v [S, D]; returns o, row max."""
    s = (q @ k.T) * sm
    if causal:
        S = k.shape[0]
        s = s.masked_fill(torch.ones(q.shape[0], S, dtype=torch.bool).triu(1), float("-inf"))
    m = s.max(-1).values
    return torch.softmax(s, -1) @ v, m


def inputs(B, H, S, D, seed, dtype, hkv=None):
    hkv = H if hkv is None else hkv
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, S, D, generator=g).to(dtype)
    k = torch.randn(B, hkv, S, D, generator=g).to(dtype)
    v = torch.randn(B, hkv, S, D, generator=g).to(dtype)
    return [t.to(DEV) for t in (q, k, v)], [t.double() for t in (q, k, v)]


def check(o, m, cpu, sm, causal, slices):
    qd, kd, vd = cpu
    H, hkv = qd.shape[1], kd.shape[1]
    for b, h in slices:
        ro, rm = dense(qd[b, h], kd[b, h // (H // hkv)], vd[b, h // (H // hkv)], sm, causal)
        got = o[b, h].double().cpu()
        assert torch.isfinite(got).all()
        assert (got - ro).abs().max().item() < O_MAXABS
        assert ((got - ro).norm() / ro.norm()).item() < REL_L2
        assert (m[b, h].double().cpu() - rm).abs().max().item() < 1e-3 * max(1.0, rm.abs().max())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("B,H,S,D,hkv", [(1, 1, 1, 64, None), (2, 3, 300, 64, None),
                                         (1, 2, 128, 128, None), (1, 2, 77, 128, None),
                                         (2, 4, 1000, 128, 2), (1, 2, 513, 64, 1)])
def test_plain_attention_matches_dense_softmax(dtype, causal, B, H, S, D, hkv):
    (q, k, v), cpu = inputs(B, H, S, D, 11 + S, dtype, hkv)
    sm = 1 / math.sqrt(D)
    o, m, lse = _forward(q, k, v, causal, None, return_lse=True)
    torch.cuda.synchronize()
    assert _lib.take_device_error() == 0
    slices = [(b, h) for b in range(B) for h in range(H)]
    check(o, m, cpu, sm, causal, slices)
    # log-sum-exp of the scaled logits
    b, h = slices[-1]
    s = (cpu[0][b, h] @ cpu[1][b, h // (H // cpu[1].shape[1])].T) * sm
    if causal:
        s = s.masked_fill(torch.ones(S, S, dtype=torch.bool).triu(1), float("-inf"))
    assert (lse[b, h].double().cpu() - torch.logsumexp(s, -1)).abs().max().item() < 1e-3


def test_plain_attention_module_layout_and_autograd_surface():
    """[B, S, H, D] projections passed as strided [B, H, S, D] views give the
    contiguous result; FlashAttention saves (q, k, v, o, M) and its backward
    refuses instead of returning zero gradients."""
    B, S, H, D = 2, 200, 4, 64
    g = torch.Generator().manual_seed(5)
    x = [torch.randn(B, S, H, D, generator=g).bfloat16().to(DEV) for _ in range(3)]
    q, k, v = (t.transpose(1, 2) for t in x)
    o1 = flash_attention(q, k, v)
    o2 = flash_attention(q.contiguous(), k.contiguous(), v.contiguous())
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)
    qq = q.detach().clone().requires_grad_(True)
    out = FlashAttention.apply(qq, k, v, True, None)
    with pytest.raises(NotImplementedError):
        out.sum().backward()
    with pytest.raises(NotImplementedError):
        flash_attention(q.float(), k.float(), v.float())


def test_plain_attention_bench_shape_sampled_slices():
    """B=4, H=32, S=4096, D=128 bf16 causal (the CoRoPE bench shape): every
    row of two (b, h) slices against the dense reference."""
    (q, k, v), cpu = inputs(4, 32, 4096, 128, 1, torch.bfloat16)
    sm = 1 / math.sqrt(128)
    o, m = _forward(q, k, v, True, None)
    torch.cuda.synchronize()
    assert _lib.take_device_error() == 0
    check(o, m, cpu, sm, True, [(0, 0), (3, 31)])
