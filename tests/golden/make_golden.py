"""Generate the golden fixtures in this folder from the REFERENCE implementation.

Run where a checkout of the reference is available (read-only is enough),
passing its path:

    TRITON_INTERPRET=1 python tests/golden/make_golden.py /path/to/reference

What it records (all on CPU, fp32):

* ``check_s4.npz``      -- check.py's own __main__ case (B=H=1, S=D=4,
  torch.manual_seed(42), q,k,v,do drawn in that order): O from
  ``check.forward_reference`` and dq/dk/dv from autograd through it
  (check.py:105-148).
* ``ref_b1h2s40d8.npz``  -- B=1,H=2,S=40,D=8: O and grads from
  ``check.forward_reference`` + autograd, plus O, M, L, A from the reference
  Triton forward kernel ``co_rope_fwd_kernel`` (CoROPE/forward.py:7-120) run
  under the Triton interpreter with the launch arguments of
  CoROPE/forward.py:149-171.
* ``ref_b2h2s64d16_t500k.npz`` -- B=2,H=2,S=64,D=16, theta=5e5, same content.
* ``mqa_b1h4s48d16.npz`` -- MQA: q [1,4,48,16], k,v [1,1,48,16] and an
  explicit lower-triangular bias; O, M, L, A from the reference MQA Triton
  kernel (CoROPE/co_rope_mqa_forward.py:7-104, launch args of :151-174) under
  the interpreter.  Batch 1 only: the reference kernel offsets K/V by the
  query batch stride (co_rope_mqa_forward.py:26-27,161), so B>1 reads the
  wrong memory.
* ``config1_b1h4s256d64.npz`` -- the CPU configuration (B=1,H=4,S=256,D=64,
  fp32, theta=1e4): inputs from ``torch.Generator().manual_seed(0)`` drawing
  q,k,v,dO in order; O from ``check.forward_reference`` and grads by autograd.

The fixtures are the oracle's pin: tests/test_oracle.py checks the CPU
restatement in ``oracle/`` against them, and the GPU tests check the CUDA
kernels against them.
"""
import math
import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

if len(sys.argv) != 2:
    sys.exit("usage: TRITON_INTERPRET=1 python tests/golden/make_golden.py /path/to/reference")
REF = sys.argv[1]
sys.path.insert(0, REF)
HERE = os.path.dirname(os.path.abspath(__file__))

import check  # noqa: E402  (reference module)
from CoROPE.forward import co_rope_fwd_kernel  # noqa: E402
from CoROPE.co_rope_mqa_forward import co_rope_mqa_fwd_kernel  # noqa: E402


def ref_autograd(q, k, v, do, sm_scale, theta):
    qq = q.clone().requires_grad_(True)
    kk = k.clone().requires_grad_(True)
    vv = v.clone().requires_grad_(True)
    o, _ = check.forward_reference(qq, kk, vv, sm_scale=sm_scale, theta=theta)
    o.backward(do)
    return o.detach(), qq.grad, kk.grad, vv.grad


def ref_triton_fwd(q, k, v, sm_scale, theta):
    """CoROPE/forward.py:123-178 with the CUDA assert removed (CPU tensors,
    interpreter).  Same launch arguments."""
    B, H, S, D = q.shape
    thetas = 1.0 / (theta ** (torch.arange(0, D, 2).float() / D))
    thetas = thetas.repeat_interleave(2)
    o = torch.empty_like(q)
    m = torch.empty(B, H, S)
    l = torch.empty(B, H, S)
    a = torch.empty(B, H, S)
    co_rope_fwd_kernel[(S, B * H)](
        Q=q.contiguous(), K=k.contiguous(), V=v.contiguous(), O=o, M=m, L=l, A=a,
        thetas=thetas, stride_batch=q.stride(0), stride_head=q.stride(1),
        stride_seq=q.stride(2), stride_dim=q.stride(3), stride_a=a.stride(1),
        seq_len=S, SM_SCALE=sm_scale, BLOCK_M=1, BLOCK_N=32, NUM_HEADS=H,
        HEAD_DIM=D, CAUSAL=True, CAUSAL_MASK_VALUE=-torch.finfo(torch.float32).max)
    return o, m, l, a


def ref_triton_mqa(q, k, v, bias, sm_scale, theta):
    """CoROPE/co_rope_mqa_forward.py:107-176 with the random bias replaced by
    ``bias`` (same shape and role) and the CUDA assert removed."""
    B, H, S, D = q.shape
    assert B == 1
    thetas = 1.0 / (theta ** (torch.arange(0, D, 2).float() / D))
    thetas = thetas.repeat_interleave(2)
    o = torch.empty_like(q)
    m = torch.empty(B, H, S)
    l = torch.empty(B, H, S)
    a = torch.empty(B, H, S)
    co_rope_mqa_fwd_kernel[(S, B * H)](
        Q=q.contiguous(), K=k.contiguous(), V=v.contiguous(), O=o, M=m, L=l, A=a,
        thetas=thetas, contextual_bias=bias, stride_batch=q.stride(0),
        stride_head=q.stride(1), stride_seq=q.stride(2), stride_dim=q.stride(3),
        stride_a=a.stride(1), seq_len=S, SM_SCALE=sm_scale, BLOCK_M=1, BLOCK_N=32,
        NUM_HEADS=H, HEAD_DIM=D, CAUSAL=True,
        CAUSAL_MASK_VALUE=-torch.finfo(torch.float32).max)
    return o, m, l, a


def save(name, **arrs):
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **{k: (v.detach().numpy() if torch.is_tensor(v) else np.asarray(v))
                                 for k, v in arrs.items()})
    print("wrote", path, os.path.getsize(path), "bytes")


def case_check_main():
    torch.manual_seed(42)
    q = torch.randn(1, 1, 4, 4)
    k = torch.randn(1, 1, 4, 4)
    v = torch.randn(1, 1, 4, 4)
    do = torch.randn(1, 1, 4, 4)
    sm = 1.0 / math.sqrt(4)
    o, dq, dk, dv = ref_autograd(q, k, v, do, sm, 10000.0)
    save("check_s4.npz", q=q, k=k, v=v, do=do, sm_scale=sm, theta=10000.0,
         o=o, dq=dq, dk=dk, dv=dv)


def case_mha(name, B, H, S, D, theta, seed):
    g = torch.Generator().manual_seed(seed)
    q, k, v, do = (torch.randn(B, H, S, D, generator=g) for _ in range(4))
    sm = 1.0 / math.sqrt(D)
    o, dq, dk, dv = ref_autograd(q, k, v, do, sm, theta)
    to, tm, tl, ta = ref_triton_fwd(q, k, v, sm, theta)
    save(name, q=q, k=k, v=v, do=do, sm_scale=sm, theta=theta, o=o, dq=dq, dk=dk,
         dv=dv, tri_o=to, tri_m=tm, tri_l=tl, tri_a=ta)


def case_mqa():
    g = torch.Generator().manual_seed(7)
    B, H, S, D = 1, 4, 48, 16
    q = torch.randn(B, H, S, D, generator=g)
    k = torch.randn(B, 1, S, D, generator=g)
    v = torch.randn(B, 1, S, D, generator=g)
    bias = torch.tril(torch.randn(S, S, generator=g) * 0.02)
    sm = 1.0 / math.sqrt(D)
    theta = 10000.0
    to, tm, tl, ta = ref_triton_mqa(q, k, v, bias, sm, theta)
    save("mqa_b1h4s48d16.npz", q=q, k=k, v=v, bias=bias, sm_scale=sm, theta=theta,
         tri_o=to, tri_m=tm, tri_l=tl, tri_a=ta)


def case_config1():
    B, H, S, D = 1, 4, 256, 64
    g = torch.Generator().manual_seed(0)
    q, k, v, do = (torch.randn(B, H, S, D, generator=g) for _ in range(4))
    sm = 1.0 / math.sqrt(D)
    o, dq, dk, dv = ref_autograd(q, k, v, do, sm, 10000.0)
    save("config1_b1h4s256d64.npz", q=q, k=k, v=v, do=do, sm_scale=sm, theta=10000.0,
         o=o, dq=dq, dk=dk, dv=dv)


if __name__ == "__main__":
    torch.set_num_threads(os.cpu_count() or 1)
    case_check_main()
    case_mha("ref_b1h2s40d8.npz", 1, 2, 40, 8, 10000.0, 3)
    case_mha("ref_b2h2s64d16_t500k.npz", 2, 2, 64, 16, 500000.0, 5)
    case_mqa()
    case_config1()
