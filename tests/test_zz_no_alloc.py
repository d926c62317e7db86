"""corope_bwd_noalloc: the backward for callers that cannot allocate device
memory (a host engine whose plugin interface passes only input and output
buffers, or a process running under a fixed, pre-reserved memory budget).

It takes its scratch from an array built into the library instead of a
caller workspace.  This test calls it through the C ABI twice in a row and
compares dq, dk, dv with corope_bwd given torch-allocated workspaces (one of
the scratch's size, one full), on a small shape and on one near the
scratch's limit; it also checks that an oversized shape is refused.  It
lives in its own file, collected last, so that a failure here leaves every
other test already run.
"""
import ctypes
import math

import pytest
import torch

from CoROPE import _lib
from CoROPE.forward import co_rope_forward

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
# Against corope_bwd with a workspace of the scratch's size the kernels are
# the same and only the order of the fp32 atomic adds differs (one bf16 ulp
# here and there): the suite's bf16 gradient tolerance (max-abs 5e-2) and a
# relative L2 bound far tighter than its 1e-2.  Against the full workspace
# the dK side may take another path (reading the dQ kernel's per-pair
# results instead of recomputing them, with another expansion length), so
# that comparison uses the suite's own bounds.
G_MAXABS, REL_L2_SAME, REL_L2_OTHER = 5e-2, 1e-3, 1e-2


def _params(q, k, v, o, do, m, l, a, dq, dk, dv, sm):
    B, H, S, D = q.shape
    p = _lib.BwdParams()
    p.q, p.k, p.v, p.o, p.dout = (t.data_ptr() for t in (q, k, v, o, do))
    p.m, p.l, p.a = m.data_ptr(), l.data_ptr(), a.data_ptr()
    p.dq, p.dk, p.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    p.q_stride, p.k_stride, p.v_stride = _lib._strides(q), _lib._strides(k), _lib._strides(v)
    p.o_stride, p.do_stride = _lib._strides(o), _lib._strides(do)
    p.dq_stride, p.dk_stride, p.dv_stride = _lib._strides(dq), _lib._strides(dk), _lib._strides(dv)
    p.batch, p.heads, p.kv_heads, p.seq_len, p.head_dim = B, H, k.shape[1], S, D
    p.sm_scale, p.theta, p.causal, p.dtype, p.algo = sm, 1e4, 1, _lib._dtype_code(q), 0
    return p


def _inputs(B, H, S, D, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(B, H, S, D, generator=g).bfloat16().to(DEV) for _ in range(4)]


def _workspace_backward(lib, args, sm, nbytes, stream):
    out = [torch.empty_like(args[0]) for _ in range(3)]
    p = _params(*args, *out, sm)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    p.workspace, p.workspace_bytes = ws.data_ptr(), nbytes
    assert lib.corope_bwd(ctypes.byref(p), stream) == 0, lib.corope_last_error()
    torch.cuda.synchronize()
    return out


# (B, H, S, D): a small shape whose scratch, scaled-key panels and whole
# hand-off region fit the built-in array, and a near-cap one (bf16, D=128,
# S=4096) whose minimum scratch takes about half of it, so that the panels
# and the hand-off region do not fit and the kernels take their fallback
# paths through the remaining bytes.
@pytest.mark.parametrize("B,H,S,D", [(2, 4, 384, 64), (1, 8, 4096, 128)])
def test_noalloc_backward_matches_workspace_backward_twice(B, H, S, D):
    lib = _lib.load_library()
    q, k, v, do = _inputs(B, H, S, D, 5)
    sm = 1 / math.sqrt(D)
    saved, o = co_rope_forward(q, k, v, sm)
    m, l, a = saved[4], saved[5], saved[6]
    args = (q, k, v, o, do, m, l, a)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    cap = lib.corope_bwd_noalloc_scratch_bytes()
    probe = _params(*args, q, k, v, sm)
    assert lib.corope_bwd_min_workspace_bytes(ctypes.byref(probe)) <= cap
    full = lib.corope_bwd_workspace_bytes(ctypes.byref(probe))
    # the reference results: corope_bwd with a workspace of the scratch's size
    # (the same path through the kernels) and with its full workspace
    refs = [_workspace_backward(lib, args, sm, cap, stream),
            _workspace_backward(lib, args, sm, full, stream)]

    for _ in range(2):
        out = [torch.full_like(q, float("nan")) for _ in range(3)]
        pn = _params(*args, *out, sm)
        rc = lib.corope_bwd_noalloc(ctypes.byref(pn), stream)
        assert rc == 0, lib.corope_last_error()
        torch.cuda.synchronize()
        for ref, bound in zip(refs, (REL_L2_SAME, REL_L2_OTHER)):
            for x, y in zip(out, ref):
                assert torch.isfinite(x).all()
                d = x.float() - y.float()
                assert d.abs().max().item() < G_MAXABS
                assert (d.norm() / y.float().norm()).item() < bound


def test_noalloc_backward_refuses_oversized_shape():
    lib = _lib.load_library()
    cap = lib.corope_bwd_noalloc_scratch_bytes()
    assert cap == 64 << 20
    # dk/dv fp32 accumulators alone: 2 * B*H*S*D*4 bytes > 64 MiB
    p = _lib.BwdParams()
    fake = 1 << 20
    for n in ("q", "k", "v", "o", "dout", "m", "l", "a", "dq", "dk", "dv"):
        setattr(p, n, fake)
    B, H, S, D = 1, 16, 8192, 128
    st = _lib._I64x3(H * S * D, S * D, D)
    for n in ("q_stride", "k_stride", "v_stride", "o_stride", "do_stride", "dq_stride",
              "dk_stride", "dv_stride"):
        setattr(p, n, st)
    p.batch, p.heads, p.kv_heads, p.seq_len, p.head_dim = B, H, H, S, D
    p.sm_scale, p.theta, p.causal, p.dtype = 0.1, 1e4, 1, 2
    assert lib.corope_bwd_workspace_bytes(ctypes.byref(p)) > cap
    assert lib.corope_bwd_noalloc(ctypes.byref(p), None) == _lib.ERR_WORKSPACE
    assert b"scratch" in lib.corope_last_error()
