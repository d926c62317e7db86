"""CUDA kernels (through the C ABI) against the oracle and the golden fixtures.

Tolerances (bf16 inputs, fp32 accumulation): max-abs <= 2e-2 on O, <= 5e-2
on gradients, relative L2 <= 1e-2.  fp32 inputs through the exact kernels:
max-abs <= 1e-4 (O) and <= 1e-3 (gradients).
"""
import ctypes
import math

import pytest
import torch

from oracle import corope_oracle as O
from golden_io import load, MHA_CASES

import CoROPE
from CoROPE.co_rope_backward import co_rope_backward
from CoROPE.co_rope_mqa_forward import co_rope_mqa_forward
from CoROPE.forward import co_rope_forward

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
O_MAXABS, G_MAXABS, REL_L2 = 2e-2, 5e-2, 1e-2
# kernel families exercised by the forward parity tests
FWD_ALGOS = ["exact", "tensor"]


def rel_l2(x, y):
    """Relative L2 error; an absolute norm when the reference is zero (e.g. dq
    of a one-key sequence, where the softmax gradient vanishes exactly)."""
    x, y = x.double().cpu(), y.double().cpu()
    ny = y.norm()
    if ny < 1e-6:
        return (x - y).norm().item()
    return ((x - y).norm() / ny).item()


def maxabs(x, y):
    return (x.double().cpu() - y.double().cpu()).abs().max().item()


def inputs(B, H, S, D, seed, dtype, hkv=None):
    """q, k, v, dO ~ N(0,1) drawn in that order from a CPU generator, cast to
    dtype; returns (cuda tensors, fp64 CPU copies of the rounded values)."""
    hkv = H if hkv is None else hkv
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, S, D, generator=g)
    k = torch.randn(B, hkv, S, D, generator=g)
    v = torch.randn(B, hkv, S, D, generator=g)
    do = torch.randn(B, H, S, D, generator=g)
    cast = [t.to(dtype) for t in (q, k, v, do)]
    return [t.to(DEV) for t in cast], [t.double() for t in cast]


def algos(dtype, D):
    out = ["exact"]
    if dtype in (torch.bfloat16, torch.float16) and D in (64, 128):
        out.append("tensor")
    return out


# ---------------------------------------------------------------- golden ----
@pytest.mark.parametrize("name", MHA_CASES)
def test_golden_forward_backward_fp32_exact(name):
    f = load(name)
    q, k, v, do = (f[x].to(DEV) for x in ("q", "k", "v", "do"))
    saved, o = co_rope_forward(q, k, v, f["sm_scale"], theta=f["theta"], algo="exact")
    assert maxabs(o, f["o"]) < 1e-4
    if "tri_m" in f:
        assert maxabs(saved[4], f["tri_m"]) < 1e-4
        assert maxabs(saved[6], f["tri_a"]) < 1e-4
        assert ((saved[5].cpu() - f["tri_l"]).abs() / f["tri_l"]).max() < 1e-4
    dq, dk, dv = co_rope_backward(saved, do, f["sm_scale"], f["theta"], algo="exact")
    for mine, ref in ((dq, f["dq"]), (dk, f["dk"]), (dv, f["dv"])):
        assert maxabs(mine, ref) < 1e-3 * max(1.0, ref.abs().max().item())


def test_golden_mqa_bias_exact():
    f = load("mqa_b1h4s48d16.npz")
    q, k, v, bias = (f[x].to(DEV) for x in ("q", "k", "v", "bias"))
    saved, o = co_rope_mqa_forward(q, k, v, f["sm_scale"], theta=f["theta"],
                                   contextual_bias=bias, algo="exact")
    assert maxabs(o, f["tri_o"]) < 1e-4
    assert maxabs(saved[4], f["tri_m"]) < 1e-4
    assert maxabs(saved[6], f["tri_a"]) < 1e-4


# ------------------------------------------------------- sampled forward ----
def check_rows(o, m, a, cpu, b, h, rows, sm, theta, hkv_div=1, bias=None):
    qd, kd, vd = cpu[0], cpu[1], cpu[2]
    ro, rm, rl, ra = O.forward_rows(qd[b, h], kd[b, h // hkv_div], vd[b, h // hkv_div], rows, sm,
                                    theta, bias=bias)
    got = o[b, h, rows].cpu()
    assert maxabs(got, ro) < O_MAXABS
    assert rel_l2(got, ro) < REL_L2
    assert maxabs(m[b, h, rows], rm) < 2e-2
    assert maxabs(a[b, h, rows], ra) < 2e-3 * max(1.0, ra.abs().max().item())


def sample_rows(S, n=24):
    r = torch.unique(torch.cat([torch.tensor([0, 1, S - 1, S - 2]),
                                torch.randint(0, S, (n,), generator=torch.Generator().manual_seed(S))]))
    return r


@pytest.mark.parametrize("algo", FWD_ALGOS)
def test_config2_forward_bf16_sampled(algo):
    """B=4, H=32, S=4096, D=128 bf16, seed 1, theta 1e4 (fwd, fp32 LSE)."""
    (q, k, v, _), cpu = inputs(4, 32, 4096, 128, 1, torch.bfloat16)
    sm = 1 / math.sqrt(128)
    saved, o, lse = co_rope_forward(q, k, v, sm, theta=1e4, algo=algo, return_lse=True)
    torch.cuda.synchronize()
    m, l, a = saved[4], saved[5], saved[6]
    assert torch.isfinite(o).all() and torch.isfinite(lse).all()
    assert torch.allclose(lse, m + torch.log(l), atol=1e-5)
    rows = sample_rows(4096)
    for b, h in ((0, 0), (3, 31), (1, 17)):
        check_rows(o, m, a, cpu, b, h, rows, sm, 1e4)


def test_bench_workload_forward_backward():
    """The bench step itself: B=4, H=32, S=4096, D=128 bf16, theta 1e4, on the
    bench's own inputs (``bench.make_inputs``), forward + backward through the
    public API with the default ("auto") workspace, as ``bench.py`` runs it.
    Against the per-row oracle: dq of sampled rows and dk, dv of the last 32
    keys (every row that reaches them is sampled) on three (b, h) slices, and
    the forward of every row of a fourth slice."""
    import bench
    from CoROPE import _lib
    B, H, S, D, theta = 4, 32, 4096, 128, 1e4
    assert (bench.WORKLOAD["B"], bench.WORKLOAD["H"], bench.WORKLOAD["S"], bench.WORKLOAD["D"],
            bench.WORKLOAD["theta"]) == (B, H, S, D, theta)
    q, k, v, do = bench.make_inputs(0, torch.device(DEV))
    sm = 1 / math.sqrt(D)
    saved, o = co_rope_forward(q, k, v, sm, theta=theta)
    dq, dk, dv = co_rope_backward(saved, do, sm, theta)
    torch.cuda.synchronize()
    assert _lib.take_device_error() == 0
    m, a = saved[4], saved[6]
    cpu = [t.double().cpu() for t in (q, k, v, do)]
    n = 32
    rows = torch.cat([torch.tensor([0, 1]),
                      torch.randint(2, S - n, (6,), generator=torch.Generator().manual_seed(5)),
                      torch.arange(S - n, S)])
    for b, h in ((0, 0), (3, 31), (1, 17)):
        rq, rk, rv = O.backward_rows(cpu[0][b, h], cpu[1][b, h], cpu[2][b, h], cpu[3][b, h],
                                     rows, sm, theta)
        for name, mine, r in (("dq", dq[b, h, rows], rq), ("dk", dk[b, h, S - n:], rk[S - n:]),
                              ("dv", dv[b, h, S - n:], rv[S - n:])):
            assert torch.isfinite(mine).all(), name
            assert maxabs(mine, r) < G_MAXABS, (name, b, h)
            assert rel_l2(mine, r) < REL_L2, (name, b, h)
    check_rows(o, m, a, cpu, 2, 7, torch.arange(S), sm, theta)


@pytest.mark.parametrize("algo", FWD_ALGOS)
def test_config4_mqa_forward_bf16_sampled(algo):
    """MQA: B=4, Hq=32, Hkv=1, S=8192, D=128 bf16, seed 3, theta 5e5."""
    (q, k, v, _), cpu = inputs(4, 32, 8192, 128, 3, torch.bfloat16, hkv=1)
    sm = 1 / math.sqrt(128)
    saved, o = co_rope_mqa_forward(q, k, v, sm, theta=5e5, algo=algo)
    torch.cuda.synchronize()
    rows = sample_rows(8192, 12)
    for b, h in ((0, 0), (3, 31), (2, 5)):
        check_rows(o, saved[4], saved[6], cpu, b, h, rows, sm, 5e5, hkv_div=32)


def test_mqa_reference_bias_draw_is_reproducible():
    (q, k, v, _), cpu = inputs(2, 4, 256, 64, 9, torch.bfloat16, hkv=1)
    torch.manual_seed(123)
    s1, o1, b1 = co_rope_mqa_forward(q, k, v, None, contextual_bias="reference", return_bias=True)
    torch.manual_seed(123)
    expect = torch.tril(torch.randn(256, 256, device=DEV) * 0.02)
    assert torch.equal(b1, expect)
    rows = sample_rows(256, 8)
    for b, h in ((0, 0), (1, 3)):
        check_rows(o1, s1[4], s1[6], cpu, b, h, rows, 1 / 8, 1e4, hkv_div=4, bias=expect.double().cpu())


# ------------------------------------------------------ full fwd + bwd ----
@pytest.mark.parametrize("algo", ["exact", "tensor"])
def test_config3_forward_backward_bf16(algo):
    """B=8, H=16, S=2048, D=64 bf16, seed 2, theta 1e4: dq, dk, dv of two
    (b, h) slices against the closed-form oracle gradients, on both kernel
    families (the tensor-core backward at D=64 keeps its transposed GEMMs
    at M=128 with a zero second slab)."""
    (q, k, v, do), cpu = inputs(8, 16, 2048, 64, 2, torch.bfloat16)
    sm = 1 / math.sqrt(64)
    saved, o = co_rope_forward(q, k, v, sm, theta=1e4, algo=algo)
    dq, dk, dv = co_rope_backward(saved, do, sm, 1e4, algo=algo)
    torch.cuda.synchronize()
    for b, h in ((0, 0), (7, 15)):
        sl = [t[b:b + 1, h:h + 1].float() for t in cpu]
        ref = O.forward_dense(sl[0], sl[1], sl[2], sm, 1e4)
        assert maxabs(o[b, h], ref["o"][0, 0]) < O_MAXABS
        rq, rk, rv = O.backward_dense(sl[0], sl[1], sl[2], sl[3], sm, 1e4, row_chunk=32)
        for mine, r in ((dq, rq), (dk, rk), (dv, rv)):
            assert maxabs(mine[b, h], r[0, 0]) < G_MAXABS
            assert rel_l2(mine[b, h], r[0, 0]) < REL_L2


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("S,D,H,hkv", [(1, 64, 2, 2), (77, 32, 3, 3), (200, 128, 2, 1),
                                        (129, 16, 4, 2), (64, 64, 2, 2)])
def test_edge_shapes_forward_backward(dtype, S, D, H, hkv):
    """Ragged S (not a tile multiple), S = 1, odd head counts, GQA/MQA
    grouping in the backward, every dtype."""
    (q, k, v, do), cpu = inputs(2, H, S, D, 11, dtype, hkv=hkv)
    sm = 1 / math.sqrt(D)
    fn = co_rope_forward if hkv == H else co_rope_mqa_forward
    if hkv not in (1, H):
        # grouped heads go through the C ABI's MQA entry (kv_heads < heads)
        from CoROPE import _lib
        o = torch.empty_like(q)
        m, l, a = (torch.empty(2, H, S, device=DEV) for _ in range(3))
        _lib.fwd(q, k, v, o, m, l, a, None, sm, 1e4, algo="exact", mqa=True)
        saved = (q, k, v, o, m, l, a)
    else:
        saved, o = fn(q, k, v, sm, algo="exact")
    dq, dk, dv = co_rope_backward(saved, do, sm, 1e4, algo="exact")
    ref = O.forward_dense(*[t.float() for t in cpu[:3]], sm, 1e4)
    rq, rk, rv = O.backward_dense(*[t.float() for t in cpu], sm, 1e4)
    tol_o = 1e-4 if dtype == torch.float32 else O_MAXABS
    tol_g = 1e-3 if dtype == torch.float32 else G_MAXABS
    assert maxabs(o, ref["o"]) < tol_o
    assert maxabs(saved[6], ref["a"]) < 1e-3
    for mine, r in ((dq, rq), (dk, rk), (dv, rv)):
        assert maxabs(mine, r) < tol_g * max(1.0, r.abs().max().item())


def test_strided_inputs_and_module():
    """CoRoPEAttention passes [B,S,H,D]-strided views; gradients through the
    autograd Function equal those of contiguous inputs."""
    torch.manual_seed(0)
    B, S, H, D = 2, 96, 4, 32
    base = torch.randn(3, B, S, H, D, device=DEV)
    q, k, v = (base[i].transpose(1, 2).requires_grad_(True) for i in range(3))
    out = CoROPE.CoRoPEAttentionFunction.apply(q, k, v, True, None, 10000.0)
    g = torch.randn_like(out)
    out.backward(g)
    qc, kc, vc = (x.detach().contiguous().requires_grad_(True) for x in (q, k, v))
    outc = CoROPE.CoRoPEAttentionFunction.apply(qc, kc, vc, True, None, 10000.0)
    outc.backward(g.contiguous())
    assert maxabs(out, outc) < 1e-5
    for a_, b_ in ((q.grad, qc.grad), (k.grad, kc.grad), (v.grad, vc.grad)):
        assert maxabs(a_, b_) < 1e-4
    mod = CoROPE.CoRoPEAttention(128, 4).to(DEV)
    x = torch.randn(2, 64, 128, device=DEV)
    y = mod(x)
    assert y.shape == x.shape and torch.isfinite(y).all()
    y.sum().backward()
    for p in mod.parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all()


def test_linearity_in_v_full_size():
    """O is linear in V for fixed q, k: a size-independent property checked
    at the config-2 shape."""
    (q, k, v, do), _ = inputs(4, 32, 4096, 128, 1, torch.bfloat16)
    _, o1 = co_rope_forward(q, k, v, None)
    _, o2 = co_rope_forward(q, k, do, None)
    _, o3 = co_rope_forward(q, k, (v.float() + do.float()).bfloat16(), None)
    assert rel_l2(o3, o1.float() + o2.float()) < 1e-2


def test_state_bounds_full_size():
    """0 <= A_t <= t+1, 1 <= L_t <= t+1, M_t finite -- at the config-2 shape."""
    (q, k, v, _), _ = inputs(4, 32, 4096, 128, 1, torch.bfloat16)
    saved, _ = co_rope_forward(q, k, v, None)
    m, l, a = saved[4], saved[5], saved[6]
    t1 = torch.arange(1, 4097, device=DEV, dtype=torch.float32)
    assert (a >= 0).all() and (a <= t1 + 1e-3).all()
    assert (l >= 1 - 1e-5).all() and (l <= t1 * (1 + 1e-5)).all()
    assert torch.isfinite(m).all()


def test_exact_and_tensor_agree_on_gate_sum():
    (q, k, v, _), _ = inputs(1, 4, 1024, 128, 5, torch.bfloat16)
    s1, o1 = co_rope_forward(q, k, v, None, algo="exact")
    try:
        s2, o2 = co_rope_forward(q, k, v, None, algo="tensor")
    except NotImplementedError:
        pytest.skip("tensor-core forward not built")
    assert maxabs(s1[6], s2[6]) < 1e-2
    assert maxabs(o1, o2) < O_MAXABS


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("S,D,theta", [(1, 64, 1e4), (40, 128, 1e4), (300, 64, 1e4),
                                        (513, 128, 5e5), (1024, 128, 1e4)])
def test_tensor_forward_small_shapes(dtype, S, D, theta):
    """Tensor-core forward against the full oracle: ragged S (partial
    windows, tiles and query tiles), both head dims, both half types."""
    (q, k, v, _), cpu = inputs(2, 3, S, D, 21, dtype)
    sm = 1 / math.sqrt(D)
    saved, o, lse = co_rope_forward(q, k, v, sm, theta=theta, algo="tensor", return_lse=True)
    torch.cuda.synchronize()
    from CoROPE import _lib
    assert _lib.take_device_error() == 0
    ref = O.forward_dense(*[t.double() for t in cpu[:3]], sm, theta)
    assert maxabs(o, ref["o"]) < O_MAXABS
    assert rel_l2(o, ref["o"]) < REL_L2
    assert maxabs(saved[4], ref["m"]) < 2e-2
    assert maxabs(saved[6], ref["a"]) < 1e-3 * max(1.0, S / 100)
    assert maxabs(lse, ref["lse"]) < 2e-2


def test_tensor_forward_strided_module_layout():
    """[B,S,H,D]-strided views (the CoRoPEAttention layout) go straight to
    the TMA descriptors."""
    torch.manual_seed(3)
    B, S, H, D = 2, 200, 4, 128
    base = torch.randn(3, B, S, H, D, device=DEV).bfloat16()
    q, k, v = (base[i].transpose(1, 2) for i in range(3))
    _, o1 = co_rope_forward(q, k, v, None, algo="tensor")
    _, o2 = co_rope_forward(q.contiguous(), k.contiguous(), v.contiguous(), None, algo="tensor")
    assert maxabs(o1, o2) == 0.0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("S,theta,hkv", [(1, 1e4, 3), (40, 1e4, 3), (300, 1e4, 3), (513, 5e5, 3),
                                         (300, 1e4, 1)])
@pytest.mark.parametrize("D", [64, 128])
def test_tensor_backward_small_shapes(dtype, S, theta, hkv, D):
    """Tensor-core backward (D=64 and 128) against the closed-form oracle
    gradients: ragged S (partial windows and query tiles), both half types, MQA
    grouping (k/v gradients summed over the heads that share a K/V head)."""
    H = 3
    (q, k, v, do), cpu = inputs(2, H, S, D, 31, dtype, hkv=hkv)
    sm = 1 / math.sqrt(D)
    from CoROPE import _lib
    if hkv == H:
        saved, o = co_rope_forward(q, k, v, sm, theta=theta, algo="tensor")
    else:
        saved, o = co_rope_mqa_forward(q, k, v, sm, theta=theta, algo="tensor")
    dq, dk, dv = co_rope_backward(saved, do, sm, theta, algo="tensor")
    torch.cuda.synchronize()
    assert _lib.take_device_error() == 0
    rq, rk, rv = O.backward_dense(*[t.double() for t in cpu], sm, theta)
    for name, mine, r in (("dq", dq, rq), ("dk", dk, rk), ("dv", dv, rv)):
        assert torch.isfinite(mine).all(), name
        assert maxabs(mine, r) < G_MAXABS, name
        assert rel_l2(mine, r) < REL_L2, name


def test_tensor_backward_s2048_d128():
    """B=1, H=2, S=2048, D=128 bf16: full gradients of both heads."""
    (q, k, v, do), cpu = inputs(1, 2, 2048, 128, 41, torch.bfloat16)
    sm = 1 / math.sqrt(128)
    saved, o = co_rope_forward(q, k, v, sm, algo="tensor")
    dq, dk, dv = co_rope_backward(saved, do, sm, algo="tensor")
    torch.cuda.synchronize()
    rq, rk, rv = O.backward_dense(*[t.float() for t in cpu], sm, 1e4, row_chunk=32)
    for name, mine, r in (("dq", dq, rq), ("dk", dk, rk), ("dv", dv, rv)):
        assert maxabs(mine, r) < G_MAXABS, name
        assert rel_l2(mine, r) < REL_L2, name


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("mode", ["full", "chunked", "chunked-no-panels", "panels", "min"])
def test_tensor_backward_workspace_paths(mode, D):
    """The ways the tensor-core backward uses its workspace give the oracle's
    gradients: scaled-key panels plus a full hand-off region (the dK kernel
    reads the dQ kernel's per-pair results), panels plus a region for 17 of
    the 24 (b, h) slices (two rounds of both kernels), panels alone (the dK
    kernel recomputes), and the minimum (no panels: the dQ kernel builds its
    operands, the dK kernel recomputes) -- and 16 slices without the panels
    (the dQ kernel builds its operands, both kernels run slice by slice)."""
    from CoROPE import _lib
    B, H, S = 2, 12, 300
    (q, k, v, do), cpu = inputs(B, H, S, D, 57, torch.bfloat16)
    sm = 1 / math.sqrt(D)
    saved, o = co_rope_forward(q, k, v, sm, algo="tensor")
    q_, k_, v_, o_, m_, l_, a_ = saved
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)

    def sizes():
        p = _lib.BwdParams()
        p.theta, p.sm_scale = 1e4, sm
        p.batch, p.heads, p.kv_heads, p.seq_len, p.head_dim = B, H, H, S, D
        p.dtype, p.algo = _lib._dtype_code(q), _lib.algo_code("tensor")
        lib = _lib.load_library()
        return (lib.corope_bwd_min_workspace_bytes(ctypes.byref(p)),
                lib.corope_bwd_workspace_bytes(ctypes.byref(p)),
                lib.corope_bwd_panel_bytes(ctypes.byref(p)))

    lo, hi, panels = sizes()
    per_bh = (hi - lo - panels) // (B * H)
    assert panels > 0 and per_bh > 0 and lo + panels + per_bh * B * H == hi
    ws = {"full": "full", "min": "min", "panels": lo + panels,
          "chunked": lo + panels + 17 * per_bh,
          # 16 slices (the fewest a launch takes at this length) fit but the
          # panels do not (they come first when they fit)
          "chunked-no-panels": lo + 16 * per_bh}[mode]
    if mode == "chunked-no-panels":
        assert 16 * per_bh < panels
    _lib.bwd(q_, k_, v_, o_, do, m_, l_, a_, dq, dk, dv, sm, 1e4, algo="tensor", workspace=ws)
    torch.cuda.synchronize()
    assert _lib.take_device_error() == 0
    rq, rk, rv = O.backward_dense(*[t.double() for t in cpu], sm, 1e4)
    for name, mine, r in (("dq", dq, rq), ("dk", dk, rk), ("dv", dv, rv)):
        assert torch.isfinite(mine).all(), name
        assert maxabs(mine, r) < G_MAXABS, name
        assert rel_l2(mine, r) < REL_L2, name


@pytest.mark.parametrize("mode", ["auto", "two-slices", "min"])
def test_long_context_s32768(mode):
    """The long-context shape of one GPU's share (S=32768, D=128 bf16, theta
    5e5, seed 4) on 4 heads: forward rows and the backward against the
    per-row oracle -- dq of sampled rows, dk and dv of the last 32 keys (whose
    contributing rows are all sampled) -- with the "auto" workspace (the whole
    hand-off region of the 4 slices, 4.3 GB, after the panels), two (b, h)
    slices at a time (the fewest a launch takes at this length), or none."""
    from CoROPE import _lib
    B, H, S, D, theta = 1, 4, 32768, 128, 5e5
    (q, k, v, do), cpu = inputs(B, H, S, D, 4, torch.bfloat16)
    sm = 1 / math.sqrt(D)
    saved, o = co_rope_forward(q, k, v, sm, theta=theta, algo="tensor")
    q_, k_, v_, o_, m_, l_, a_ = saved
    p = _lib.BwdParams()
    p.batch, p.heads, p.kv_heads, p.seq_len, p.head_dim = B, H, H, S, D
    p.dtype, p.algo = _lib._dtype_code(q), _lib.algo_code("tensor")
    p.theta, p.sm_scale = theta, sm  # the sizes depend on them (theta < 1: exact kernels)
    lib = _lib.load_library()
    lo = lib.corope_bwd_min_workspace_bytes(ctypes.byref(p))
    hi = lib.corope_bwd_workspace_bytes(ctypes.byref(p))
    panels = lib.corope_bwd_panel_bytes(ctypes.byref(p))
    per_bh = (hi - lo - panels) // (B * H)
    ws = {"auto": "auto", "min": "min", "two-slices": lo + panels + 2 * per_bh}[mode]
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    _lib.bwd(q_, k_, v_, o_, do, m_, l_, a_, dq, dk, dv, sm, theta, algo="tensor", workspace=ws)
    torch.cuda.synchronize()
    assert _lib.take_device_error() == 0
    n = 32
    rows = torch.cat([torch.tensor([0, 1, 777, 9000, 20000]), torch.arange(S - n, S)])
    for h in (0, 3):
        if mode == "auto":
            check_rows(o, m_, a_, cpu, 0, h, rows, sm, theta)
        rq, rk, rv = O.backward_rows(cpu[0][0, h], cpu[1][0, h], cpu[2][0, h], cpu[3][0, h],
                                     rows, sm, theta)
        for name, mine, r in (("dq", dq[0, h, rows], rq), ("dk", dk[0, h, S - n:], rk[S - n:]),
                              ("dv", dv[0, h, S - n:], rv[S - n:])):
            assert torch.isfinite(mine).all(), name
            assert maxabs(mine, r) < G_MAXABS, name
            assert rel_l2(mine, r) < REL_L2, name


@pytest.mark.parametrize("algo", ["exact", "tensor"])
@pytest.mark.parametrize("D", [64, 128])
def test_backward_with_contextual_bias(algo, D):
    """MQA forward and backward with an additive [S, S] bias (the reference MQA
    kernel's extra term), gradients against the closed-form oracle."""
    B, H, S = 1, 4, 200
    (q, k, v, do), cpu = inputs(B, H, S, D, 71, torch.bfloat16, hkv=1)
    g = torch.Generator().manual_seed(72)
    bias = (torch.randn(S, S, generator=g) * 0.5).tril()
    sm = 1 / math.sqrt(D)
    saved, o = co_rope_mqa_forward(q, k, v, sm, contextual_bias=bias.to(DEV), algo=algo)
    dq, dk, dv = co_rope_backward(saved, do, sm, 1e4, algo=algo, contextual_bias=bias.to(DEV))
    torch.cuda.synchronize()
    from CoROPE import _lib
    assert _lib.take_device_error() == 0
    ref = O.forward_dense(*[t.double() for t in cpu[:3]], sm, 1e4, bias=bias.double())
    assert maxabs(o, ref["o"]) < O_MAXABS
    rq, rk, rv = O.backward_dense(*[t.double() for t in cpu], sm, 1e4, bias=bias.double())
    for name, mine, r in (("dq", dq, rq), ("dk", dk, rk), ("dv", dv, rv)):
        assert torch.isfinite(mine).all(), name
        assert maxabs(mine, r) < G_MAXABS, name
        assert rel_l2(mine, r) < REL_L2, name


@pytest.mark.parametrize("algo,D,hkv", [("tensor", 128, None), ("tensor", 64, 1), ("exact", 64, None)])
def test_query_chunks_equal_whole_sequence(algo, D, hkv):
    """corope_fwd_chunk / corope_bwd_chunk over the query chunks of a
    sequence (as the ranks of a sequence-sharded job would run them, here one
    after the other on one GPU) reproduce the whole-sequence calls: O, M, L, A
    and dq bit for bit (each row is computed the same way), dk / dv up to the
    order of the fp32 additions."""
    from CoROPE import _lib
    B, H, S = 2, 4, 1024
    (q, k, v, do), cpu = inputs(B, H, S, D, 81, torch.bfloat16, hkv=hkv)
    sm = 1 / math.sqrt(D)
    mqa = hkv is not None
    fwd = co_rope_mqa_forward if mqa else co_rope_forward
    saved, o = fwd(q, k, v, sm, theta=5e5, algo=algo)
    m, l, a = saved[4], saved[5], saved[6]
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    _lib.bwd(q, k, v, o, do, m, l, a, dq, dk, dv, sm, 5e5, algo=algo)
    # four query chunks, visited in a shuffled order
    bounds = [(0, 256), (256, 640), (640, 768), (768, 1024)]
    oc, dqc = torch.empty_like(o), torch.empty_like(dq)
    dk_acc = torch.zeros(k.shape, dtype=torch.float32, device=DEV)
    dv_acc = torch.zeros_like(dk_acc)
    for r0, r1 in (bounds[2], bounds[0], bounds[3], bounds[1]):
        n = r1 - r0
        mc, lc, ac = (torch.empty(B, H, n, device=DEV) for _ in range(3))
        _lib.fwd(q[:, :, r0:r1], k, v, oc[:, :, r0:r1], mc, lc, ac, None, sm, 5e5, algo=algo,
                 mqa=True, q_row0=r0)
        assert torch.equal(mc, m[:, :, r0:r1]) and torch.equal(lc, l[:, :, r0:r1])
        assert torch.equal(ac, a[:, :, r0:r1])
        _lib.bwd(q[:, :, r0:r1], k, v, oc[:, :, r0:r1], do[:, :, r0:r1], mc, lc, ac,
                 dqc[:, :, r0:r1], None, None, sm, 5e5, algo=algo, q_row0=r0,
                 dk_accum=dk_acc, dv_accum=dv_acc)
    torch.cuda.synchronize()
    assert _lib.take_device_error() == 0
    assert torch.equal(oc, o)
    assert torch.equal(dqc, dq)
    for name, mine, ref in (("dk", dk_acc, dk), ("dv", dv_acc, dv)):
        ref = ref.float()
        assert (mine - ref).abs().max().item() <= 1e-2 * ref.abs().max().item() + 1e-6, name
        assert rel_l2(mine.to(ref.dtype), ref) < 5e-3, name


def test_query_chunk_argument_checks():
    """Chunk offsets off the 128-row tiles and key ranges too short for the
    chunk are refused before any device work."""
    from CoROPE import _lib
    (q, k, v, _), _ = inputs(1, 2, 256, 64, 5, torch.bfloat16)
    o = torch.empty_like(q)
    m, l, a = (torch.empty(1, 2, 128, device=DEV) for _ in range(3))
    with pytest.raises(ValueError):
        _lib.fwd(q[:, :, 100:228], k, v, o[:, :, 100:228], m, l, a, None, 0.125, 1e4,
                 mqa=True, q_row0=100)
    with pytest.raises(ValueError):
        _lib.fwd(q[:, :, 128:256], k[:, :, :200], v[:, :, :200], o[:, :, 128:256], m, l, a,
                 None, 0.125, 1e4, mqa=True, q_row0=128)


@pytest.mark.parametrize("algo,ws,hkv,dtype", [
    ("tensor", "auto", 4, torch.bfloat16),   # dQ kernel + dK kernel via the hand-off
    ("tensor", "min", 4, torch.bfloat16),    # the dK side recomputed (no hand-off)
    ("tensor", "auto", 1, torch.float16),    # 4 query heads add to each key row
    ("exact", "auto", 4, torch.float32),
])
def test_deterministic_backward_is_bit_identical(algo, ws, hkv, dtype):
    """COROPE_BWD_DETERMINISTIC: two calls give bit-identical dq, dk, dv (the
    fp32-atomic default need not), equal to the default within rounding and
    to the oracle within the gradient bounds."""
    from CoROPE import _lib
    B, H, S, D = 2, 4, 640, 64
    (q, k, v, do), cpu = inputs(B, H, S, D, 61, dtype, hkv=hkv)
    sm = 1 / math.sqrt(D)
    fwd = co_rope_forward if hkv == H else co_rope_mqa_forward
    saved, o = fwd(q, k, v, sm, algo=algo)
    q_, k_, v_, o_, m_, l_, a_ = saved

    def run(det):
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        _lib.bwd(q_, k_, v_, o_, do, m_, l_, a_, dq, dk, dv, sm, 1e4, algo=algo, workspace=ws,
                 deterministic=det)
        return dq, dk, dv

    first = run(True)
    second = run(True)
    plain = run(False)
    torch.cuda.synchronize()
    assert _lib.take_device_error() == 0
    for x, y in zip(first, second):
        assert torch.equal(x, y)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    for x, y in zip(first, plain):
        assert maxabs(x, y) < tol * max(1.0, y.abs().max().item())
    rq, rk, rv = O.backward_dense(*cpu, sm, 1e4)
    g_tol = 1e-3 if dtype == torch.float32 else G_MAXABS
    for name, mine, r in zip(("dq", "dk", "dv"), first, (rq, rk, rv)):
        assert maxabs(mine, r) < g_tol * max(1.0, r.abs().max().item()), name
        assert rel_l2(mine, r) < REL_L2, name
    # the public call takes the same path
    dq, dk, dv = co_rope_backward(saved, do, sm, algo=algo, deterministic=True)
    if ws == "auto":
        assert torch.equal(dk, first[1]) and torch.equal(dv, first[2])


def test_theta_below_one_and_reference_tables():
    """The tensor-core expansions assume every frequency theta_p <= 1 and take
    their coefficients from a scalar base: theta < 1 under "auto" runs the
    exact kernels (and "tensor" refuses it); the reference's 11-argument
    backward, which passes only the thetas table, has the table's base
    recovered (tensor path, results of that base); a table of no base raises
    under "tensor".  All against the oracle."""
    from CoROPE import _lib
    S, D = 300, 64
    sm = 1 / math.sqrt(D)
    (q, k, v, do), cpu = inputs(1, 2, S, D, 41, torch.bfloat16)
    with pytest.raises(NotImplementedError):
        co_rope_forward(q, k, v, sm, theta=0.5, algo="tensor")
    saved, o = co_rope_forward(q, k, v, sm, theta=0.5)
    dq, dk, dv = co_rope_backward(saved, do, sm, 0.5)
    torch.cuda.synchronize()
    assert _lib.take_device_error() == 0
    ref = O.forward_dense(*cpu[:3], sm, 0.5)
    assert maxabs(o, ref["o"]) < O_MAXABS
    for name, mine, r in zip(("dq", "dk", "dv"), (dq, dk, dv),
                             O.backward_dense(*cpu, sm, 0.5)):
        assert maxabs(mine, r) < G_MAXABS, name

    # reference call form: repeat-interleaved [H, D] table of base 500, theta
    # left at its default 1e4
    saved, o = co_rope_forward(q, k, v, sm, theta=500.0)
    tab = 1.0 / (500.0 ** (torch.arange(0, D, 2, device=DEV).float() / D))
    thetas = tab.repeat_interleave(2).expand(2, D).contiguous()
    args = (*saved, do, thetas, True, sm)
    dq, dk, dv, dth = co_rope_backward(*args, algo="tensor")
    torch.cuda.synchronize()
    assert _lib.take_device_error() == 0 and dth is None
    for name, mine, r in zip(("dq", "dk", "dv"), (dq, dk, dv),
                             O.backward_dense(*cpu, sm, 500.0)):
        assert maxabs(mine, r) < G_MAXABS, name
        assert rel_l2(mine, r) < REL_L2, name
    bent = thetas.clone()
    bent[:, 10:12] *= 1.5
    with pytest.raises(ValueError):
        co_rope_backward(*saved, do, bent, True, sm, algo="tensor")
    dq2, _, _, _ = co_rope_backward(*saved, do, bent, True, sm)
    torch.cuda.synchronize()
    assert torch.isfinite(dq2).all()


@pytest.mark.parametrize("D,hkv,theta,bias", [(128, None, 1e4, False), (64, None, 5e5, True),
                                              (128, 1, 5e5, False), (128, 2, 1e4, True)])
def test_forward_panels_equal_in_kernel_builders(D, hkv, theta, bias):
    """The tensor-core forward with its scaled-key panels (written once per
    call, loaded by TMA; per-key-offset expansions) and without them (built in
    every CTA; one expansion per window) agree: A bit for bit (the same gate
    arithmetic), O, M, L within the expansions' truncation error."""
    from CoROPE import _lib
    B, H, S = 2, 4, 700
    (q, k, v, _), _ = inputs(B, H, S, D, 91, torch.bfloat16, hkv=hkv)
    bias_t = (torch.randn(S, S, generator=torch.Generator().manual_seed(9)) * 0.3).to(DEV) if bias else None
    outs = []
    for ws in (True, False):
        o = torch.empty_like(q)
        m, l, a = (torch.empty(B, H, S, device=DEV) for _ in range(3))
        _lib.fwd(q, k, v, o, m, l, a, None, 1 / math.sqrt(D), theta, bias=bias_t, algo="tensor",
                 mqa=True, workspace=ws)
        outs.append((o, m, l, a))
    torch.cuda.synchronize()
    assert _lib.take_device_error() == 0
    (o1, m1, l1, a1), (o2, m2, l2, a2) = outs
    assert torch.equal(a1, a2)
    assert maxabs(o1, o2) < 2e-2  # bf16 outputs: one ulp at |O| ~ 2 is 1.6e-2
    assert maxabs(m1, m2) < 2e-2
    assert ((l1 - l2).abs() / l2.abs()).max().item() < 2e-2


@pytest.mark.parametrize("D", [64, 128])
def test_backward_panels_equal_in_kernel_builders(D):
    """The dQ kernel fed by the scaled-key panels and the one building its
    operands in every CTA (both per-key-offset expansions, the same
    coefficient table) give bit-identical dq, within tolerance of the
    definition's gradient."""
    from CoROPE import _lib
    B, H, S = 2, 4, 640
    (q, k, v, do), cpu = inputs(B, H, S, D, 93, torch.bfloat16)
    sm = 1 / math.sqrt(D)
    saved, o = co_rope_forward(q, k, v, sm, theta=5e5, algo="tensor")
    p = _lib.BwdParams()
    p.theta, p.sm_scale = 5e5, sm
    p.batch, p.heads, p.kv_heads, p.seq_len, p.head_dim = B, H, H, S, D
    p.dtype, p.algo = _lib._dtype_code(q), _lib.algo_code("tensor")
    lib = _lib.load_library()
    lo, panels = (lib.corope_bwd_min_workspace_bytes(ctypes.byref(p)),
                  lib.corope_bwd_panel_bytes(ctypes.byref(p)))
    res = []
    for ws in (lo, lo + panels):
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        _lib.bwd(*saved[:4], do, *saved[4:], dq, dk, dv, sm, 5e5, algo="tensor", workspace=ws)
        res.append(dq)
    torch.cuda.synchronize()
    assert _lib.take_device_error() == 0
    assert torch.equal(res[0], res[1])
    rq, _, _ = O.backward_dense(*[t.double() for t in cpu], sm, 5e5)
    assert maxabs(res[0], rq) < G_MAXABS and rel_l2(res[0], rq) < REL_L2


def test_forward_backward_capture_in_cuda_graph():
    """The public forward and backward make no host synchronisation and
    allocate only through torch, so a training step can be captured in a CUDA
    graph and replayed: the replay reproduces the eager outputs (O and dq bit
    for bit; dk, dv up to the order of the fp32 atomics)."""
    B, H, S, D = 2, 4, 512, 128
    (q, k, v, do), _ = inputs(B, H, S, D, 101, torch.bfloat16)
    sm = 1 / math.sqrt(D)

    def step():
        saved, o = co_rope_forward(q, k, v, sm, theta=1e4)
        dq, dk, dv = co_rope_backward(saved, do, sm, 1e4)
        return o, dq, dk, dv

    eager = step()
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()  # warm the allocator and the kernel attributes on the side stream
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        captured = step()
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    from CoROPE import _lib
    assert _lib.take_device_error() == 0
    assert torch.equal(captured[0], eager[0]) and torch.equal(captured[1], eager[1])
    for x, y in zip(captured[2:], eager[2:]):
        assert rel_l2(x, y) < 1e-3
