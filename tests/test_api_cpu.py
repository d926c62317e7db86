"""Host-side behaviour of the drop-in Python package (no GPU needed)."""
import math

import pytest
import torch

import CoROPE
import importlib
from CoROPE.co_rope_backward import co_rope_backward
from CoROPE.co_rope_mqa_forward import co_rope_mqa_forward
from CoROPE.forward import co_rope_forward


def test_module_layout_matches_reference_imports():
    # the imports used by the reference's own callers
    from CoROPE.co_rope_forward import co_rope_forward as f2  # co_rope_attn.py:2
    from CoROPE.co_rope_attn import CoRoPEAttention, CoRoPEAttentionFunction  # test.py:2
    assert f2 is co_rope_forward
    assert CoROPE.CoRoPEAttention is CoRoPEAttention


def test_causal_false_refused():
    q = torch.zeros(1, 1, 4, 4)
    with pytest.raises(NotImplementedError):
        co_rope_forward(q, q, q, 0.5, causal=False)
    with pytest.raises(NotImplementedError):
        co_rope_mqa_forward(q, q, q, 0.5, causal=False)


def test_cpu_tensors_refused_like_reference():
    q = torch.zeros(1, 1, 4, 4)
    with pytest.raises(AssertionError, match="CUDA"):
        co_rope_forward(q, q, q, 0.5)


def test_mqa_shape_error_like_reference():
    q = torch.zeros(1, 2, 4, 4)
    with pytest.raises(ValueError):
        co_rope_mqa_forward(q, q, q, 0.5)


def test_backward_accepts_both_conventions(monkeypatch):
    bwd_mod = importlib.import_module("CoROPE.co_rope_backward")
    seen = []

    def fake_run(q, k, v, o, m, l, a, do, sm_scale, theta, thetas, bias, algo, det=False):
        seen.append((sm_scale, theta, None if thetas is None else thetas.tolist()))
        return "dq", "dk", "dv"

    monkeypatch.setattr(bwd_mod, "_run", fake_run)
    t = torch.zeros(1, 1, 4, 4)
    r = co_rope_backward((t,) * 7, t, 0.3, 500.0)
    assert r == ("dq", "dk", "dv") and seen[-1] == (0.3, 500.0, None)
    D = 4
    th = 1.0 / (1e4 ** (torch.arange(0, D, 2).float() / D))
    thetas = th.repeat_interleave(2).unsqueeze(0).repeat(3, 1)
    r = co_rope_backward(t, t, t, t, t, t, t, t, thetas, True, 0.25)
    assert r == ("dq", "dk", "dv", None)
    assert seen[-1][0] == 0.25 and seen[-1][2] == pytest.approx(th.tolist())
    with pytest.raises(NotImplementedError):
        co_rope_backward(t, t, t, t, t, t, t, t, thetas, False, 0.25)


def test_backward_deterministic_follows_torch_setting(monkeypatch):
    """deterministic=None takes torch.are_deterministic_algorithms_enabled();
    an explicit value wins, in both calling conventions."""
    bwd_mod = importlib.import_module("CoROPE.co_rope_backward")
    seen = []

    def fake_run(q, k, v, o, m, l, a, do, sm_scale, theta, thetas, bias, algo, det=False):
        seen.append(det)
        return "dq", "dk", "dv"

    monkeypatch.setattr(bwd_mod, "_run", fake_run)
    t = torch.zeros(1, 1, 4, 4)
    was = torch.are_deterministic_algorithms_enabled()
    try:
        torch.use_deterministic_algorithms(False)
        co_rope_backward((t,) * 7, t, 0.3, 500.0)
        co_rope_backward((t,) * 7, t, 0.3, 500.0, deterministic=True)
        torch.use_deterministic_algorithms(True)
        co_rope_backward((t,) * 7, t, 0.3, 500.0)
        co_rope_backward(t, t, t, t, t, t, t, t, None, True, 0.25)
        co_rope_backward((t,) * 7, t, 0.3, 500.0, deterministic=False)
    finally:
        torch.use_deterministic_algorithms(was)
    assert seen == [False, True, True, True, False]


@pytest.mark.parametrize("D", [64, 128])
def test_backward_table_base_reaches_tensor_kernels(monkeypatch, D):
    """The reference's autograd backward passes only the thetas table
    (co_rope_attn.py:35-47): its base is recovered for the tensor-core
    kernels; a table of no base runs exact under "auto", raises under
    "tensor"."""
    bwd_mod = importlib.import_module("CoROPE.co_rope_backward")
    seen = []

    def fake_run(q, k, v, o, m, l, a, do, sm_scale, theta, thetas, bias, algo, det=False):
        seen.append((theta, algo))
        return "dq", "dk", "dv"

    monkeypatch.setattr(bwd_mod, "_run", fake_run)
    t = torch.zeros(1, 1, 4, D)
    for base in (10000.0, 500000.0, 1e6, 123.5):
        th = 1.0 / (base ** (torch.arange(0, D, 2).float() / D))
        thetas = th.repeat_interleave(2).unsqueeze(0).repeat(2, 1)
        co_rope_backward(t, t, t, t, t, t, t, t, thetas, True, 0.25)
        assert seen[-1][1] == "auto"
        assert seen[-1][0] == pytest.approx(base, rel=1e-6)
    assert seen[-3][0] == 500000.0  # integer bases come back exact
    junk = torch.rand(D)
    co_rope_backward(t, t, t, t, t, t, t, t, junk, True, 0.25)
    assert seen[-1] == (10000.0, "exact")
    with pytest.raises(ValueError):
        co_rope_backward(t, t, t, t, t, t, t, t, junk, True, 0.25, algo="tensor")
    co_rope_backward(t, t, t, t, t, t, t, t, junk, True, 0.25, algo="exact")
    assert seen[-1] == (10000.0, "exact")


def test_theta_table_matches_reference_expression():
    from CoROPE import _lib
    D, theta = 128, 10000.0
    ref = 1.0 / (theta ** (torch.arange(0, D, 2).float() / D))
    assert torch.equal(_lib.theta_table(D, theta, "cpu"), ref)
    assert _lib.default_scale(64, None) == pytest.approx(1 / math.sqrt(64))


def test_auto_workspace_fits_whole_slices():
    """The "auto" backward workspace: the full hand-off region when it fits,
    else the minimum plus whole (b, h) slices (long sequences), else the
    minimum."""
    from CoROPE._lib import fit_workspace
    least, per, units = 1000, 256 * 40, 8
    full = least + per * units
    assert fit_workspace(full, least, units, budget=full) == full
    assert fit_workspace(full, least, units, budget=10 ** 12) == full
    assert fit_workspace(full, least, units, budget=least + 3 * per + 5) == least + 3 * per
    assert fit_workspace(full, least, units, budget=least + per - 1) == least
    assert fit_workspace(full, least, units, budget=0) == least
    # no hand-off region at all (exact path, or head dims without one)
    assert fit_workspace(least, least, units, budget=0) == least
    # with scaled-key panels: [least][panels][slices]
    panels = 5000
    full = least + panels + per * units
    assert fit_workspace(full, least, units, full, panels) == full
    assert fit_workspace(full, least, units, least + panels + 2 * per + 7, panels) == \
        least + panels + 2 * per
    assert fit_workspace(full, least, units, least + panels + 10, panels) == least + panels
    assert fit_workspace(full, least, units, least + panels - 1, panels) == least


def test_auto_workspace_policy_without_gpu():
    """The "auto" backward workspace: the whole hand-off region at the bench
    shape (B=4, H=32, S=4096, D=128 bf16: under 4 GiB), and for one GPU's
    share of the long-context shape (B=1, H=32, S=32768) the minimum, the
    panels and the 4 whole hand-off slices that make 1024-CTA launches."""
    import ctypes
    from CoROPE import _lib
    lib = _lib.load_library()

    def params(B, H, S, D, theta):
        p = _lib.BwdParams()
        p.batch, p.heads, p.kv_heads, p.seq_len, p.head_dim = B, H, H, S, D
        p.dtype, p.algo, p.theta, p.sm_scale = _lib.DTYPE_BF16, _lib.ALGO_AUTO, theta, D ** -0.5
        return p

    p = params(4, 32, 4096, 128, 1e4)
    full = lib.corope_bwd_workspace_bytes(ctypes.byref(p))
    assert _lib.auto_workspace_bytes(lib, p, "cuda:0") == full <= _lib.AUTO_WORKSPACE_BUDGET
    p = params(1, 32, 32768, 128, 5e5)
    full = lib.corope_bwd_workspace_bytes(ctypes.byref(p))
    least = lib.corope_bwd_min_workspace_bytes(ctypes.byref(p))
    panels = lib.corope_bwd_panel_bytes(ctypes.byref(p))
    per = (full - least - panels) // 32
    assert _lib.floor_slices(32, 32768) == 4
    assert _lib.auto_workspace_bytes(lib, p, "cuda:0") == least + panels + 4 * per
