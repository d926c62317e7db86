"""The CPU oracle against the reference's own outputs (golden fixtures)."""
import math

import pytest
import torch

from oracle import corope_oracle as O
from golden_io import load, MHA_CASES


@pytest.mark.parametrize("name", MHA_CASES)
def test_oracle_forward_and_grads_match_reference(name):
    f = load(name)
    r = O.forward_dense(f["q"], f["k"], f["v"], f["sm_scale"], f["theta"])
    assert (r["o"] - f["o"]).abs().max() < 2e-6
    dq, dk, dv = O.backward_dense(f["q"], f["k"], f["v"], f["do"], f["sm_scale"], f["theta"])
    for mine, ref in ((dq, f["dq"]), (dk, f["dk"]), (dv, f["dv"])):
        tol = 2e-5 * max(1.0, ref.abs().max().item())
        assert (mine - ref).abs().max() < tol


@pytest.mark.parametrize("name", ["ref_b1h2s40d8.npz", "ref_b2h2s64d16_t500k.npz"])
def test_oracle_state_matches_reference_triton_kernel(name):
    """M, L, A as stored by co_rope_fwd_kernel (CoROPE/forward.py:110-120)."""
    f = load(name)
    r = O.forward_dense(f["q"], f["k"], f["v"], f["sm_scale"], f["theta"])
    assert (r["o"] - f["tri_o"]).abs().max() < 2e-6
    assert (r["m"] - f["tri_m"]).abs().max() < 1e-5
    assert ((r["l"] - f["tri_l"]).abs() / f["tri_l"]).max() < 1e-5
    assert (r["a"] - f["tri_a"]).abs().max() < 1e-5


def test_oracle_mqa_with_bias_matches_reference_triton_kernel():
    f = load("mqa_b1h4s48d16.npz")
    r = O.forward_dense(f["q"], f["k"], f["v"], f["sm_scale"], f["theta"], bias=f["bias"])
    for key in "omla":
        ref = f["tri_" + key]
        tol = 2e-5 * max(1.0, ref.abs().max().item())
        assert (r[key] - ref).abs().max() < tol, key


def test_loop_form_equals_dense_form():
    f = load("ref_b1h2s40d8.npz")
    o_loop, _ = O.forward_reference_loop(f["q"], f["k"], f["v"], f["sm_scale"], f["theta"])
    assert (o_loop - f["o"]).abs().max() < 2e-6


def test_closed_form_backward_equals_autograd_fp64():
    g = torch.Generator().manual_seed(1)
    q = torch.randn(1, 4, 24, 8, generator=g, dtype=torch.float64)
    k = torch.randn(1, 2, 24, 8, generator=g, dtype=torch.float64)
    v = torch.randn(1, 2, 24, 8, generator=g, dtype=torch.float64)
    do = torch.randn(1, 4, 24, 8, generator=g, dtype=torch.float64)
    bias = torch.randn(24, 24, generator=g, dtype=torch.float64) * 0.1
    _, a1, a2, a3 = O.autograd_reference(q, k, v, do, 0.3, 100.0, bias)
    b1, b2, b3 = O.backward_dense(q, k, v, do, 0.3, 100.0, bias)
    for x, y in ((a1, b1), (a2, b2), (a3, b3)):
        assert (x - y).abs().max() < 1e-12


def test_forward_rows_equals_dense():
    f = load("ref_b2h2s64d16_t500k.npz")
    r = O.forward_dense(f["q"], f["k"], f["v"], f["sm_scale"], f["theta"])
    rows = torch.tensor([0, 1, 17, 63])
    o, m, l, a = O.forward_rows(f["q"][1, 0], f["k"][1, 0], f["v"][1, 0], rows, f["sm_scale"],
                                f["theta"])
    assert (o - r["o"][1, 0, rows]).abs().max() < 1e-6
    assert (m - r["m"][1, 0, rows]).abs().max() < 1e-6
    assert (a - r["a"][1, 0, rows]).abs().max() < 1e-6


def test_backward_rows_equals_dense_fp64():
    """Per-row backward (long sequences): dq of the sampled rows, and dk, dv of
    the keys whose every contributing row is sampled, equal backward_dense."""
    g = torch.Generator().manual_seed(5)
    S, D = 40, 8
    q, k, v, do = (torch.randn(1, 1, S, D, generator=g, dtype=torch.float64) for _ in range(4))
    rq, rk, rv = O.backward_dense(q, k, v, do, 0.35, 500.0)
    rows = torch.arange(S - 6, S)
    dq, dk, dv = O.backward_rows(q[0, 0], k[0, 0], v[0, 0], do[0, 0], rows, 0.35, 500.0)
    assert (dq - rq[0, 0, rows]).abs().max() < 1e-12
    assert (dk[S - 6:] - rk[0, 0, S - 6:]).abs().max() < 1e-12
    assert (dv[S - 6:] - rv[0, 0, S - 6:]).abs().max() < 1e-12
    every = torch.arange(S)
    dq, dk, dv = O.backward_rows(q[0, 0], k[0, 0], v[0, 0], do[0, 0], every, 0.35, 500.0)
    assert (dk - rk[0, 0]).abs().max() < 1e-12 and (dv - rv[0, 0]).abs().max() < 1e-12


def test_planted_error_is_detected():
    """A mistake planted in the oracle's inputs (one flipped gate sign) must
    move the output well past the tolerances used by the GPU tests."""
    f = load("ref_b1h2s40d8.npz")
    k2 = f["k"].clone()
    k2[0, 0, 5] *= -1
    r = O.forward_dense(f["q"], k2, f["v"], f["sm_scale"], f["theta"])
    assert (r["o"] - f["o"]).abs().max() > 2e-2


def test_flop_convention():
    assert O.flops(1, 1, 4, 8, "fwd") == 4 * 8 * 10
    assert O.flops(4, 32, 4096, 128, "fwd+bwd") == pytest.approx(14 * 128 * 4 * 32 * 4096 * 4097 / 2)
