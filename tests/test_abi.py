"""The C-ABI library loads, exports what include/corope.h declares, and its
argument checks answer before any device work (no GPU needed)."""
import ctypes
import os
import re

import pytest

from CoROPE import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "corope.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(corope_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load_library()
    names = declared_functions()
    assert {"corope_fwd", "corope_mqa_fwd", "corope_bwd", "corope_bwd_workspace_bytes",
            "corope_last_error", "corope_abi_version"} <= set(names)
    for n in names:
        assert hasattr(lib, n), n


def test_abi_version_and_struct_layout():
    lib = _lib.load_library()
    assert lib.corope_abi_version() == 4
    assert lib.corope_params_size(0) == ctypes.sizeof(_lib.FwdParams)
    assert lib.corope_params_size(1) == ctypes.sizeof(_lib.BwdParams)


def _fwd_params(**kw):
    p = _lib.FwdParams()
    fake = 1 << 20
    p.q = p.k = p.v = p.o = fake
    S, D = kw.get("S", 64), kw.get("D", 64)
    st = _lib._I64x3(4 * S * D, S * D, D)
    p.q_stride = p.k_stride = p.v_stride = p.o_stride = st
    p.batch, p.heads, p.kv_heads = 1, kw.get("H", 4), kw.get("Hkv", 4)
    p.seq_len, p.head_dim = S, D
    p.sm_scale, p.theta = 0.125, 10000.0
    p.causal, p.dtype, p.algo = kw.get("causal", 1), kw.get("dtype", 2), kw.get("algo", 0)
    return p


@pytest.mark.parametrize("kw,code,fn", [
    (dict(Hkv=3), _lib.ERR_INVALID, "corope_mqa_fwd"),
    (dict(Hkv=1), _lib.ERR_INVALID, "corope_fwd"),
    (dict(causal=0), _lib.ERR_UNSUPPORTED, "corope_fwd"),
    (dict(D=256), _lib.ERR_UNSUPPORTED, "corope_fwd"),
    (dict(D=6), _lib.ERR_UNSUPPORTED, "corope_fwd"),
    (dict(dtype=7), _lib.ERR_INVALID, "corope_fwd"),
])
def test_forward_argument_checks(kw, code, fn):
    lib = _lib.load_library()
    p = _fwd_params(**kw)
    rc = getattr(lib, fn)(ctypes.byref(p), None)
    assert rc == code
    assert lib.corope_last_error()


def test_null_params_and_bad_stride():
    lib = _lib.load_library()
    assert lib.corope_fwd(None, None) == _lib.ERR_INVALID
    p = _fwd_params()
    p.q_stride = _lib._I64x3(4 * 64 * 64, 64 * 64, 63)
    assert lib.corope_fwd(ctypes.byref(p), None) == _lib.ERR_INVALID


def test_backward_workspace_checks():
    lib = _lib.load_library()
    p = _lib.BwdParams()
    fake = 1 << 20
    for n in ("q", "k", "v", "o", "dout", "m", "l", "a", "dq", "dk", "dv"):
        setattr(p, n, fake)
    st = _lib._I64x3(2 * 128 * 64, 128 * 64, 64)
    for n in ("q_stride", "k_stride", "v_stride", "o_stride", "do_stride", "dq_stride",
              "dk_stride", "dv_stride"):
        setattr(p, n, st)
    p.batch, p.heads, p.kv_heads, p.seq_len, p.head_dim = 1, 2, 2, 128, 64
    p.sm_scale, p.theta, p.causal, p.dtype = 0.125, 1e4, 1, 2
    need = lib.corope_bwd_min_workspace_bytes(ctypes.byref(p))
    full = lib.corope_bwd_workspace_bytes(ctypes.byref(p))
    # delta + lse rows, fp32 dk/dv accumulators; the full size adds the
    # tensor-core hand-off region (bf16, head_dim 64)
    assert need >= 2 * 2 * 128 * 4 + 2 * 2 * 128 * 64 * 4
    assert full > need
    assert lib.corope_bwd(ctypes.byref(p), None) == _lib.ERR_WORKSPACE
    p.workspace, p.workspace_bytes = fake, need - 1
    assert lib.corope_bwd(ctypes.byref(p), None) == _lib.ERR_WORKSPACE


def _bwd_params(**kw):
    p = _lib.BwdParams()
    fake = 1 << 20
    for n in ("q", "k", "v", "o", "dout", "m", "l", "a", "dq", "dk", "dv"):
        setattr(p, n, fake)
    S, D = 128, kw.get("D", 64)
    st = _lib._I64x3(2 * S * D, S * D, D)
    for n in ("q_stride", "k_stride", "v_stride", "o_stride", "do_stride", "dq_stride",
              "dk_stride", "dv_stride"):
        setattr(p, n, st)
    p.batch, p.heads, p.kv_heads, p.seq_len, p.head_dim = 1, 2, kw.get("Hkv", 2), S, D
    p.sm_scale, p.theta = 0.125, 1e4
    p.causal, p.dtype, p.algo = kw.get("causal", 1), kw.get("dtype", 2), kw.get("algo", 0)
    for n in kw.get("null", ()):
        setattr(p, n, None)
    return p


@pytest.mark.parametrize("fn", ["corope_bwd", "corope_bwd_noalloc"])
@pytest.mark.parametrize("kw,code", [
    (dict(dtype=7), _lib.ERR_INVALID),
    (dict(causal=0), _lib.ERR_UNSUPPORTED),
    (dict(algo=9), _lib.ERR_INVALID),
    (dict(D=256), _lib.ERR_UNSUPPORTED),
    (dict(Hkv=3), _lib.ERR_INVALID),
    (dict(null=("q",)), _lib.ERR_INVALID),
    (dict(null=("dk",)), _lib.ERR_INVALID),
    (dict(null=("m", "l", "a")), _lib.ERR_INVALID),
])
def test_backward_argument_checks(fn, kw, code):
    """corope_bwd and corope_bwd_noalloc refuse bad arguments with the same
    status, before any device work (so without a GPU too)."""
    lib = _lib.load_library()
    p = _bwd_params(**kw)
    assert getattr(lib, fn)(ctypes.byref(p), None) == code
    assert lib.corope_last_error()
    assert getattr(lib, fn)(None, None) == _lib.ERR_INVALID


@pytest.mark.parametrize("kw,code", [
    (dict(dtype=7), _lib.ERR_INVALID),
    (dict(dtype=0), _lib.ERR_UNSUPPORTED),
    (dict(D=32), _lib.ERR_UNSUPPORTED),
    (dict(causal=2), _lib.ERR_INVALID),
    (dict(Hkv=3), _lib.ERR_INVALID),
])
def test_plain_attention_argument_checks(kw, code):
    """corope_flash_fwd refuses bad arguments before any device work."""
    lib = _lib.load_library()
    p = _fwd_params(**kw)
    assert lib.corope_flash_fwd(ctypes.byref(p), None) == code
    assert lib.corope_last_error()
    assert lib.corope_flash_fwd(None, None) == _lib.ERR_INVALID


def test_chunk_argument_checks_without_gpu():
    """corope_fwd_chunk / corope_bwd_chunk refuse a NULL chunk, an offset off
    the 128-row tiles, a key range shorter than the chunk and missing fp32
    accumulators before touching the device."""
    lib = _lib.load_library()
    p = _fwd_params(S=128)
    c = _lib.ChunkParams()
    assert lib.corope_fwd_chunk(ctypes.byref(p), None, None) == _lib.ERR_INVALID
    c.q_row0, c.kv_len = 100, 1024
    assert lib.corope_fwd_chunk(ctypes.byref(p), ctypes.byref(c), None) == _lib.ERR_INVALID
    c.q_row0, c.kv_len = 256, 300
    assert lib.corope_fwd_chunk(ctypes.byref(p), ctypes.byref(c), None) == _lib.ERR_INVALID
    assert b"kv_len" in lib.corope_last_error()
    b = _lib.BwdParams()
    fake = 1 << 20
    b.q = b.k = b.v = b.o = b.dout = b.dq = fake
    b.m = b.l = b.a = fake
    st = _lib._I64x3(4 * 128 * 64, 128 * 64, 64)
    b.q_stride = b.k_stride = b.v_stride = b.o_stride = b.do_stride = b.dq_stride = st
    b.batch, b.heads, b.kv_heads, b.seq_len, b.head_dim = 1, 4, 4, 128, 64
    b.sm_scale, b.theta, b.causal, b.dtype = 0.125, 1e4, 1, 2
    c.q_row0, c.kv_len = 256, 512
    assert lib.corope_bwd_chunk(ctypes.byref(b), ctypes.byref(c), None) == _lib.ERR_INVALID
    assert b"dk_accum" in lib.corope_last_error()
    # the chunk workspace holds delta / lse rows and the dQ kernel's expansion
    # coefficients (16 offsets x 16 terms x 64 pairs, complex fp32), the
    # scaled-key panels of all kv_len keys and the chunk's hand-off
    lo = lib.corope_bwd_chunk_min_workspace_bytes(ctypes.byref(b), ctypes.byref(c))
    hi = lib.corope_bwd_chunk_workspace_bytes(ctypes.byref(b), ctypes.byref(c))
    keys = _lib.BwdParams.from_buffer_copy(b)
    keys.seq_len = 512
    panels = lib.corope_bwd_panel_bytes(ctypes.byref(keys))
    assert lo == 2 * 4 * 128 * 4 + 16 * 16 * 64 * 8 and panels > 0
    assert hi - lo - panels == 4 * ((256 + 127) // 16 + 1) * 4096


def test_deterministic_flag_without_gpu():
    """COROPE_BWD_DETERMINISTIC (OR'd into algo): 64-bit dk / dv accumulators
    in the minimum workspace (twice the fp32 size), any base algo, refused
    for query chunks before any device work; theta < 1 (exact kernels only)
    asks for no tensor-core workspace."""
    lib = _lib.load_library()
    hdr = open(HEADER).read()
    assert "#define COROPE_BWD_DETERMINISTIC 0x100" in hdr
    assert _lib.BWD_DETERMINISTIC == 0x100
    kv = 1 * 2 * 128 * 64
    for algo in (_lib.ALGO_AUTO, _lib.ALGO_EXACT, _lib.ALGO_TENSOR):
        p = _bwd_params(algo=algo)
        d = _bwd_params(algo=algo | _lib.BWD_DETERMINISTIC)
        lo, lo_det = (lib.corope_bwd_min_workspace_bytes(ctypes.byref(x)) for x in (p, d))
        assert lo_det - lo == 2 * kv * 4
        hi, hi_det = (lib.corope_bwd_workspace_bytes(ctypes.byref(x)) for x in (p, d))
        assert hi_det - hi == 2 * kv * 4
        # the workspace check still answers first (no device touched)
        assert lib.corope_bwd(ctypes.byref(d), None) == _lib.ERR_WORKSPACE
    bad = _bwd_params(algo=9 | _lib.BWD_DETERMINISTIC)
    assert lib.corope_bwd(ctypes.byref(bad), None) == _lib.ERR_INVALID
    c = _lib.ChunkParams()
    c.q_row0, c.kv_len = 0, 128
    d = _bwd_params(algo=_lib.BWD_DETERMINISTIC)
    acc = _lib.ChunkParams.from_buffer_copy(c)
    acc.dk_accum = acc.dv_accum = 1 << 20
    assert lib.corope_bwd_chunk(ctypes.byref(d), ctypes.byref(acc), None) == _lib.ERR_UNSUPPORTED
    assert b"DETERMINISTIC" in lib.corope_last_error()
    # theta < 1: no coefficient table, panels or hand-off region
    p = _bwd_params()
    p.theta = 0.5
    assert lib.corope_bwd_panel_bytes(ctypes.byref(p)) == 0
    assert lib.corope_bwd_min_workspace_bytes(ctypes.byref(p)) == \
        lib.corope_bwd_workspace_bytes(ctypes.byref(p)) == 2 * 2 * 128 * 4 + 2 * kv * 4


def test_size_queries_accept_null():
    """Every size query answers 0 for a NULL params / chunk instead of
    dereferencing it."""
    lib = _lib.load_library()
    assert lib.corope_fwd_workspace_bytes(None) == 0
    assert lib.corope_fwd_chunk_workspace_bytes(None, None) == 0
    assert lib.corope_bwd_workspace_bytes(None) == 0
    assert lib.corope_bwd_min_workspace_bytes(None) == 0
    assert lib.corope_bwd_panel_bytes(None) == 0
    assert lib.corope_bwd_chunk_workspace_bytes(None, None) == 0
    assert lib.corope_bwd_chunk_min_workspace_bytes(None, None) == 0
    p = _fwd_params()
    assert lib.corope_fwd_chunk_workspace_bytes(ctypes.byref(p), None) == 0
