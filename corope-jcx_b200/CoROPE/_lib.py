"""ctypes binding of libcorope_b200.so (the C ABI declared in include/corope.h).

The shared library is looked up next to this file (built in-tree by
``corope-jcx_b200/build.py``).  There is no fallback: if the library or a
CUDA device is missing, every call raises.
"""
from __future__ import annotations

import ctypes
import math
import os
import threading
from typing import Optional

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcorope_b200.so")

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
ALGO_AUTO, ALGO_EXACT, ALGO_TENSOR = 0, 1, 2
_ALGOS = {"auto": ALGO_AUTO, "exact": ALGO_EXACT, "tensor": ALGO_TENSOR}
# corope.h COROPE_BWD_DETERMINISTIC, OR'd into the backward's algo
BWD_DETERMINISTIC = 0x100

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_WORKSPACE, ERR_DEVICE = range(6)

_I64x3 = ctypes.c_int64 * 3


class FwdParams(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("m", ctypes.c_void_p), ("l", ctypes.c_void_p), ("a", ctypes.c_void_p),
        ("lse", ctypes.c_void_p),
        ("thetas", ctypes.c_void_p),
        ("bias", ctypes.c_void_p), ("bias_row_stride", ctypes.c_int64),
        ("q_stride", _I64x3), ("k_stride", _I64x3), ("v_stride", _I64x3),
        ("o_stride", _I64x3),
        ("batch", ctypes.c_int32), ("heads", ctypes.c_int32), ("kv_heads", ctypes.c_int32),
        ("seq_len", ctypes.c_int32), ("head_dim", ctypes.c_int32),
        ("sm_scale", ctypes.c_float), ("theta", ctypes.c_float),
        ("causal", ctypes.c_int32), ("dtype", ctypes.c_int32), ("algo", ctypes.c_int32),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
    ]


class BwdParams(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p), ("dout", ctypes.c_void_p),
        ("m", ctypes.c_void_p), ("l", ctypes.c_void_p), ("a", ctypes.c_void_p),
        ("thetas", ctypes.c_void_p),
        ("bias", ctypes.c_void_p), ("bias_row_stride", ctypes.c_int64),
        ("dq", ctypes.c_void_p), ("dk", ctypes.c_void_p), ("dv", ctypes.c_void_p),
        ("q_stride", _I64x3), ("k_stride", _I64x3), ("v_stride", _I64x3),
        ("o_stride", _I64x3), ("do_stride", _I64x3),
        ("dq_stride", _I64x3), ("dk_stride", _I64x3), ("dv_stride", _I64x3),
        ("batch", ctypes.c_int32), ("heads", ctypes.c_int32), ("kv_heads", ctypes.c_int32),
        ("seq_len", ctypes.c_int32), ("head_dim", ctypes.c_int32),
        ("sm_scale", ctypes.c_float), ("theta", ctypes.c_float),
        ("causal", ctypes.c_int32), ("dtype", ctypes.c_int32), ("algo", ctypes.c_int32),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
    ]


class ChunkParams(ctypes.Structure):
    """corope_chunk_t: a query chunk at sequence position q_row0 against
    kv_len key rows (sequence-sharded callers)."""
    _fields_ = [
        ("q_row0", ctypes.c_int64), ("kv_len", ctypes.c_int32),
        ("accum_chunk_rows", ctypes.c_int32),
        ("dk_accum", ctypes.c_void_p), ("dv_accum", ctypes.c_void_p),
    ]


_lib = None
_lock = threading.Lock()


def load_library():
    """Load (once) and return the ctypes handle; raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"CoROPE CUDA library not found at {LIB_PATH}; build it with "
                    "`python corope-jcx_b200/build.py` (no CPU fallback exists)")
            lib = ctypes.CDLL(LIB_PATH)
            lib.corope_fwd.argtypes = [ctypes.POINTER(FwdParams), ctypes.c_void_p]
            lib.corope_fwd.restype = ctypes.c_int
            lib.corope_mqa_fwd.argtypes = [ctypes.POINTER(FwdParams), ctypes.c_void_p]
            lib.corope_mqa_fwd.restype = ctypes.c_int
            lib.corope_bwd.argtypes = [ctypes.POINTER(BwdParams), ctypes.c_void_p]
            lib.corope_bwd.restype = ctypes.c_int
            lib.corope_bwd_workspace_bytes.argtypes = [ctypes.POINTER(BwdParams)]
            lib.corope_bwd_workspace_bytes.restype = ctypes.c_size_t
            lib.corope_bwd_min_workspace_bytes.argtypes = [ctypes.POINTER(BwdParams)]
            lib.corope_bwd_min_workspace_bytes.restype = ctypes.c_size_t
            lib.corope_last_error.argtypes = []
            lib.corope_last_error.restype = ctypes.c_char_p
            lib.corope_bwd_noalloc.argtypes = [ctypes.POINTER(BwdParams), ctypes.c_void_p]
            lib.corope_bwd_noalloc.restype = ctypes.c_int
            lib.corope_bwd_noalloc_scratch_bytes.argtypes = []
            lib.corope_bwd_noalloc_scratch_bytes.restype = ctypes.c_size_t
            lib.corope_take_device_error.argtypes = []
            lib.corope_take_device_error.restype = ctypes.c_int
            lib.corope_params_size.argtypes = [ctypes.c_int]
            lib.corope_params_size.restype = ctypes.c_size_t
            lib.corope_abi_version.argtypes = []
            lib.corope_abi_version.restype = ctypes.c_int
            chunk_p = ctypes.POINTER(ChunkParams)
            lib.corope_fwd_workspace_bytes.argtypes = [ctypes.POINTER(FwdParams)]
            lib.corope_fwd_workspace_bytes.restype = ctypes.c_size_t
            lib.corope_fwd_chunk_workspace_bytes.argtypes = [ctypes.POINTER(FwdParams), chunk_p]
            lib.corope_fwd_chunk_workspace_bytes.restype = ctypes.c_size_t
            lib.corope_fwd_chunk.argtypes = [ctypes.POINTER(FwdParams), chunk_p, ctypes.c_void_p]
            lib.corope_fwd_chunk.restype = ctypes.c_int
            lib.corope_bwd_chunk.argtypes = [ctypes.POINTER(BwdParams), chunk_p, ctypes.c_void_p]
            lib.corope_bwd_chunk.restype = ctypes.c_int
            lib.corope_bwd_panel_bytes.argtypes = [ctypes.POINTER(BwdParams)]
            lib.corope_bwd_panel_bytes.restype = ctypes.c_size_t
            lib.corope_flash_fwd.argtypes = [ctypes.POINTER(FwdParams), ctypes.c_void_p]
            lib.corope_flash_fwd.restype = ctypes.c_int
            for name in ("corope_bwd_chunk_workspace_bytes", "corope_bwd_chunk_min_workspace_bytes"):
                getattr(lib, name).argtypes = [ctypes.POINTER(BwdParams), chunk_p]
                getattr(lib, name).restype = ctypes.c_size_t
            _lib = lib
    return _lib


def take_device_error() -> int:
    """Read and clear the tensor-core kernels' device error word (0 = none)."""
    return load_library().corope_take_device_error()


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return DTYPE_F32
    if t.dtype == torch.float16:
        return DTYPE_F16
    if t.dtype == torch.bfloat16:
        return DTYPE_BF16
    raise TypeError(f"CoRoPE kernels support float32/float16/bfloat16, got {t.dtype}")


def _rowmajor(t: torch.Tensor) -> torch.Tensor:
    """Last dim contiguous with even strides (pairs are loaded together)."""
    if t.stride(-1) != 1 or any(s % 2 for s in t.stride()[:3]):
        t = t.contiguous()
    return t


def _strides(t: torch.Tensor):
    return _I64x3(t.stride(0), t.stride(1), t.stride(2))


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _check(rc: int, what: str):
    if rc == OK:
        return
    msg = load_library().corope_last_error().decode(errors="replace")
    if rc == ERR_UNSUPPORTED:
        raise NotImplementedError(f"{what}: {msg}")
    if rc == ERR_INVALID:
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg} (status {rc})")


def algo_code(algo) -> int:
    if isinstance(algo, int):
        return algo
    try:
        return _ALGOS[algo]
    except KeyError:
        raise ValueError(f"algo must be one of {sorted(_ALGOS)}, got {algo!r}") from None


_theta_cache = {}


def theta_table(head_dim: int, theta: float, device) -> torch.Tensor:
    """[D/2] fp32 table ``1 / theta ** (arange(0, D, 2) / D)`` computed with the
    same torch expression as the reference (CoROPE/forward.py:130-132), on
    the device, cached per (D, theta, device)."""
    key = (head_dim, float(theta), str(device))
    t = _theta_cache.get(key)
    if t is None:
        t = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device).float() / head_dim))
        t = t.contiguous()
        _theta_cache[key] = t
    return t


def default_scale(head_dim: int, sm_scale) -> float:
    return 1.0 / math.sqrt(head_dim) if sm_scale is None else float(sm_scale)


def fwd(q, k, v, o, m, l, a, lse, sm_scale, theta, bias=None, algo="auto", thetas=None,
        mqa=False, q_row0=None, workspace=True):
    """Launch corope_fwd / corope_mqa_fwd on the current stream of q.  With
    ``q_row0`` (corope_fwd_chunk) q, o, m, l, a, lse are the query rows at
    sequence positions q_row0.. and k, v hold every key row from 0.
    ``workspace=False`` runs the tensor-core forward without its scaled-key
    panels (the kernel builds the operands itself; same results)."""
    lib = load_library()
    B, H, S, D = q.shape
    p = FwdParams()
    p.q, p.k, p.v, p.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    p.m, p.l, p.a, p.lse = _ptr(m), _ptr(l), _ptr(a), _ptr(lse)
    th = thetas if thetas is not None else theta_table(D, theta, q.device)
    p.thetas = th.data_ptr()
    if bias is not None:
        p.bias = bias.data_ptr()
        p.bias_row_stride = bias.stride(0)
    p.q_stride, p.k_stride, p.v_stride, p.o_stride = (_strides(q), _strides(k), _strides(v),
                                                      _strides(o))
    p.batch, p.heads, p.kv_heads, p.seq_len, p.head_dim = B, H, k.shape[1], S, D
    p.sm_scale, p.theta = float(sm_scale), float(theta)
    p.causal, p.dtype, p.algo = 1, _dtype_code(q), algo_code(algo)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    c = None
    if q_row0 is not None:
        c = ChunkParams()
        c.q_row0, c.kv_len = int(q_row0), k.shape[2]
    ws = None
    if workspace:
        nbytes = (lib.corope_fwd_workspace_bytes(ctypes.byref(p)) if c is None else
                  lib.corope_fwd_chunk_workspace_bytes(ctypes.byref(p), ctypes.byref(c)))
        if nbytes:
            ws, nbytes = _alloc_workspace(nbytes, 0, q.device)
            if nbytes:
                p.workspace, p.workspace_bytes = ws.data_ptr(), nbytes
    if c is not None:
        with torch.cuda.device(q.device):
            rc = lib.corope_fwd_chunk(ctypes.byref(p), ctypes.byref(c), ctypes.c_void_p(stream))
        _check(rc, "corope_fwd_chunk")
        return
    fn = lib.corope_mqa_fwd if mqa else lib.corope_fwd
    with torch.cuda.device(q.device):
        rc = fn(ctypes.byref(p), ctypes.c_void_p(stream))
    _check(rc, "corope_mqa_fwd" if mqa else "corope_fwd")


def flash_fwd(q, k, v, o, m, lse, sm_scale, causal):
    """Launch corope_flash_fwd (plain softmax attention on the tensor-core
    pipeline) on the current stream of q."""
    lib = load_library()
    B, H, S, D = q.shape
    p = FwdParams()
    p.q, p.k, p.v, p.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    p.m, p.lse = _ptr(m), _ptr(lse)
    p.q_stride, p.k_stride, p.v_stride, p.o_stride = (_strides(q), _strides(k), _strides(v),
                                                      _strides(o))
    p.batch, p.heads, p.kv_heads, p.seq_len, p.head_dim = B, H, k.shape[1], S, D
    p.sm_scale = float(sm_scale)
    p.causal, p.dtype = 1 if causal else 0, _dtype_code(q)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    with torch.cuda.device(q.device):
        rc = lib.corope_flash_fwd(ctypes.byref(p), ctypes.c_void_p(stream))
    _check(rc, "corope_flash_fwd")


# Workspace the "auto" backward takes at most, unless one slice group of the
# hand-off needs more (see auto_workspace_bytes).
AUTO_WORKSPACE_BUDGET = 4 << 30


def _alloc_workspace(nbytes, least, device):
    """torch-allocated workspace; if the allocator cannot give ``nbytes`` the
    call falls back to ``least`` (the kernels then skip the optional parts)."""
    try:
        return torch.empty(nbytes, dtype=torch.uint8, device=device), nbytes
    except torch.OutOfMemoryError:
        if nbytes <= least:
            raise
        return torch.empty(least, dtype=torch.uint8, device=device), least


def floor_slices(units, seq_len, ctas=1024):
    """(b, h) slices whose hand-off launches make at least ``ctas`` CTAs of 128
    query rows (about 7 waves of 148 SMs), or all units."""
    qtiles = (seq_len + 127) // 128
    return min(units, (ctas + qtiles - 1) // qtiles)


def auto_workspace_bytes(lib, p, device, chunk=None):
    """The workspace "auto" gives corope_bwd: the full size when it fits in
    AUTO_WORKSPACE_BUDGET (4 GiB), else the minimum plus the scaled-key
    panels plus as many whole (b, h) hand-off slices as fit there -- but never
    fewer than make launches of 1024 CTAs (long sequences: 4 slices of 1.1 GB
    at S=32768, 8.1 GB in all, within 3% of the whole 38 GB region's speed;
    below that the launch tails cost more, and without a hand-off the dK
    kernel recomputes the per-pair work).  The budget is fixed, not a share of
    free memory: asking the driver for free memory would cost a round trip on
    every backward, and a fixed request lets torch's cache serve it again."""
    if chunk is None:
        full = lib.corope_bwd_workspace_bytes(ctypes.byref(p))
        least = lib.corope_bwd_min_workspace_bytes(ctypes.byref(p))
        panels = lib.corope_bwd_panel_bytes(ctypes.byref(p))
    else:
        full = lib.corope_bwd_chunk_workspace_bytes(ctypes.byref(p), ctypes.byref(chunk))
        least = lib.corope_bwd_chunk_min_workspace_bytes(ctypes.byref(p), ctypes.byref(chunk))
        keys = BwdParams.from_buffer_copy(p)
        keys.seq_len = chunk.kv_len
        panels = lib.corope_bwd_panel_bytes(ctypes.byref(keys))
    units = p.batch * p.heads
    budget = AUTO_WORKSPACE_BUDGET
    if full > budget and full > least + panels:
        per = (full - least - panels) // units
        budget = max(budget, least + panels + floor_slices(units, p.seq_len) * per)
    return fit_workspace(full, least, units, budget, panels)


def fit_workspace(full, least, units, budget, panels=0):
    """Largest of full / least + panels + k whole hand-off slices / least
    within `budget` bytes (least even when it does not fit: the call then
    fails in the allocator, as the caller's own allocation would).  The
    library lays the workspace out as [least][panels][hand-off]."""
    if full <= budget or full == least:
        return full
    if least + panels > budget:
        return least
    base = least + panels
    per = (full - base) // units  # >= one slice's bytes (the region is 256-aligned)
    if per <= 0:
        return base
    slices = max(0, (budget - base) // per)
    return base + min(slices, units) * per


def bwd(q, k, v, o, do, m, l, a, dq, dk, dv, sm_scale, theta, bias=None, algo="auto",
        thetas=None, workspace="auto", q_row0=None, dk_accum=None, dv_accum=None,
        accum_chunk_rows=0, deterministic=False):
    """Launch corope_bwd on the current stream of q with a torch-allocated
    workspace: "auto" (auto_workspace_bytes: the full size up to 4 GiB, else
    as many hand-off slices as fit), "full" (corope_bwd_workspace_bytes, the fastest),
    "min" (corope_bwd_min_workspace_bytes) or a byte count in between.

    With ``q_row0`` (corope_bwd_chunk) q, o, do, m, l, a, dq are the query rows
    at sequence positions q_row0.., k, v hold every key row, ``dk``/``dv`` are
    ignored and this chunk's key gradients are added to the contiguous fp32
    ``dk_accum``/``dv_accum``: [B, Hkv, kv_len, D], or with
    ``accum_chunk_rows`` = C the zig-zag owner-major layout
    [2, N, B, Hkv, C, D] of 2N chunks of C keys (corope_chunk_t).

    ``deterministic`` sets COROPE_BWD_DETERMINISTIC: dk and dv summed in
    64-bit fixed point, bit-identical from call to call (not with q_row0)."""
    lib = load_library()
    B, H, S, D = q.shape
    p = BwdParams()
    p.q, p.k, p.v, p.o, p.dout = (q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                  do.data_ptr())
    p.m, p.l, p.a = m.data_ptr(), l.data_ptr(), a.data_ptr()
    th = thetas if thetas is not None else theta_table(D, theta, q.device)
    p.thetas = th.data_ptr()
    if bias is not None:
        p.bias = bias.data_ptr()
        p.bias_row_stride = bias.stride(0)
    p.dq = dq.data_ptr()
    p.q_stride, p.k_stride, p.v_stride = _strides(q), _strides(k), _strides(v)
    p.o_stride, p.do_stride, p.dq_stride = _strides(o), _strides(do), _strides(dq)
    chunk = None
    if q_row0 is None:
        p.dk, p.dv = dk.data_ptr(), dv.data_ptr()
        p.dk_stride, p.dv_stride = _strides(dk), _strides(dv)
    else:
        for t in (dk_accum, dv_accum):
            assert t is not None and t.dtype == torch.float32 and t.is_contiguous()
            assert t.numel() == k.numel()
        chunk = ChunkParams()
        chunk.q_row0, chunk.kv_len = int(q_row0), k.shape[2]
        chunk.accum_chunk_rows = int(accum_chunk_rows)
        chunk.dk_accum, chunk.dv_accum = dk_accum.data_ptr(), dv_accum.data_ptr()
    p.batch, p.heads, p.kv_heads, p.seq_len, p.head_dim = B, H, k.shape[1], S, D
    p.sm_scale, p.theta = float(sm_scale), float(theta)
    p.causal, p.dtype, p.algo = 1, _dtype_code(q), algo_code(algo)
    if deterministic:
        p.algo |= BWD_DETERMINISTIC
    if workspace == "auto":
        nbytes = auto_workspace_bytes(lib, p, q.device, chunk)
    elif workspace == "full":
        nbytes = (lib.corope_bwd_workspace_bytes(ctypes.byref(p)) if chunk is None else
                  lib.corope_bwd_chunk_workspace_bytes(ctypes.byref(p), ctypes.byref(chunk)))
    elif workspace == "min":
        nbytes = (lib.corope_bwd_min_workspace_bytes(ctypes.byref(p)) if chunk is None else
                  lib.corope_bwd_chunk_min_workspace_bytes(ctypes.byref(p), ctypes.byref(chunk)))
    else:
        nbytes = int(workspace)
    least = (lib.corope_bwd_min_workspace_bytes(ctypes.byref(p)) if chunk is None else
             lib.corope_bwd_chunk_min_workspace_bytes(ctypes.byref(p), ctypes.byref(chunk)))
    ws, nbytes = _alloc_workspace(nbytes, least, q.device)
    p.workspace, p.workspace_bytes = ws.data_ptr(), nbytes
    stream = torch.cuda.current_stream(q.device).cuda_stream
    with torch.cuda.device(q.device):
        if chunk is None:
            rc = lib.corope_bwd(ctypes.byref(p), ctypes.c_void_p(stream))
        else:
            rc = lib.corope_bwd_chunk(ctypes.byref(p), ctypes.byref(chunk), ctypes.c_void_p(stream))
    _check(rc, "corope_bwd" if chunk is None else "corope_bwd_chunk")
    return ws
