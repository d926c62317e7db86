// C ABI of libcorope_b200.so: argument checks, workspace carving and kernel
// dispatch.  No device memory is allocated here; errors are reported as
// status codes plus a thread-local message (nothing throws across the ABI).
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "common.cuh"

namespace corope {
cudaError_t exact_fwd_launch(const FwdArgs& a, int dtype, cudaStream_t st);
cudaError_t exact_bwd_launch(const BwdArgs& a, int dtype, cudaStream_t st);
bool exact_supports_head_dim(int D);
// tensor-core path (tc_fwd.cu); returns cudaErrorNotSupported when the
// shape is outside its coverage
bool tc_fwd_supported(const FwdArgs& a, int dtype);
cudaError_t tc_fwd_launch(const FwdArgs& a, int dtype, cudaStream_t st, void* ws,
                          size_t ws_bytes);
size_t tc_fwd_workspace_bytes(const FwdArgs& a);
int tc_take_device_error();
bool tc_bwd_supported(const BwdArgs& a, int dtype);
cudaError_t tc_bwd_launch(const BwdArgs& a, int dtype, cudaStream_t st, void* handoff,
                          size_t handoff_bytes, void* panels);
size_t tc_bwd_panel_bytes(const BwdArgs& a);
size_t tc_bwd_coef_bytes();
bool tc_flash_supported(const FwdArgs& a, int dtype);
cudaError_t tc_flash_launch(const FwdArgs& a, int dtype, bool causal, cudaStream_t st);
int tcf_take_device_error();
int64_t tc_bwd_handoff_bytes_per_bh(int S, int r0);
int tcb_take_device_error();
cudaError_t bwd_pre_launch(const BwdArgs& a, int dtype, cudaStream_t st);
cudaError_t bwd_post_launch(const BwdArgs& a, int dtype, cudaStream_t st);
}  // namespace corope

using namespace corope;

static thread_local char g_err[512] = "";

static int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

namespace corope {
// Record `msg` as this thread's last error and return `code` (for the other
// translation units of the library).
int set_last_error(int code, const char* msg) {
  snprintf(g_err, sizeof(g_err), "%s", msg);
  return code;
}
}  // namespace corope

static int cuda_fail(cudaError_t e, const char* what) {
  return fail(COROPE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

static bool aligned(const void* p, size_t n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

static size_t dtype_size(int dt) {
  switch (dt) {
    case COROPE_DTYPE_F32: return 4;
    case COROPE_DTYPE_F16: return 2;
    case COROPE_DTYPE_BF16: return 2;
    default: return 0;
  }
}

// Device must be compute capability 10.0 (B200) for the sm_100a image.
static int check_device() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0)
    return fail(COROPE_ERR_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a", dev,
                major, minor);
  return COROPE_OK;
}

static int check_common(int B, int H, int Hkv, int S, int D, int causal, int dtype, float sm,
                        float theta) {
  if (B <= 0 || H <= 0 || Hkv <= 0 || S <= 0 || D <= 0)
    return fail(COROPE_ERR_INVALID, "sizes must be positive (B=%d H=%d Hkv=%d S=%d D=%d)", B, H,
                Hkv, S, D);
  if (H % Hkv != 0)
    return fail(COROPE_ERR_INVALID, "kv_heads (%d) must divide heads (%d)", Hkv, H);
  if (D % 2 != 0) return fail(COROPE_ERR_INVALID, "head_dim must be even (got %d)", D);
  if (!exact_supports_head_dim(D))
    return fail(COROPE_ERR_UNSUPPORTED, "head_dim %d not supported (4, 8, 16, 32, 64, 128)", D);
  if (!causal)
    return fail(COROPE_ERR_UNSUPPORTED,
                "causal=False is not implemented (the reference kernels are causal only)");
  if (dtype_size(dtype) == 0) return fail(COROPE_ERR_INVALID, "unknown dtype %d", dtype);
  if (!(sm > 0.f) || !(theta > 0.f))
    return fail(COROPE_ERR_INVALID, "sm_scale and theta must be positive");
  return COROPE_OK;
}

static int check_tensor(const void* p, const int64_t* st, const char* name, int dtype) {
  if (!p) return fail(COROPE_ERR_INVALID, "%s is NULL", name);
  if (!aligned(p, dtype_size(dtype)))
    return fail(COROPE_ERR_INVALID, "%s is not aligned to its element size", name);
  for (int i = 0; i < 3; ++i)
    if (st[i] < 0) return fail(COROPE_ERR_INVALID, "%s has a negative stride", name);
  if (st[0] % 2 || st[1] % 2 || st[2] % 2 || !aligned(p, 2 * dtype_size(dtype)))
    return fail(COROPE_ERR_INVALID, "%s strides must be even (rows start on a pair)", name);
  return COROPE_OK;
}

static void copy3(int64_t* d, const int64_t* s) { d[0] = s[0]; d[1] = s[1]; d[2] = s[2]; }

// A query chunk: row offset tile-aligned, k / v long enough for every row.
static int check_chunk(const corope_chunk_t* c, int seq_len) {
  if (!c) return fail(COROPE_ERR_INVALID, "chunk is NULL");
  if (c->q_row0 < 0 || c->q_row0 % 128 != 0)
    return fail(COROPE_ERR_INVALID, "q_row0 must be a non-negative multiple of 128 (got %lld)",
                (long long)c->q_row0);
  if (c->q_row0 + seq_len > (int64_t)c->kv_len || c->q_row0 + seq_len > INT32_MAX)
    return fail(COROPE_ERR_INVALID, "kv_len (%d) must cover q_row0 + seq_len (%lld)", c->kv_len,
                (long long)(c->q_row0 + seq_len));
  if (c->accum_chunk_rows < 0 || c->accum_chunk_rows % 16 != 0 ||
      (c->accum_chunk_rows > 0 && c->kv_len % (2 * c->accum_chunk_rows) != 0))
    return fail(COROPE_ERR_INVALID,
                "accum_chunk_rows (%d) must be 0 or a multiple of 16 dividing kv_len (%d) into "
                "an even number of chunks", c->accum_chunk_rows, c->kv_len);
  return COROPE_OK;
}

static int fwd_common(const corope_fwd_params_t* p, corope_stream_t stream, bool mqa,
                      const corope_chunk_t* chunk = nullptr) {
  if (!p) return fail(COROPE_ERR_INVALID, "params is NULL");
  int rc = check_common(p->batch, p->heads, p->kv_heads, p->seq_len, p->head_dim, p->causal,
                        p->dtype, p->sm_scale, p->theta);
  if (rc) return rc;
  if (chunk && (rc = check_chunk(chunk, p->seq_len))) return rc;
  const int r0 = chunk ? (int)chunk->q_row0 : 0;
  const int Sk = chunk ? chunk->kv_len : p->seq_len;
  if (!mqa && p->kv_heads != p->heads)
    return fail(COROPE_ERR_INVALID, "corope_fwd needs kv_heads == heads; use corope_mqa_fwd");
  if ((rc = check_tensor(p->q, p->q_stride, "q", p->dtype))) return rc;
  if ((rc = check_tensor(p->k, p->k_stride, "k", p->dtype))) return rc;
  if ((rc = check_tensor(p->v, p->v_stride, "v", p->dtype))) return rc;
  if ((rc = check_tensor(p->o, p->o_stride, "o", p->dtype))) return rc;
  if (p->bias && p->bias_row_stride < r0 + p->seq_len)
    return fail(COROPE_ERR_INVALID, "bias_row_stride must be >= seq_len (q_row0 + seq_len)");
  if ((rc = check_device())) return rc;

  FwdArgs a{};
  a.q = p->q; a.k = p->k; a.v = p->v; a.o = p->o;
  a.m = p->m; a.l = p->l; a.a = p->a; a.lse = p->lse;
  a.thetas = p->thetas; a.bias = p->bias; a.bias_rs = p->bias_row_stride;
  copy3(a.qs, p->q_stride); copy3(a.ks, p->k_stride); copy3(a.vs, p->v_stride);
  copy3(a.os, p->o_stride);
  a.B = p->batch; a.H = p->heads; a.Hkv = p->kv_heads; a.S = p->seq_len; a.D = p->head_dim;
  a.sm_scale = p->sm_scale; a.theta = p->theta;
  a.r0 = r0; a.Sk = Sk;

  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool tc_ok = tc_fwd_supported(a, p->dtype);
  if (p->algo == COROPE_ALGO_TENSOR && !tc_ok)
    return fail(COROPE_ERR_UNSUPPORTED,
                "tensor-core forward needs bf16/f16, head_dim 64 or 128, theta >= 1 and "
                "16-byte aligned rows");
  if (p->algo != COROPE_ALGO_EXACT && p->algo != COROPE_ALGO_AUTO && p->algo != COROPE_ALGO_TENSOR)
    return fail(COROPE_ERR_INVALID, "unknown algo %d", p->algo);
  if (p->workspace && !aligned(p->workspace, 256))
    return fail(COROPE_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  cudaError_t e = (p->algo != COROPE_ALGO_EXACT && tc_ok)
                      ? tc_fwd_launch(a, p->dtype, st, p->workspace, p->workspace_bytes)
                      : exact_fwd_launch(a, p->dtype, st);
  if (e != cudaSuccess) return cuda_fail(e, "forward launch");
  return COROPE_OK;
}

static size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// The backward's algorithm without the COROPE_BWD_DETERMINISTIC flag.
static int bwd_algo(const corope_bwd_params_t* p) { return p->algo & ~COROPE_BWD_DETERMINISTIC; }
static bool bwd_fixed(const corope_bwd_params_t* p) {
  return (p->algo & COROPE_BWD_DETERMINISTIC) != 0;
}

// Whether the tensor-core backward may run for these parameters (the rest of
// its conditions, on the tensors, are checked at launch).
static bool bwd_tc_possible(const corope_bwd_params_t* p) {
  return (p->head_dim == 64 || p->head_dim == 128) && bwd_algo(p) != COROPE_ALGO_EXACT &&
         (p->dtype == COROPE_DTYPE_BF16 || p->dtype == COROPE_DTYPE_F16) && p->theta >= 1.f;
}

// The tensor-core backward's expansion coefficients (tc_bwd_coef_bytes) when
// that path can run for these parameters, else 0.
static size_t bwd_coef_ws(const corope_bwd_params_t* p) {
  return bwd_tc_possible(p) ? align256(tc_bwd_coef_bytes()) : 0;
}

// Minimum workspace: delta and lse rows, the tensor-core path's expansion
// coefficients, dk / dv accumulators -- fp32, or 64-bit fixed point with
// COROPE_BWD_DETERMINISTIC (a query chunk accumulates into the caller's fp32
// dk_accum / dv_accum instead).
static size_t bwd_ws(const corope_bwd_params_t* p, bool chunk = false) {
  const size_t rows = (size_t)p->batch * p->heads * p->seq_len;
  const size_t kv = (size_t)p->batch * p->kv_heads * p->seq_len * p->head_dim;
  const size_t acc = kv * (bwd_fixed(p) ? 8 : 4);
  return 2 * align256(rows * 4) + bwd_coef_ws(p) + (chunk ? 0 : 2 * align256(acc));
}

// Optional hand-off region after it (tensor-core backward only): the dQ
// kernel's per-(row, key) results for the dK kernel, 20,992 bytes per 128 query
// rows x 16 keys; with less, the (b, h) slices go through it in chunks, or the
// dK kernel recomputes them.
static size_t bwd_handoff_ws(const corope_bwd_params_t* p, int r0 = 0) {
  if (!bwd_tc_possible(p)) return 0;
  return align256((size_t)p->batch * p->heads *
                  (size_t)tc_bwd_handoff_bytes_per_bh(p->seq_len, r0));
}

// Optional scaled-key panels of the dQ kernel (tensor-core path), placed
// right after the minimum workspace when the workspace has room for them.
static size_t bwd_panel_ws(const corope_bwd_params_t* p, int kv_len) {
  if (!bwd_tc_possible(p)) return 0;
  BwdArgs a{};
  a.B = p->batch; a.Hkv = p->kv_heads; a.Sk = kv_len; a.D = p->head_dim;
  a.theta = p->theta; a.sm_scale = p->sm_scale;
  return align256(tc_bwd_panel_bytes(a));
}

static bool sizes_ok(const corope_bwd_params_t* p) {
  return p && p->batch > 0 && p->heads > 0 && p->kv_heads > 0 && p->seq_len > 0 &&
         p->head_dim > 0;
}

static int bwd_common(const corope_bwd_params_t* p, corope_stream_t stream,
                      const corope_chunk_t* chunk);

extern "C" {

int corope_fwd(const corope_fwd_params_t* p, corope_stream_t stream) {
  return fwd_common(p, stream, false);
}

size_t corope_fwd_workspace_bytes(const corope_fwd_params_t* p) {
  if (!p || p->batch <= 0 || p->heads <= 0 || p->kv_heads <= 0 || p->seq_len <= 0 ||
      (p->head_dim != 64 && p->head_dim != 128) || p->algo == COROPE_ALGO_EXACT ||
      (p->dtype != COROPE_DTYPE_BF16 && p->dtype != COROPE_DTYPE_F16) || !(p->theta >= 1.f))
    return 0;
  FwdArgs a{};
  a.B = p->batch; a.Hkv = p->kv_heads; a.Sk = p->seq_len; a.D = p->head_dim;
  a.theta = p->theta; a.sm_scale = p->sm_scale;
  return tc_fwd_workspace_bytes(a);
}

size_t corope_fwd_chunk_workspace_bytes(const corope_fwd_params_t* p, const corope_chunk_t* c) {
  if (!p || !c || c->kv_len <= 0) return 0;
  corope_fwd_params_t q = *p;
  q.seq_len = c->kv_len;
  return corope_fwd_workspace_bytes(&q);
}

int corope_mqa_fwd(const corope_fwd_params_t* p, corope_stream_t stream) {
  return fwd_common(p, stream, true);
}

size_t corope_bwd_workspace_bytes(const corope_bwd_params_t* p) {
  if (!sizes_ok(p)) return 0;
  return bwd_ws(p) + bwd_panel_ws(p, p->seq_len) + bwd_handoff_ws(p);
}

size_t corope_bwd_panel_bytes(const corope_bwd_params_t* p) {
  if (!sizes_ok(p)) return 0;
  return bwd_panel_ws(p, p->seq_len);
}

size_t corope_bwd_min_workspace_bytes(const corope_bwd_params_t* p) {
  if (!sizes_ok(p)) return 0;
  return bwd_ws(p);
}

int corope_bwd(const corope_bwd_params_t* p, corope_stream_t stream) {
  return bwd_common(p, stream, nullptr);
}

int corope_fwd_chunk(const corope_fwd_params_t* p, const corope_chunk_t* chunk,
                     corope_stream_t stream) {
  if (!chunk) return fail(COROPE_ERR_INVALID, "chunk is NULL");
  return fwd_common(p, stream, true, chunk);
}

size_t corope_bwd_chunk_workspace_bytes(const corope_bwd_params_t* p, const corope_chunk_t* c) {
  if (!sizes_ok(p) || !c || c->q_row0 < 0 || c->q_row0 % 128 != 0 || c->kv_len <= 0) return 0;
  return bwd_ws(p, true) + bwd_panel_ws(p, c->kv_len) + bwd_handoff_ws(p, (int)c->q_row0);
}

size_t corope_bwd_chunk_min_workspace_bytes(const corope_bwd_params_t* p,
                                            const corope_chunk_t* c) {
  if (!sizes_ok(p) || !c) return 0;
  return bwd_ws(p, true);
}

int corope_bwd_chunk(const corope_bwd_params_t* p, const corope_chunk_t* chunk,
                     corope_stream_t stream) {
  if (!chunk) return fail(COROPE_ERR_INVALID, "chunk is NULL");
  return bwd_common(p, stream, chunk);
}

}  // extern "C"

// The backward's argument checks, everything before its workspace: sizes,
// flags, tensors, saved state, bias stride and algo.  Touches no device.
static int bwd_check_args(const corope_bwd_params_t* p, const corope_chunk_t* chunk) {
  if (!p) return fail(COROPE_ERR_INVALID, "params is NULL");
  int rc = check_common(p->batch, p->heads, p->kv_heads, p->seq_len, p->head_dim, p->causal,
                        p->dtype, p->sm_scale, p->theta);
  if (rc) return rc;
  if (chunk && (rc = check_chunk(chunk, p->seq_len))) return rc;
  const int r0 = chunk ? (int)chunk->q_row0 : 0;
  if ((rc = check_tensor(p->q, p->q_stride, "q", p->dtype))) return rc;
  if ((rc = check_tensor(p->k, p->k_stride, "k", p->dtype))) return rc;
  if ((rc = check_tensor(p->v, p->v_stride, "v", p->dtype))) return rc;
  if ((rc = check_tensor(p->o, p->o_stride, "o", p->dtype))) return rc;
  if ((rc = check_tensor(p->dout, p->do_stride, "dout", p->dtype))) return rc;
  if ((rc = check_tensor(p->dq, p->dq_stride, "dq", p->dtype))) return rc;
  if (chunk) {
    if (!chunk->dk_accum || !chunk->dv_accum || !aligned(chunk->dk_accum, 4) ||
        !aligned(chunk->dv_accum, 4))
      return fail(COROPE_ERR_INVALID, "chunk dk_accum and dv_accum (fp32) are required");
  } else {
    if ((rc = check_tensor(p->dk, p->dk_stride, "dk", p->dtype))) return rc;
    if ((rc = check_tensor(p->dv, p->dv_stride, "dv", p->dtype))) return rc;
  }
  if (!p->m || !p->l || !p->a) return fail(COROPE_ERR_INVALID, "m, l and a are required");
  if (p->bias && p->bias_row_stride < r0 + p->seq_len)
    return fail(COROPE_ERR_INVALID, "bias_row_stride must be >= seq_len (q_row0 + seq_len)");
  const int algo = bwd_algo(p);
  if (algo != COROPE_ALGO_EXACT && algo != COROPE_ALGO_AUTO && algo != COROPE_ALGO_TENSOR)
    return fail(COROPE_ERR_INVALID, "unknown algo %d", p->algo);
  if (chunk && bwd_fixed(p))
    return fail(COROPE_ERR_UNSUPPORTED,
                "COROPE_BWD_DETERMINISTIC is not available for query chunks (their "
                "accumulators are the caller's fp32 dk_accum / dv_accum)");
  return COROPE_OK;
}

namespace corope {
// For the other translation units: the backward's argument checks (above) and
// the device check, which corope_bwd runs before and after its workspace
// checks respectively.
int bwd_check_args(const corope_bwd_params_t* p) { return ::bwd_check_args(p, nullptr); }
int device_check() { return check_device(); }
}  // namespace corope

static int bwd_common(const corope_bwd_params_t* p, corope_stream_t stream,
                      const corope_chunk_t* chunk) {
  int rc = bwd_check_args(p, chunk);
  if (rc) return rc;
  const int r0 = chunk ? (int)chunk->q_row0 : 0;
  const int Sk = chunk ? chunk->kv_len : p->seq_len;
  const size_t need = bwd_ws(p, chunk != nullptr);
  if (!p->workspace || p->workspace_bytes < need)
    return fail(COROPE_ERR_WORKSPACE, "workspace of %zu bytes required (got %zu)", need,
                p->workspace ? p->workspace_bytes : (size_t)0);
  if (!aligned(p->workspace, 256)) return fail(COROPE_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  if ((rc = check_device())) return rc;

  BwdArgs a{};
  a.q = p->q; a.k = p->k; a.v = p->v; a.o = p->o; a.dout = p->dout;
  a.m = p->m; a.l = p->l; a.a = p->a;
  a.thetas = p->thetas; a.bias = p->bias; a.bias_rs = p->bias_row_stride;
  a.dq = p->dq;
  a.dk = chunk ? nullptr : p->dk;
  a.dv = chunk ? nullptr : p->dv;
  copy3(a.qs, p->q_stride); copy3(a.ks, p->k_stride); copy3(a.vs, p->v_stride);
  copy3(a.os, p->o_stride); copy3(a.dos, p->do_stride); copy3(a.dqs, p->dq_stride);
  copy3(a.dks, p->dk_stride); copy3(a.dvs, p->dv_stride);
  a.B = p->batch; a.H = p->heads; a.Hkv = p->kv_heads; a.S = p->seq_len; a.D = p->head_dim;
  a.sm_scale = p->sm_scale; a.theta = p->theta;
  a.r0 = r0; a.Sk = Sk;

  const size_t rows = (size_t)p->batch * p->heads * p->seq_len;
  const size_t kv = (size_t)p->batch * p->kv_heads * p->seq_len * p->head_dim;
  char* ws = static_cast<char*>(p->workspace);
  a.delta = reinterpret_cast<float*>(ws);
  a.lse = reinterpret_cast<float*>(ws + align256(rows * 4));
  const size_t coef = bwd_coef_ws(p);
  a.coef = coef ? reinterpret_cast<float2*>(ws + 2 * align256(rows * 4)) : nullptr;
  if (chunk) {
    a.dk32 = chunk->dk_accum;
    a.dv32 = chunk->dv_accum;
    a.acc_chunk = chunk->accum_chunk_rows;
  } else {
    // fp32, or 64-bit fixed-point sums (deterministic)
    a.fixed = bwd_fixed(p) ? 1 : 0;
    const size_t acc = align256(kv * (a.fixed ? 8 : 4));
    a.dk32 = reinterpret_cast<float*>(ws + 2 * align256(rows * 4) + coef);
    a.dv32 = reinterpret_cast<float*>(ws + 2 * align256(rows * 4) + coef + acc);
  }

  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int algo = bwd_algo(p);
  const bool tc_ok = tc_bwd_supported(a, p->dtype);
  if (algo == COROPE_ALGO_TENSOR && !tc_ok)
    return fail(COROPE_ERR_UNSUPPORTED,
                "tensor-core backward needs bf16/f16, head_dim 64 or 128, theta >= 1 and "
                "16-byte aligned rows");
  cudaError_t e = cudaSuccess;
  if (!chunk) e = cudaMemsetAsync(a.dk32, 0, 2 * align256(kv * (a.fixed ? 8 : 4)), st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(workspace)");
  if (algo != COROPE_ALGO_EXACT && tc_ok) {
    e = bwd_pre_launch(a, p->dtype, st);
    // [minimum][panels, when they fit][hand-off region: the rest]
    size_t base = need;
    const size_t panels = bwd_panel_ws(p, Sk);
    void* panel_ptr = nullptr;
    if (panels && p->workspace_bytes >= base + panels) {
      panel_ptr = static_cast<char*>(p->workspace) + base;
      base += panels;
    }
    if (e == cudaSuccess)
      e = tc_bwd_launch(a, p->dtype, st, static_cast<char*>(p->workspace) + base,
                        p->workspace_bytes - base, panel_ptr);
    if (e == cudaSuccess && !chunk) e = bwd_post_launch(a, p->dtype, st);
  } else {
    e = exact_bwd_launch(a, p->dtype, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "backward launch");
  return COROPE_OK;
}

extern "C" {

const char* corope_last_error(void) { return g_err; }

int corope_take_device_error(void) {
  const int f = tc_take_device_error();
  const int g = tcb_take_device_error();
  const int h = tcf_take_device_error();
  return f != 0 ? f : g != 0 ? g : h;
}

int corope_flash_fwd(const corope_fwd_params_t* p, corope_stream_t stream) {
  if (!p) return fail(COROPE_ERR_INVALID, "params is NULL");
  if (p->batch <= 0 || p->heads <= 0 || p->kv_heads <= 0 || p->seq_len <= 0 || p->head_dim <= 0)
    return fail(COROPE_ERR_INVALID, "sizes must be positive (B=%d H=%d Hkv=%d S=%d D=%d)",
                p->batch, p->heads, p->kv_heads, p->seq_len, p->head_dim);
  if (p->heads % p->kv_heads != 0)
    return fail(COROPE_ERR_INVALID, "kv_heads (%d) must divide heads (%d)", p->kv_heads,
                p->heads);
  if (p->dtype != COROPE_DTYPE_BF16 && p->dtype != COROPE_DTYPE_F16)
    return fail(p->dtype == COROPE_DTYPE_F32 ? COROPE_ERR_UNSUPPORTED : COROPE_ERR_INVALID,
                "plain attention takes bf16 or f16 (dtype %d)", p->dtype);
  if (p->head_dim != 64 && p->head_dim != 128)
    return fail(COROPE_ERR_UNSUPPORTED, "plain attention head_dim must be 64 or 128 (got %d)",
                p->head_dim);
  if (p->causal != 0 && p->causal != 1)
    return fail(COROPE_ERR_INVALID, "causal must be 0 or 1 (got %d)", p->causal);
  if (!(p->sm_scale > 0.f)) return fail(COROPE_ERR_INVALID, "sm_scale must be positive");
  int rc;
  if ((rc = check_tensor(p->q, p->q_stride, "q", p->dtype))) return rc;
  if ((rc = check_tensor(p->k, p->k_stride, "k", p->dtype))) return rc;
  if ((rc = check_tensor(p->v, p->v_stride, "v", p->dtype))) return rc;
  if ((rc = check_tensor(p->o, p->o_stride, "o", p->dtype))) return rc;
  if ((rc = check_device())) return rc;
  FwdArgs a{};
  a.q = p->q; a.k = p->k; a.v = p->v; a.o = p->o;
  a.m = p->m; a.lse = p->lse;
  copy3(a.qs, p->q_stride); copy3(a.ks, p->k_stride); copy3(a.vs, p->v_stride);
  copy3(a.os, p->o_stride);
  a.B = p->batch; a.H = p->heads; a.Hkv = p->kv_heads; a.S = p->seq_len; a.D = p->head_dim;
  a.Sk = p->seq_len;
  a.sm_scale = p->sm_scale;
  if (!tc_flash_supported(a, p->dtype))
    return fail(COROPE_ERR_UNSUPPORTED, "plain attention needs 16-byte aligned rows");
  const cudaError_t e =
      tc_flash_launch(a, p->dtype, p->causal != 0, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "plain attention launch");
  return COROPE_OK;
}

size_t corope_params_size(int which) {
  return which == 0 ? sizeof(corope_fwd_params_t) : which == 1 ? sizeof(corope_bwd_params_t) : 0;
}

int corope_abi_version(void) { return COROPE_ABI_VERSION; }

}  // extern "C"
