/*
 * corope.h -- C ABI of the B200 CoRoPE attention library (libcorope_b200.so).
 *
 * CoRoPE ("contextual RoPE") attention: for query t and key j <= t the gate
 * z_tj = sigmoid(q_t . k_j) is summed into the contextual position
 * a_tj = sum_{i=j+1..t} z_ti, and the logit is
 * sm_scale * <R(a_tj * theta_p) q_t, k_j> with the interleaved pair rotation
 * R of RoPE and theta_p = theta^(-2p/D).  Causal softmax, then O = P V.
 *
 * Every entry point takes plain device pointers, element strides and sizes,
 * launches on the given CUDA stream and returns a corope_status_t.  Nothing
 * throws; corope_last_error() returns a message for the last failing call of
 * the calling thread.  The library allocates no device memory: the caller
 * passes outputs and (for the backward) a workspace of the size reported by
 * corope_bwd_workspace_bytes().  Calls are stateless and may run concurrently
 * on different streams.
 *
 * Tensor layout: q, o, dO, dq are [B, H, S, D]; k, v, dk, dv are
 * [B, Hkv, S, D] with Hkv dividing H (Hkv == H for MHA, 1 for MQA).  Each
 * tensor is described by its base pointer and three element strides
 * (batch, head, seq); the head_dim stride must be 1.  m, l, a (and lse) are
 * contiguous fp32 [B, H, S].
 */
#ifndef COROPE_B200_H
#define COROPE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t; declared here so that callers need no CUDA
 * headers.  NULL means the legacy default stream. */
typedef struct CUstream_st *corope_stream_t;

typedef enum {
  COROPE_DTYPE_F32 = 0,
  COROPE_DTYPE_F16 = 1,
  COROPE_DTYPE_BF16 = 2
} corope_dtype_t;

typedef enum {
  /* tensor-core kernels where the shape allows them, else exact */
  COROPE_ALGO_AUTO = 0,
  /* per-pair sine/cosine on CUDA cores (fp32 math, any supported shape) */
  COROPE_ALGO_EXACT = 1,
  /* tcgen05 kernels with the windowed Chebyshev expansion of the rotation;
   * COROPE_ERR_UNSUPPORTED when the shape or dtype is not covered */
  COROPE_ALGO_TENSOR = 2
} corope_algo_t;

/* Backward only: OR'd into corope_bwd_params_t.algo, dk and dv are summed in
 * 64-bit fixed point (each contribution rounded to a multiple of 2^-36, sums
 * below 2^27 in magnitude) instead of with fp32 atomics, so that the same
 * inputs give bit-identical dk / dv from call to call (dq is deterministic
 * either way).  The dk / dv accumulators of the minimum workspace double in
 * size; the chunk entry points answer COROPE_ERR_UNSUPPORTED.  The reference
 * has no such mode: its backward adds dk / dv with fp32 atomics as well
 * (CoROPE/co_rope_backward.py:104-110). */
#define COROPE_BWD_DETERMINISTIC 0x100

typedef enum {
  COROPE_OK = 0,
  COROPE_ERR_INVALID = 1,     /* bad argument (shape, stride, pointer) */
  COROPE_ERR_UNSUPPORTED = 2, /* valid but not implemented (e.g. head_dim) */
  COROPE_ERR_CUDA = 3,        /* a CUDA runtime call failed */
  COROPE_ERR_WORKSPACE = 4,   /* workspace missing or too small */
  COROPE_ERR_DEVICE = 5       /* device not sm_100 or kernel image missing */
} corope_status_t;

typedef struct {
  const void *q, *k, *v;   /* inputs, dtype `dtype` */
  void *o;                 /* output [B,H,S,D], dtype `dtype` */
  float *m, *l, *a;        /* outputs [B,H,S] fp32: running max of the
                              logits, sum of exp(logit - m), total gate sum */
  float *lse;              /* optional output [B,H,S] fp32: m + log(l) */
  const float *thetas;     /* optional [D/2] fp32 frequency table; NULL:
                              theta^(-2p/D) computed from `theta`.  The
                              tensor-core kernels derive their expansion
                              coefficients from `theta` (not read back from
                              the table), so under AUTO/TENSOR the table must
                              be theta^(-2p/D) of the same `theta`; theta < 1
                              always runs the exact kernels */
  const float *bias;       /* optional additive logit bias [S,S] fp32 */
  int64_t bias_row_stride; /* elements between bias rows */
  int64_t q_stride[3], k_stride[3], v_stride[3], o_stride[3];
  int32_t batch, heads, kv_heads, seq_len, head_dim;
  float sm_scale, theta;
  int32_t causal; /* must be 1 */
  int32_t dtype;  /* corope_dtype_t */
  int32_t algo;   /* corope_algo_t */
  void *workspace;          /* optional device scratch, 256-byte aligned */
  size_t workspace_bytes;   /* see corope_fwd_workspace_bytes */
} corope_fwd_params_t;

typedef struct {
  const void *q, *k, *v, *o, *dout;   /* saved inputs/output and dO */
  const float *m, *l, *a;             /* saved forward state [B,H,S] */
  const float *thetas;                /* optional [D/2] table, as above */
  const float *bias;                  /* optional bias used in the forward */
  int64_t bias_row_stride;
  void *dq, *dk, *dv;                 /* outputs, dtype `dtype` */
  int64_t q_stride[3], k_stride[3], v_stride[3], o_stride[3], do_stride[3];
  int64_t dq_stride[3], dk_stride[3], dv_stride[3];
  int32_t batch, heads, kv_heads, seq_len, head_dim;
  float sm_scale, theta;
  int32_t causal;
  int32_t dtype;
  int32_t algo;
  void *workspace;                    /* device scratch, 256-byte aligned */
  size_t workspace_bytes;
} corope_bwd_params_t;

/* Bytes of workspace with which the tensor-core forward reads its scaled-key
 * operands from panels written once per call (one launch before the forward
 * kernel) instead of rebuilding them in every CTA; 0 when the path has none.
 * Any workspace smaller than this (or none) gives the same results. */
size_t corope_fwd_workspace_bytes(const corope_fwd_params_t *p);

/* Forward.  Replaces the launch of co_rope_fwd_kernel in
 * CoROPE/forward.py:123-178 (host wrapper co_rope_forward, launch at
 * :149-171); same outputs O, M, L, A (forward.py:110-120). */
int corope_fwd(const corope_fwd_params_t *p, corope_stream_t stream);

/* MQA/GQA forward: k/v carry kv_heads < heads heads shared by groups of
 * heads/kv_heads query heads, optional bias.  Replaces the launch of
 * co_rope_mqa_fwd_kernel in CoROPE/co_rope_mqa_forward.py:107-176 (launch at
 * :151-174; the bias term of :72-75). */
int corope_mqa_fwd(const corope_fwd_params_t *p, corope_stream_t stream);

/* Bytes of workspace corope_bwd uses at its fastest for these parameters:
 * the minimum below plus, for the tensor-core path (head_dim 64 or 128, bf16/f16),
 * the scaled-key panels and a hand-off region of 4,096 bytes per 128 query
 * rows x 16 keys through which the dQ kernel passes its per-(row, key)
 * softmax-gradient weights (f16) to the dK kernel.
 * Any size between the two works (smaller hand-off regions are used slice by
 * slice, or not at all). */
size_t corope_bwd_workspace_bytes(const corope_bwd_params_t *p);

/* Smallest workspace corope_bwd accepts: delta and lse rows, the tensor-core
 * path's expansion coefficients (128 KiB, written per call) and fp32 dk / dv
 * accumulators, 64-bit with COROPE_BWD_DETERMINISTIC (the dK kernel then
 * recomputes the per-(row, key) results).
 * No counterpart in the reference. */
size_t corope_bwd_min_workspace_bytes(const corope_bwd_params_t *p);

/* Part of corope_bwd_workspace_bytes() holding the dQ kernel's scaled-key
 * panels (written once per call instead of rebuilt in every CTA).  The
 * workspace is laid out as [minimum][panels][hand-off region]: the panels are
 * used when the workspace holds at least minimum + panels, and the hand-off
 * region takes what is left. */
size_t corope_bwd_panel_bytes(const corope_bwd_params_t *p);

/* Backward: dq, dk, dv of the CoRoPE attention (gradients through the
 * softmax, the rotation, the contextual positions and the sigmoid gates).
 * Replaces the launch of co_rope_bwd_kernel in
 * CoROPE/co_rope_backward.py:116-211 (launch at :158-185), whose own result
 * is not the gradient of the forward; parity is with autograd through the
 * reference definition check.py:44-103. */
int corope_bwd(const corope_bwd_params_t *p, corope_stream_t stream);

/* Backward without a caller workspace.  No counterpart in the reference:
 * it exists for callers that cannot allocate device memory (a host engine
 * whose plugin interface passes only inputs and outputs, or a process under
 * a fixed pre-reserved memory budget).  The scratch corope_bwd would take
 * from `workspace` comes instead from a 64 MiB array built into the library
 * (every GPU that loads the library holds it until exit); `workspace` and
 * `workspace_bytes` are ignored.  Shapes whose scratch exceeds
 * corope_bwd_noalloc_scratch_bytes() are rejected with COROPE_ERR_WORKSPACE.
 * The first call on a device looks up the array's device address (make it
 * before any stream capture).  All calls on a device share the array, so
 * calls that overlap on the GPU race; serialise them.  Calls no allocator. */
int corope_bwd_noalloc(const corope_bwd_params_t *p, corope_stream_t stream);

/* Size in bytes of the built-in scratch of corope_bwd_noalloc. */
size_t corope_bwd_noalloc_scratch_bytes(void);

/* ---- Query chunks (sequence-sharded callers).  No counterpart in the
 * reference, which runs whole sequences on one device.  A rank of a
 * sequence-sharded job holds some query rows of a sequence and, after an
 * all-gather, every key / value row: the chunk calls compute exactly the
 * rows a whole-sequence call would produce for those query positions.
 *
 * In the params, q, o, m, l, a, lse, dout and dq hold `seq_len` rows that
 * sit at sequence positions q_row0 .. q_row0 + seq_len - 1; k and v hold
 * kv_len rows from position 0; a bias is indexed by sequence positions. */
typedef struct {
  int64_t q_row0;      /* sequence position of row 0 of q; a multiple of 128 */
  int32_t kv_len;      /* rows of k and v; at least q_row0 + seq_len */
  int32_t accum_chunk_rows; /* layout of dk_accum / dv_accum: 0 = [B, kv_heads,
                          kv_len, D]; C > 0 = the zig-zag owner-major layout of a
                          sequence cut into 2N chunks of C rows (C a multiple
                          of 16, kv_len = 2 N C):
                          [2][N][B][kv_heads][C][D], where [0][r] holds chunk r
                          and [1][r] chunk 2N-1-r, the two chunks rank r owns, so
                          that a reduce-scatter of each half hands every rank its
                          keys' sums with no reordering copy */
  float *dk_accum;     /* backward: fp32, contiguous in the layout above;
                          the call ADDS this chunk's dk (zero it once first) */
  float *dv_accum;     /* backward: the same for dv */
} corope_chunk_t;

/* Forward of a query chunk (MHA, or MQA/GQA with kv_heads dividing heads),
 * and its optional workspace (panels of all kv_len keys). */
int corope_fwd_chunk(const corope_fwd_params_t *p, const corope_chunk_t *chunk,
                     corope_stream_t stream);
size_t corope_fwd_chunk_workspace_bytes(const corope_fwd_params_t *p, const corope_chunk_t *chunk);

/* Workspace of corope_bwd_chunk at its fastest, and the least it accepts
 * (delta and lse rows only; dk / dv go to the chunk's accumulators). */
size_t corope_bwd_chunk_workspace_bytes(const corope_bwd_params_t *p, const corope_chunk_t *chunk);
size_t corope_bwd_chunk_min_workspace_bytes(const corope_bwd_params_t *p,
                                            const corope_chunk_t *chunk);

/* Backward of a query chunk: writes dq of its rows and adds its dk, dv
 * (all kv_len key rows; keys past the chunk's last row get nothing) to
 * chunk->dk_accum / dv_accum; p->dk and p->dv are not used. */
int corope_bwd_chunk(const corope_bwd_params_t *p, const corope_chunk_t *chunk,
                     corope_stream_t stream);

/* ---- Plain attention (no contextual positions), the baseline kernel on
 * the same tensor-core pipeline.  Replaces the launch of
 * flash_attention_kernel in CoROPE/flash.py:213-290 (kernel :63-202, launch
 * at :248): O = softmax(sm_scale Q K^T) V, causal (p->causal = 1) or not
 * (0), and the row max M of the scaled logits (:239, stored when p->m is
 * set) plus the optional log-sum-exp.  Uses q, k, v, o, m, lse, the strides,
 * batch, heads, kv_heads (dividing heads), seq_len, head_dim (64 or 128),
 * sm_scale, causal and dtype (bf16 or f16) of the params; the rest is
 * ignored.  Keys past seq_len never enter the softmax (the reference counts
 * the zero-filled keys of its last 64-key block when causal is 0 and seq_len
 * is not a multiple of 64). */
int corope_flash_fwd(const corope_fwd_params_t *p, corope_stream_t stream);

/* Message for the last non-zero status returned on this thread. */
const char *corope_last_error(void);

/* Error word of the tensor-core kernels: every wait inside them is bounded
 * in time; a wait that runs out records a non-zero code here and the kernel
 * returns early instead of hanging.  Returns the code (0 = none, -1 = the
 * read failed) and clears it.  Synchronises with the device. */
int corope_take_device_error(void);

/* sizeof(corope_fwd_params_t) for which == 0, sizeof(corope_bwd_params_t)
 * for which == 1, else 0; lets FFI bindings check their struct layout. */
size_t corope_params_size(int which);

/* ABI version of this header (COROPE_ABI_VERSION). */
int corope_abi_version(void);

#define COROPE_ABI_VERSION 4

#ifdef __cplusplus
}
#endif

#endif /* COROPE_B200_H */
