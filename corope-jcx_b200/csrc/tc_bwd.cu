// Tensor-core (tcgen05) CoRoPE backward for sm_100a, head_dim 64 and 128.
//
// Gradients of  logit_tj = sm <R(a_tj theta) q_t, k_j>  with the contextual
// position a_tj = sum_{i=j+1..t} sigmoid(q_t . k_i).  As in the forward, keys
// go in windows of 16 and a_tj = C_t + c0 + c0 u_tj (C_t: gate sum of the
// keys after the window; u_tj in [-1, 1]).  Windows run ascending so the two
// scans are running prefixes: C_t = A_t - (gate prefix through the window),
// with A_t the total gate sum saved by the forward, and
// dz_ti = sum_{j<i} da_tj (the gradient of the gates).  Per window and row:
//
//   A operand  v_t = R((C_t + c0) theta) q_t                    (64 sin/cos)
//   G GEMM     G_m(t,j) = v_t . K^(m)_j        (K^(m): the forward's scaled keys)
//   Clenshaw   l_tj = sum_m T_m(u) G_m,  l'_tj = sum_m T_m'(u) G_m
//   softmax    P = exp2(l - lse2), dl = P (dP - delta)   (dP = dO V^T GEMM)
//   positions  da = dl ln2 l' / c0, dz = exclusive prefix of da, ds = dz z (1-z)
//   Y_m(t,j) = dl_tj T_m(u_tj)
//
// Two launches share that per-pair work and differ in what they accumulate:
//
//   dQ launch:  X = Y . K^(m) (K = 16 terms x 16 keys) and dq_t +=
//               ln2 R(-(C_t + c0) theta) X_t  (per-row rotation after the GEMM),
//               plus the gate part dq += dS K (UMMA straight into TMEM); and
//               once per window dV^T = dO^T P and dK_gate^T = Q^T dS, added
//               to the dv / dk accumulators of the workspace (fp32 atomics:
//               query tiles race on keys).
//   dK launch:  C^T = v^T . Y (M = head dim, N = 16 terms x 8 keys, K = the 128
//               query rows), then per head dim a combine over the 16 terms
//               with the coefficients and the (i)^m pair rotation, added to
//               the dk accumulator.  With a hand-off region it reads dl from
//               the dQ launch and recomputes only the gates (dk3_kernel);
//               without one it recomputes the whole per-pair chain.
//
// Roles per CTA (128 query rows of one (b, h), 512 threads): warps 0-7 are
// two row warpgroups that share every row -- warpgroup g takes keys 4g..4g+3
// of each 8-key half window and rotation pairs 32g..32g+31 of the A operand
// and the dQ update, and the two meet once per half through shared memory
// for the running gate-gradient prefix; warp 8 TMA; warp 9 UMMA for the G
// GEMMs; warp 10 UMMA for the launch's own GEMMs; warp 11 UMMA for the gate
// and dP GEMMs; warps 12-15 build K^(m) (unless it comes from the panels) and
// add the launch's accumulators to the workspace (dQ launch: dV^T and
// dK_gate^T; dK launch: the per-dimension combine of C^T).  Each UMMA issue
// costs the issuing thread about as long as the tensor core takes to read the
// operands from shared memory, so the GEMM families sit on separate threads.
// Registers are re-balanced with setmaxnreg: rows 176, builders 104, the
// TMA/UMMA warpgroup 56 (2 x 176 + 104 + 56 = 4 x 128, the launch budget).
// Every wait is bounded as in the forward.
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"
#include "tc_common.cuh"

namespace corope {

// First error recorded by a bounded wait of the backward kernels (0: none).
__device__ int g_corope_bwd_error = 0;

int tcb_take_device_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_corope_bwd_error, sizeof(int)) != cudaSuccess) return -1;
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_corope_bwd_error, &zero, sizeof(int));
  }
  return v;
}

namespace tcb {

using tcx::ElemTraits;
using tcx::kC0;
using tcx::kLn2;
using tcx::kLog2e;
using tcx::kSmemLimit;
using tcx::kW;
using tcx::sigmoid_f;
using tcx::bwd_slot_key;

// Head dims 64 and 128.  Shared-memory tiles are always laid out for 128
// (two 64-element slabs); with 64 the second slab of Q, dO and the A rows is
// zero, which keeps the transposed GEMMs (M = head dim) at M = 128.
// Chebyshev terms: 16 in every backward kernel (the position derivative of a
// 14-term expansion errs by up to 2.4% at the highest frequency, 0.2% with 16).
constexpr int kMB = 16;      // Chebyshev terms of the backward
constexpr int NS = 2;        // 64-element slabs in the shared-memory layout
constexpr int NPX = 64;      // rotation pairs of the widest head dim (table width)
constexpr int kBM = 128;     // query rows per CTA
constexpr int kKT = 16;      // keys per K/V tile (one window)
constexpr int kThreads = 512;
constexpr int kRowRegs = 176, kBldRegs = 104, kCtlRegs = 56;
static_assert(2 * kRowRegs + kBldRegs + kCtlRegs == 4 * 128, "register split");
constexpr int MODE_DQ = 0, MODE_DK = 1;

enum : int {
  kErrQ = 201, kErrKvEmpty, kErrKvFull, kErrSd, kErrSdEmpty, kErrAv, kErrAvEmpty, kErrB,
  kErrBEmpty, kErrG, kErrGEmpty, kErrY, kErrX, kErrXFree, kErrC, kErrCEmpty, kErrDrain, kErrXch
};

struct Params {
  CUtensorMap tm_q, tm_k, tm_v, tm_do;
  CUtensorMap tm_km[2];  // precomputed K^(m) panels per slab (KMT launches)
  int km_nhw;            // half windows per (b, kv head) in the panels
  int km_rows[2];        // panel rows per slab
  void* dq;              // dQ launch output, element type of q
  float *dk32, *dv32;    // accumulators [B, Hkv, Sk, D] (or the owner-major chunk layout)
  int acc_chunk;         // 0, or the chunk rows of the owner-major layout (accum_row)
  int fixed;             // accumulators hold 64-bit fixed-point sums (acc_add)
  const float *lse, *delta, *a;  // [B, H, S]
  const float* thetas;
  const float* bias;
  int64_t bias_rs;
  int64_t dqs[3];
  int B, H, Hkv, S;
  int r0, Sk;  // sequence position of row 0 of q / dO / dq (a multiple of kBM); rows of k, v
  float theta;
  int nrow[8];
  int nb;
  int b_slab_off[2];
  int b_buf_bytes;
  int max_items;   // K^(m) item descriptors per builder thread
  int bop;         // shared-memory offset of the K^(m) buffers
  float2* cf;           // dQ launch: per-offset expansion coefficients [16][16][64]
  uint8_t* handoff;     // dQ launch -> dK launch, per (b, h, query tile, window) block
  int64_t blocks_bh;    // hand-off blocks per (b, h)
  int bh0;              // first (b, h) of this launch (blockIdx.y counts from it)
  float coef[kMB][64];
};

// shared memory (bytes from the 1024-aligned base)
constexpr int S_Q = 0;                       // [NS][128 rows][128 B]
constexpr int S_DO = S_Q + NS * 16384;
constexpr int S_K = S_DO + NS * 16384;       // [2 stages][NS][16 rows][128 B]
constexpr int S_V = S_K + 2 * NS * 2048;
constexpr int S_AV = S_V + 2 * NS * 2048;    // A operand rows [NS][128][128 B]
constexpr int S_Y = S_AV + NS * 16384;       // dK: Y rows [NS][128][128 B];
                                             // dQ: staged (cos, sin) [8 chunks][256 threads][16 B]
constexpr int S_DS = S_Y + NS * 16384;       // dQ: P | dS rows [128][128 B] (bytes 64..127)
template <int MODE, int KM> struct SmemTail {
  static constexpr int COEF = S_DS + (MODE == MODE_DQ ? 16384 : 0);
  static constexpr int TH = COEF + KM * NPX * 4;
  static constexpr int BAR = TH + NPX * 4;
  static constexpr int NBAR = 40;
  static constexpr int SLOT = BAR + NBAR * 8;
  // gate-gradient key-pair sums of a window [group][128 rows] x float4
  static constexpr int XCH = (SLOT + 16 + 15) & ~15;
  static constexpr int ITEMS = XCH + 2 * 128 * 16;  // then the K^(m) buffers at Params::bop
};

// tensor memory columns (GW = 8 KM: one G half, terms x keys)
template <int KM> struct TQ {  // dQ launch
  static constexpr uint32_t GW = 8 * KM;
  static constexpr int NSD = KM > 14 ? 1 : 2;  // gate / dP buffers
  // YT: Y (4 KM cols); DVK: dV^T (16 keys) | dK_gate^T (16 keys)
  static constexpr uint32_t X = 0, DQ = 128, G = 256, SG0 = G + GW, DP0 = SG0 + 16 * NSD,
                            YT = DP0 + 16 * NSD, DVK = YT + 4 * KM;
  static_assert(DVK + 32 <= 512, "tmem");
};
template <int KM> struct TK {  // recompute dK launch
  // C0 / C1: C^T of the window's halves
  static constexpr uint32_t GW = 8 * KM;
  static constexpr uint32_t G = 0, SG0 = GW, DP0 = GW + 16, AVT = GW + 32, C0 = AVT + 64,
                            C1 = C0 + GW;
  static_assert(C1 + GW <= 512, "tmem");
};

// Hand-off block (one per (b, h, query tile, window), 128 rows x 16 keys):
// dl = P (dP - delta) of each (row, key) as f16, which the dK launch needs,
// with the in-window positions u (recomputed there from the gates), to
// rebuild Y_m = dl T_m(u).  Quad q = 2 * half + row group holds the keys in
// slots 4 group + 0..3 of the half (tcx::bwd_slot_key), 8 bytes per row.
constexpr int kHB = 4 * 128 * 8;
// dl -> f16 pair, saturated at the largest finite f16 (NaN stays NaN)
__device__ __forceinline__ uint32_t pack_dl(float a, float b) {
  uint32_t r;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}
__device__ __forceinline__ float2 unpack_dl(uint32_t v) {
  return __half22float2(*reinterpret_cast<const __half2*>(&v));
}

// Gates of one window for one row, shared by the dQ and dK launches so that
// both derive the same positions from the same gate scores: z_j =
// sigmoid(s_j) (0 where `keep` says so), u_j = (sum_{i>j} z_i) / c0 - 1 (the
// scaled in-window position of key j); returns sum_j z_j.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float gate_sigmoid(float s) {
  return rcp_approx(__fadd_rn(1.0f, ex2_approx(__fmul_rn(s, -kLog2e))));
}
// PER_OFFSET (dQ launch with panels): each key offset's own expansion,
// u_j = (sum_{i>j} z_i) / c_j - 1 (tcx::offset_halfwidth).
template <bool MASKED, bool PER_OFFSET = false>
__device__ __forceinline__ float window_gates(const uint32_t (&sraw)[16], int j0, int t,
                                              bool row_ok, float (&z)[16], float (&uu)[16]) {
#pragma unroll
  for (int jj = 0; jj < 16; ++jj) {
    const float g = gate_sigmoid(__uint_as_float(sraw[jj]));
    z[jj] = MASKED ? ((row_ok && j0 + jj <= t) ? g : 0.f) : g;
  }
  float suf = 0.f;  // in-window suffix after key jj
#pragma unroll
  for (int jj = 15; jj >= 0; --jj) {
    uu[jj] = __fmaf_rn(suf, PER_OFFSET ? tcx::offset_inv_halfwidth(16, jj) : 1.0f / kC0, -1.0f);
    suf = __fadd_rn(suf, z[jj]);
  }
  return suf;
}
// Compensated (Kahan) running gate prefix: the prefix reaches ~S/2, where
// fp32 steps are 2^-10 at S = 32768, and a plain running sum over S/16
// windows drifts by ~1e-2 -- an angle error of that size in the fastest
// rotation.  base - base_c is the prefix to ~1 ulp.  Returns the gate sum of
// the keys after the window, A_t - prefix.
__device__ __forceinline__ float advance_prefix(float zsum, float A_t, float& base,
                                                float& base_c) {
  const float y = __fsub_rn(zsum, base_c);
  const float s2 = __fadd_rn(base, y);
  base_c = __fsub_rn(__fsub_rn(s2, base), y);
  base = s2;
  return __fadd_rn(__fsub_rn(A_t, base), base_c);
}
// first block of query tile qt within its (b, h): tiles before it are full
// (8 (q + 1) windows each)
__host__ __device__ constexpr int64_t tile_block0(int qt) { return 4ll * qt * (qt + 1); }
// the same within a query chunk starting at sequence position r0 (a multiple of 128)
__host__ __device__ constexpr int64_t chunk_block0(int r0, int qt) {
  return tile_block0(r0 / 128 + qt) - tile_block0(r0 / 128);
}
enum {
  B_Q = 0, B_KVF = 1, B_KVE = 3, B_SDF = 5, B_SDE = 7, B_AVF = 9,
  B_BF = 11,  // [half][buf]
  B_BE = 15,  // [half][buf]
  B_GF = 19,  // [half]
  B_GE = 21,
  B_YA = 22, B_YDONE = 23, B_YB = 24,
  B_XF = 25, B_XFREE = 26, B_YTFREE = 27,        // dQ launch
  B_CF = 28, B_CE = 30, B_YFREE = 32,            // dK launch: [half] x 2
  B_DRAIN11 = 33, B_DRAIN5 = 34, B_DRAIN6 = 35,
  B_XCH = 36,                                    // gate-gradient pair sums (dQ launch)
  B_CF2 = 38, B_CE2 = 39                         // dQ launch: dV / dK_gate GEMMs
};

__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t (&r)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3])
               : "memory");
}

__device__ __forceinline__ uint32_t pack_cs(float c, float s) {
  const __half2 h = __floats2half2_rn(c, s);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack_cs(uint32_t v) {
  return __half22float2(*reinterpret_cast<const __half2*>(&v));
}

// KMT (dQ launch only): the K^(m) operands come from precomputed panels in
// global memory (tcx::panel_kernel) by TMA instead of warps 12-15.
// FIX: the dk / dv accumulators hold 64-bit fixed-point sums (acc_add); a
// template parameter so that the default fp32-atomic path carries no branch
template <typename T, int D, int MODE, bool HAS_BIAS, int KM, bool KMT, bool FIX>
__global__ void __launch_bounds__(kThreads, 1) bwd_kernel(const __grid_constant__ Params P) {
  static_assert(!KMT || MODE == MODE_DQ, "panels feed the dQ launch only");
  using E = ElemTraits<T>;
  using L = SmemTail<MODE, KM>;
  using tq = TQ<KM>;
  using tk = TK<KM>;
  using namespace sm100;
  constexpr int kM = KM;           // Chebyshev terms
  constexpr int NP = D / 2;        // rotation pairs
  constexpr int KSTEPS = D / 16;   // 16-element K steps over the head dim
  constexpr int DSL = D / 64;      // slabs holding data
  constexpr int PW = NP / 2;       // rotation pairs per row warpgroup
  // gate/dP accumulators: double-buffered in the dQ launch, single in the dK
  // launch (its tensor memory holds the A operand and two C regions)
  constexpr int NSD = MODE == MODE_DQ ? tq::NSD : 1;
  // the dQ launch uses the per-offset expansions (tcx::offset_terms): key
  // pairs of window keys 0..7 run 16 terms, those of keys 8..15 eleven (the
  // larger count of their keys), in both halves (tcx::bwd_slot_key); the
  // recompute dK launch one expansion per window
  constexpr bool POFF = MODE == MODE_DQ;
  constexpr int NPT0 = kM, NPT1 = POFF ? 11 : kM;
  static_assert(!POFF || (tcx::offset_terms(16, 8) <= NPT1 && kM == 16), "pair term counts");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + L::SLOT);
  float* s_coef = reinterpret_cast<float*>(smem + L::COEF);
  float* s_th = reinterpret_cast<float*>(smem + L::TH);
  int* err = &g_corope_bwd_error;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qt = gridDim.x - 1 - blockIdx.x;
  const int bh = P.bh0 + blockIdx.y;
  const int h = bh % P.H, b = bh / P.H;
  const int hk = h / (P.H / P.Hkv);
  const int q0 = P.r0 + qt * kBM;  // sequence position of the tile's first row
  const int S = P.r0 + P.S;        // end of this launch's rows (sequence position)
  const int WL = min(S - 1, q0 + kBM - 1) / kW;  // last (highest) window
  const int nb = P.nb;

  if (tid == 0) {
    mbar_init(&bars[B_Q], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[B_KVF + i], 1);
      mbar_init(&bars[B_KVE + i], KMT ? 2 : 2 + 128);  // warps 10 and 11 (+ the builders)
      mbar_init(&bars[B_SDF + i], 1);
      mbar_init(&bars[B_SDE + i], 256);
      mbar_init(&bars[B_GF + i], 1);
      mbar_init(&bars[B_CF + i], 1);
      mbar_init(&bars[B_CE + i], 128);
      mbar_init(&bars[B_XCH + i], 256);
    }
    mbar_init(&bars[B_CF2], 1);
    mbar_init(&bars[B_CE2], 128);
    for (int i = 0; i < 4; ++i) {
      mbar_init(&bars[B_BF + i], KMT ? 1 : 128);
      mbar_init(&bars[B_BE + i], MODE == MODE_DQ ? 2 : 1);  // G (+ X) done with K^(m)
    }
    mbar_init(&bars[B_AVF], 256);
    mbar_init(&bars[B_GE], 256);
    mbar_init(&bars[B_YA], 256);
    mbar_init(&bars[B_YDONE], 1);
    mbar_init(&bars[B_YB], 256);
    mbar_init(&bars[B_XF], 1);
    mbar_init(&bars[B_XFREE], 256);
    mbar_init(&bars[B_YTFREE], 1);
    mbar_init(&bars[B_YFREE], 1);
    mbar_init(&bars[B_DRAIN5], 1);
    mbar_init(&bars[B_DRAIN11], 1);
    mbar_init(&bars[B_DRAIN6], 1);
    fence_mbar_init();
  }
  for (int i = tid; i < kM * NPX; i += kThreads) s_coef[i] = P.coef[i / NPX][i % NPX];
  for (int p = tid; p < NP; p += kThreads) s_th[p] = theta_at(P.thetas, P.theta, p, D);
  // The K^(m) buffers start at zero: the builders skip the pruned (term,
  // head-dim) entries, which the dQ launch's X GEMM still reads densely.
  // With D = 64 the unused second slab of Q, dO and the A rows is zero too
  // (the dK launch's transposed GEMMs read it).
  {
    uint4* kb = reinterpret_cast<uint4*>(smem + P.bop);
    const int n16 = (2 * P.nb * P.b_buf_bytes) / 16;
    for (int i = tid; i < n16; i += kThreads) kb[i] = make_uint4(0u, 0u, 0u, 0u);
    if (DSL == 1) {
      for (int i = tid; i < 1024; i += kThreads) {
        reinterpret_cast<uint4*>(smem + S_Q + 16384)[i] = make_uint4(0u, 0u, 0u, 0u);
        reinterpret_cast<uint4*>(smem + S_DO + 16384)[i] = make_uint4(0u, 0u, 0u, 0u);
        reinterpret_cast<uint4*>(smem + S_AV + 16384)[i] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    fence_async_smem();
  }
  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t sQ = smem_u32(smem + S_Q), sDO = smem_u32(smem + S_DO);
  const uint32_t sK = smem_u32(smem + S_K), sV = smem_u32(smem + S_V);
  const uint32_t sAV = smem_u32(smem + S_AV), sY = smem_u32(smem + S_Y);
  const uint32_t sB = smem_u32(smem + P.bop);
  const uint32_t sDS = smem_u32(smem + S_DS);
  const uint32_t s_th_u = smem_u32(s_th), s_coef_u = smem_u32(s_coef);
  const uint32_t T_SG0 = MODE == MODE_DQ ? tq::SG0 : tk::SG0;
  const uint32_t T_DP0 = MODE == MODE_DQ ? tq::DP0 : tk::DP0;
  const uint32_t T_G = MODE == MODE_DQ ? tq::G : tk::G;

  // Register split.  The barrier after it matters: a warp that finished its
  // role early (warp 11 at once) re-raises its count to 128 at the end, and
  // must not draw on the pool before the row warps have taken their share.
  if (warp >= 8 && warp < 12) {
    regs_dec<kCtlRegs>();
    named_bar(1, kThreads);
    if (warp == 8) {
      // ---------------------------------------------------------- TMA
      if (lane == 0) {
        prefetch_tmap(&P.tm_q);
        prefetch_tmap(&P.tm_k);
        prefetch_tmap(&P.tm_v);
        prefetch_tmap(&P.tm_do);
        mbar_expect_tx(&bars[B_Q], 2 * DSL * 16384);
        for (int s = 0; s < DSL; ++s) {
          tma_load_4d(smem + S_Q + s * 16384, &P.tm_q, &bars[B_Q], 64 * s, q0 - P.r0, h, b);
          tma_load_4d(smem + S_DO + s * 16384, &P.tm_do, &bars[B_Q], 64 * s, q0 - P.r0, h, b);
        }
        int last_use[2] = {-1, -1};
        for (int n = 0; n <= WL; ++n) {  // tile n = the keys of window n
          const int st = n & 1, u = n >> 1;
          if (n >= 2 && !mbar_wait(&bars[B_KVE + st], (u - 1) & 1, err, kErrKvEmpty)) break;
          mbar_expect_tx(&bars[B_KVF + st], 2 * DSL * 2048);
          for (int s = 0; s < DSL; ++s) {
            tma_load_4d(smem + S_K + (st * NS + s) * 2048, &P.tm_k, &bars[B_KVF + st], 64 * s,
                        kKT * n, hk, b);
            tma_load_4d(smem + S_V + (st * NS + s) * 2048, &P.tm_v, &bars[B_KVF + st], 64 * s,
                        kKT * n, hk, b);
          }
          last_use[st] = u;
        }
        for (int st = 0; st < 2; ++st)
          if (last_use[st] >= 0) mbar_wait(&bars[B_KVF + st], last_use[st] & 1, err, kErrDrain);
      } else if (KMT && lane == 1) {
        // ------------------------------------------- K^(m) panel loads
        prefetch_tmap(&P.tm_km[0]);
        if (DSL > 1) prefetch_tmap(&P.tm_km[1]);
        const uint32_t bytes = (P.km_rows[0] + (DSL > 1 ? P.km_rows[1] : 0)) * 128;
        const int panel0 = (b * P.Hkv + hk) * P.km_nhw;
        int last[4] = {-1, -1, -1, -1};  // [half][buffer]: last use issued
        bool ok = true;
        for (int w = 0; ok && w <= WL; ++w) {
          const int buf = w % nb, use = w / nb;
          for (int hh = 0; hh < 2; ++hh) {
            const int i = 2 * hh + buf;
            if (use > 0 && !(ok = mbar_wait(&bars[B_BE + i], (use - 1) & 1, err, kErrBEmpty))) break;
            mbar_expect_tx(&bars[B_BF + i], bytes);
            uint8_t* dst = smem + P.bop + (hh * nb + buf) * P.b_buf_bytes;
            for (int s = 0; s < DSL; ++s)
              tma_load_3d(dst + P.b_slab_off[s], &P.tm_km[s], &bars[B_BF + i], 0, 0,
                          panel0 + 2 * w + hh);
            last[i] = use;
          }
        }
        // no copy may still be in flight when the CTA exits
        for (int i = 0; i < 4; ++i)
          if (last[i] >= 0) mbar_wait(&bars[B_BF + i], last[i] & 1, err, kErrDrain);
      }
    } else if (warp == 9) {
      // ---------------------------------------------- UMMA: G GEMMs
      // The barriers that complete early (K^(m) built, previous half read)
      // are checked before the A operand's, so each half is issued as soon
      // as its last input lands.
      if (lane == 0) {
        bool ok = mbar_wait(&bars[B_Q], 0, err, kErrQ);
        for (int w = 0; ok && w <= WL; ++w) {
          const int buf = w % nb, use = w / nb;
          for (int hh = 0; hh < 2 && ok; ++hh) {
            ok = mbar_wait(&bars[B_BF + 2 * hh + buf], use & 1, err, kErrB);
            // the single G region: the rows have consumed the previous half
            const int prev = 2 * w + hh - 1;
            if (ok && prev >= 0) ok = mbar_wait(&bars[B_GE], prev & 1, err, kErrGEmpty);
            if (ok && hh == 0) ok = mbar_wait(&bars[B_AVF], w & 1, err, kErrAv);
            if (!ok) break;
            tc_fence_after();
            const uint32_t bb = sB + (hh * nb + buf) * P.b_buf_bytes;
#pragma unroll
            for (int s = 0; s < KSTEPS; ++s) {
              const int nr = P.nrow[s];
              if (nr == 0) break;
              const uint64_t bd = sdesc_kmajor(bb + P.b_slab_off[s >> 2] + 32 * (s & 3));
              const uint32_t id = idesc_f16(128, nr, E::kBf16, false);
              if (MODE == MODE_DQ)
                mma_ss(tmem + T_G, sdesc_kmajor(sAV + (s >> 2) * 16384 + 32 * (s & 3)), bd, id,
                       s > 0);
              else
                mma_ts(tmem + T_G, tmem + tk::AVT + 8 * s, bd, id, s > 0);
            }
            mma_commit(&bars[B_GF + hh]);
            mma_commit(&bars[B_BE + 2 * hh + buf]);
          }
        }
        mma_commit(&bars[B_DRAIN5]);
        mbar_wait(&bars[B_DRAIN5], 0, err, kErrDrain);
      }
    } else if (warp == 11) {
      // ------------------------------------ UMMA: gate scores and dP
      // Q K^T and dO V^T of window w into buffer w % NSD, running ahead of
      // the rows as far as the buffers allow.
      if (lane == 0) {
        const uint32_t id_n16 = idesc_f16(128, 16, E::kBf16, false);
        bool ok = mbar_wait(&bars[B_Q], 0, err, kErrQ);
        for (int w = 0; ok && w <= WL; ++w) {
          const int st = w & 1, sb = w % NSD;
          if (!(ok = mbar_wait(&bars[B_KVF + st], (w >> 1) & 1, err, kErrKvFull))) break;
          if (w >= NSD &&
              !(ok = mbar_wait(&bars[B_SDE + sb], ((w / NSD) - 1) & 1, err, kErrSdEmpty)))
            break;
          tc_fence_after();
          const uint32_t kt = sK + st * NS * 2048;
          const uint32_t vt = sV + st * NS * 2048;
          const uint32_t dsg = tmem + T_SG0 + 16 * sb;
          const uint32_t ddp = tmem + T_DP0 + 16 * sb;
#pragma unroll
          for (int s = 0; s < KSTEPS; ++s) {
            const uint32_t off = (s >> 2) * 16384 + 32 * (s & 3);
            const uint32_t koff = (s >> 2) * 2048 + 32 * (s & 3);
            mma_ss(dsg, sdesc_kmajor(sQ + off), sdesc_kmajor(kt + koff), id_n16, s > 0);
            mma_ss(ddp, sdesc_kmajor(sDO + off), sdesc_kmajor(vt + koff), id_n16, s > 0);
          }
          mma_commit(&bars[B_SDF + sb]);
          mma_commit(&bars[B_KVE + st]);
        }
        mma_commit(&bars[B_DRAIN11]);
        mbar_wait(&bars[B_DRAIN11], 0, err, kErrDrain);
      }
    } else if (warp == 10) {
      // -------------------------------- UMMA: the launch's own GEMMs
      if (lane == 0) {
        bool ok = mbar_wait(&bars[B_Q], 0, err, kErrQ);
        tc_fence_after();
        if (MODE == MODE_DQ) {
          const uint32_t id_x = idesc_f16(128, 64, E::kBf16, true);   // B = K^(m), MN-major
          const uint32_t id_g = idesc_f16(128, D, E::kBf16, true);    // B = K tile, MN-major
          const uint32_t id_s = idesc_f16(128, 16, E::kBf16, true) | (1u << 15);  // A, B MN-major
          for (int w = 0; ok && w <= WL; ++w) {
            const int buf = w % nb;
            const int st = w & 1;
            for (int hh = 0; hh < 2 && ok; ++hh) {
              ok = mbar_wait(&bars[hh ? B_YB : B_YA], w & 1, err, kErrY);
              // X is free once the rows have folded the previous window into dq
              if (ok && hh == 0 && w > 0)
                ok = mbar_wait(&bars[B_XFREE], (w - 1) & 1, err, kErrXFree);
              if (!ok) break;
              tc_fence_after();
              const uint32_t bb = sB + (hh * nb + buf) * P.b_buf_bytes;
              // X[:, 0:64) += Y_hh K^(m)[slab 0];  X[:, 64:128) += Y_hh K^(m)[slab 1]
#pragma unroll 1
              for (int s = 0; s < kM / 2; ++s) {  // 16 (term, key) rows per step
                mma_ts(tmem + tq::X, tmem + tq::YT + 8 * s,
                       sdesc_mnmajor(bb + P.b_slab_off[0] + 2048 * s, 16384), id_x,
                       hh > 0 || s > 0);
                if (16 * (s + 1) <= P.nrow[4])
                  mma_ts(tmem + tq::X + 64, tmem + tq::YT + 8 * s,
                         sdesc_mnmajor(bb + P.b_slab_off[1] + 2048 * s, 16384), id_x,
                         hh > 0 || s > 0);
              }
              mma_commit(&bars[B_BE + 2 * hh + buf]);
              if (hh == 0) mma_commit(&bars[B_YDONE]);  // Y half A consumed
            }
            if (!ok) break;
            // gate part: dq += dS K_w  (A = the dS rows, bytes 96..127 of the
            // P | dS rows in shared memory; B = the window's K tile)
            if (!(ok = mbar_wait(&bars[B_KVF + st], (w >> 1) & 1, err, kErrKvFull))) break;
            mma_ss(tmem + tq::DQ, sdesc_kmajor(sDS + 96), sdesc_mnmajor(sK + st * NS * 2048, 2048),
                   id_g, w > 0);
            mma_commit(&bars[B_XF]);
            // dV^T = dO^T P and dK_gate^T = Q^T dS over the window's 16 keys
            // (B = bytes 64..95 / 96..127 of the P | dS rows, K = the 128
            // query rows), once warps 12-15 have read the previous window's
            if (w > 0 && !(ok = mbar_wait(&bars[B_CE2], (w - 1) & 1, err, kErrCEmpty))) break;
            tc_fence_after();
#pragma unroll 1
            for (int s = 0; s < 8; ++s) {
              const uint32_t ko = 2048 * s;
              mma_ss(tmem + tq::DVK, sdesc_mnmajor(sDO + ko, 16384),
                     sdesc_mnmajor(sDS + ko + 64, 16384), id_s, s > 0);
              mma_ss(tmem + tq::DVK + 16, sdesc_mnmajor(sQ + ko, 16384),
                     sdesc_mnmajor(sDS + ko + 96, 16384), id_s, s > 0);
            }
            mma_commit(&bars[B_CF2]);
            mma_commit(&bars[B_YTFREE]);  // Y, P and dS rows all read
            mma_commit(&bars[B_KVE + st]);
          }
        } else {
          const uint32_t id_c = idesc_f16(128, 8 * kM, E::kBf16, true) | (1u << 15);  // A, B MN-major
          for (int w = 0; ok && w <= WL; ++w) {
            for (int hh = 0; hh < 2 && ok; ++hh) {
              ok = mbar_wait(&bars[hh ? B_YB : B_YA], w & 1, err, kErrY);
              if (ok && w > 0) ok = mbar_wait(&bars[B_CE + hh], (w - 1) & 1, err, kErrCEmpty);
              if (!ok) break;
              tc_fence_after();
              const uint32_t creg = tmem + (hh ? tk::C1 : tk::C0);
              // C^T = v^T Y: A = v^T (M = head dim), B = Y^T (N = term x key),
              // K = the 128 query rows, 16 per step
#pragma unroll 1
              for (int s = 0; s < 8; ++s)
                mma_ss(creg, sdesc_mnmajor(sAV + 2048 * s, 16384), sdesc_mnmajor(sY + 2048 * s, 16384),
                       id_c, s > 0);
              mma_commit(&bars[B_CF + hh]);
              if (hh == 0) mma_commit(&bars[B_YDONE]);
            }
            if (!ok) break;
            mma_commit(&bars[B_YFREE]);  // A rows and Y rows all read
            mma_commit(&bars[B_KVE + (w & 1)]);
          }
        }
        mma_commit(&bars[B_DRAIN6]);
        mbar_wait(&bars[B_DRAIN6], 0, err, kErrDrain);
      }
    }
    __syncwarp();
    regs_inc<128>();
  } else if (warp >= 12) {
    // ------ K^(m) builder (without panels) + accumulation into the workspace:
    // dQ launch: dV^T and dK_gate^T of each window; dK launch: the
    // per-dimension combine of C^T
    regs_dec<kBldRegs>();
    named_bar(1, kThreads);
    const int kMaxItems = P.max_items;
    const int gt = tid - 384;
    uint2* items = reinterpret_cast<uint2*>(smem + L::ITEMS);
    int my_n = 0;
    if (!KMT) {
      int item_end[8];
      int acc = 0;
#pragma unroll
      for (int s2 = 0; s2 < 8; ++s2) {
        acc += 2 * P.nrow[s2];
        item_end[s2] = acc;
      }
#pragma unroll 1
      for (int i = 0; i < kMaxItems; ++i) {
        const int it = gt + 128 * i;
        uint2 d = make_uint2(0u, 0u);
        if (it < acc) {
          int s2 = 0, base = 0;
#pragma unroll
          for (int q = 0; q < 7; ++q)
            if (it >= item_end[q]) { s2 = q + 1; base = item_end[q]; }
          const int local = it - base;
          // key row of half 0 (bwd_slot_key(0, slot) & 7 < 4: half 1's row is
          // 4 further, with its swizzled chunk index's bit 2 flipped)
          const int r = local >> 1, c = 2 * s2 + (local & 1), m = r >> 3, j = bwd_slot_key(0, r & 7);
          const uint32_t kofs = (c >> 3) * 2048 + j * 128 + (((c & 7) ^ (j & 7)) << 4);
          // dQ launch: the per-offset complex coefficients of half 0's key
          // (P.cf, float2 index; half 1's key is 4 further: + 4 * 16 * 64);
          // dK launch: the window expansion's coefficient quad in shared memory
          const uint32_t cofs = MODE == MODE_DQ ? (uint32_t)((j * kMB + m) * 64 + 4 * c)
                                                : (uint32_t)((m * NPX + 4 * c) * 4);
          const uint32_t bofs = P.b_slab_off[c >> 3] + sw128_offset(r, c & 7);
          const uint32_t flags = (m & 1) | ((m & 2) ? 2u : 0u) | (((m + 1) & 2) ? 4u : 0u);
          d = make_uint2(kofs | (cofs << 16), bofs | (flags << 16));
          my_n = i + 1;
        }
        items[i * 128 + gt] = d;
      }
    }
    // dK combine: this thread owns head dim d = gt (lane of the C regions).
    // cm[m] = ln2 * coef_{m, d/2} * sign of (i)^m for this component; odd m
    // take the partner component (d ^ 1).
    float cm[kM];
    if (MODE == MODE_DK) {
      const int p = gt >> 1, e = gt & 1;
#pragma unroll
      for (int m = 0; m < kM; ++m) {
        float sgn;
        switch (m & 3) {
          case 0: sgn = 1.f; break;
          case 1: sgn = e ? 1.f : -1.f; break;
          case 2: sgn = -1.f; break;
          default: sgn = e ? -1.f : 1.f; break;
        }
        if ((m & 3) >= 2) sgn = -sgn;  // the rows store s_m Y_m (see the Y recurrence)
        cm[m] = kLn2 * s_coef[m * NPX + p] * sgn;  // zero for p >= D / 2
      }
    }
    const uint32_t lane_base = tmem + ((uint32_t)((warp - 12) * 32) << 16);
    const int bhk = b * P.Hkv + hk, BHkv = P.B * P.Hkv;

    auto build = [&](int w) -> bool {
      const int buf = w % nb, use = w / nb;
      const int st = w & 1;
      if (!wwait(bars[B_KVF + st], (w >> 1) & 1, err, kErrKvFull)) return false;
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        if (use > 0 && !wwait(bars[B_BE + 2 * hh + buf], (use - 1) & 1, err, kErrBEmpty))
          return false;
        const uint32_t kt = sK + st * NS * 2048;
        const uint32_t bt = sB + (hh * nb + buf) * P.b_buf_bytes;
#pragma unroll 1
        for (int i0 = 0; i0 < my_n; i0 += 4) {
          uint2 d[4];
          uint4 kv[4];
          float4 cf[4], cg[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) d[j] = items[(i0 + j < kMaxItems ? i0 + j : 0) * 128 + gt];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t ko = d[j].x & 0xffffu;
            kv[j] = lds128(kt + (hh ? ((ko + 512u) ^ 64u) : ko));
            if (MODE == MODE_DQ) {
              const float4* cp =
                  reinterpret_cast<const float4*>(P.cf + (d[j].x >> 16) + hh * 4 * kMB * 64);
              cf[j] = __ldg(cp);
              cg[j] = __ldg(cp + 1);
            } else {
              cf[j] = lds128f(s_coef_u + (d[j].x >> 16));
            }
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (MODE == MODE_DQ && i0 + j < my_n) {
              // per-offset expansions: the same arithmetic as the panel kernel
              sts128(bt + (d[j].y & 0xffffu),
                     make_uint4(tcx::cmul_pack<E>(kv[j].x, cf[j].x, cf[j].y),
                                tcx::cmul_pack<E>(kv[j].y, cf[j].z, cf[j].w),
                                tcx::cmul_pack<E>(kv[j].z, cg[j].x, cg[j].y),
                                tcx::cmul_pack<E>(kv[j].w, cg[j].z, cg[j].w)));
            } else if (i0 + j < my_n) {
              // (-i)^m: odd terms swap the pair's components (one byte
              // permute), terms 2, 3 mod 4 negate one or both (a sign-bit xor)
              const uint32_t fl = d[j].y >> 16;
              const uint32_t sel = (fl & 1u) ? 0x1032u : 0x3210u;
              const uint32_t sgn = ((fl & 2u) ? 0x8000u : 0u) | ((fl & 4u) ? 0x80000000u : 0u);
              const uint32_t in[4] = {kv[j].x, kv[j].y, kv[j].z, kv[j].w};
              const float cfa[4] = {cf[j].x, cf[j].y, cf[j].z, cf[j].w};
              uint32_t out[4];
#pragma unroll
              for (int e2 = 0; e2 < 4; ++e2) {
                const uint32_t wv = __byte_perm(in[e2], 0u, sel) ^ sgn;
                out[e2] = E::pack(cfa[e2] * E::lo(wv), cfa[e2] * E::hi(wv));
              }
              sts128(bt + (d[j].y & 0xffffu), make_uint4(out[0], out[1], out[2], out[3]));
            }
          }
        }
        fence_async_smem();
        mbar_arrive(&bars[B_BF + 2 * hh + buf]);
      }
      mbar_arrive(&bars[B_KVE + st]);
      return true;
    };

    auto combine = [&](int w) -> bool {
      float dk[16];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        if (!wwait(bars[B_CF + hh], w & 1, err, kErrC)) return false;
        tc_fence_after();
        const uint32_t creg = lane_base + (hh ? tk::C1 : tk::C0);
#pragma unroll
        for (int j = 0; j < 8; ++j) dk[8 * hh + j] = 0.f;
#pragma unroll
        for (int c0 = 0; c0 < kM / 2; c0 += 2) {  // terms 2c, 2c+1 for the 8 keys
          uint32_t g[2][16];
#pragma unroll
          for (int i = 0; i < 2; ++i)
            if (c0 + i < kM / 2) tmem_ld16(creg + 16 * (c0 + i), g[i]);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int c = c0 + i;
            if (c >= kM / 2) continue;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float own = __uint_as_float(g[i][j]);
              const float partner = __shfl_xor_sync(0xffffffffu, __uint_as_float(g[i][8 + j]), 1);
              dk[8 * hh + j] = fmaf(cm[2 * c], own, dk[8 * hh + j]);
              dk[8 * hh + j] = fmaf(cm[2 * c + 1], partner, dk[8 * hh + j]);
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&bars[B_CE + hh]);
      }
      const int d = gt;
      // a window's 16 keys lie in one accumulator chunk (chunks are multiples of 16 keys);
      // column 8 hh + s of C^T is slot s of half hh
      const int64_t row0 = accum_row(w * kW, bhk, BHkv, P.Sk, P.acc_chunk) * D + d;
      constexpr bool fixed = FIX;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int key = bwd_slot_key(j >> 3, j & 7);
        if (w * kW + key < P.Sk && d < D) acc_add(P.dk32, row0 + key * D, dk[j], fixed);
      }
      return true;
    };

    // dQ launch: dV^T = dO^T P and dK_gate^T = Q^T dS of window w (this
    // thread's head dim d, the window's 16 keys) into the accumulators
    auto dvk = [&](int w) -> bool {
      if (!wwait(bars[B_CF2], w & 1, err, kErrC)) return false;
      tc_fence_after();
      uint32_t g[2][16];
      tmem_ld16(lane_base + tq::DVK, g[0]);       // dO^T P  (16 keys)
      tmem_ld16(lane_base + tq::DVK + 16, g[1]);  // Q^T dS  (16 keys)
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&bars[B_CE2]);
      const int d = gt;
      // a window's 16 keys lie in one accumulator chunk (chunks are multiples of 16 keys)
      const int64_t row0 = accum_row(w * kW, bhk, BHkv, P.Sk, P.acc_chunk) * D + d;
      constexpr bool fixed = FIX;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (w * kW + j < P.Sk && d < D) {
          acc_add(P.dv32, row0 + j * D, __uint_as_float(g[0][j]), fixed);
          acc_add(P.dk32, row0 + j * D, __uint_as_float(g[1][j]), fixed);
        }
      }
      return true;
    };

    bool ok = KMT ? true : build(0);
    for (int w = 0; ok && w <= WL; ++w) {
      if (!KMT && w + 1 <= WL) ok = build(w + 1);
      if (ok) ok = MODE == MODE_DK ? combine(w) : dvk(w);
    }
    __syncwarp();
    regs_inc<128>();
  } else {
    // ------------------------------------------------------------ row warps
    regs_inc<kRowRegs>();
    named_bar(1, kThreads);
    const int rg = warp >> 2;  // row warpgroup
    const int r = tid & 127;
    const int t = q0 + r;
    const bool row_ok = t < S;
    // windows below the tile's first row of a tile inside the rows need no
    // causal or row mask (CTA-uniform)
    auto diag_window = [&](int w) { return w * kW + kW - 1 > q0 || q0 + kBM > S; };
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const int64_t ri = ((int64_t)b * P.H + h) * P.S + min(t - P.r0, P.S - 1);
    const float A_t = P.a[ri];
    const float lse2 = P.lse[ri] * kLog2e;
    const float delta = P.delta[ri];
    const uint32_t s_xch = smem_u32(smem + L::XCH);
    const uint32_t s_cs = sY + (rg * 128 + r) * 16;  // dQ: staged (cos, sin), chunk q at + 4096 q
    // compensated gate prefix through the current window (advance_prefix)
    float base = 0.f, base_c = 0.f;
    float carry = 0.f;   // gate sum of the keys after the current window
    float da_run = 0.f;  // gate-gradient prefix before the current window
    // this group's keys of the window: slot 4 rg + (i & 3) of half i >> 2, i.e.
    // key 4 (i >> 2) + 2 rg + (i & 1) + 8 ((i >> 1) & 1) (tcx::bwd_slot_key)
    float zo[8], uo[8], dpo[8];
    // d(position) scale of each key: ln 2 / the expansion's half-width
    float dac[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      dac[i] = POFF ? kLn2 * tcx::offset_inv_halfwidth(16, bwd_slot_key(i >> 2, 4 * rg + (i & 3)))
                    : kLn2 / kC0;
    uint32_t csc[PW];    // dQ: (cos, sin) as f16 pairs for this group's pairs
    bool ok = wwait(bars[B_Q], 0, err, kErrQ);

    // gates and positions of window w; reads the gate scores and dP
    auto gates = [&](int w) -> bool {
      const int sb = w % NSD;
      if (!wwait(bars[B_SDF + sb], (w / NSD) & 1, err, kErrSd)) return false;
      tc_fence_after();
      uint32_t sraw[16], dp[8];
      tmem_ld16(lane_base + T_SG0 + 16 * sb, sraw);
      // dP of this group's key pairs: half q >> 1, keys 0..7 (q even) or 8..15
#pragma unroll
      for (int q = 0; q < 4; ++q)
        tmem_ld2(lane_base + T_DP0 + 16 * sb + 4 * (q >> 1) + 2 * rg + 8 * (q & 1), dp[2 * q],
                 dp[2 * q + 1]);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&bars[B_SDE + sb]);
      const int j0 = w * kW;
      float z[16], uu[16];
      const float zsum = diag_window(w) ? window_gates<true, POFF>(sraw, j0, t, row_ok, z, uu)
                                        : window_gates<false, POFF>(sraw, j0, t, row_ok, z, uu);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int k0 = bwd_slot_key(i >> 2, i & 3);  // group 0's key; group 1's is 2 further
        zo[i] = rg ? z[k0 + 2] : z[k0];
        uo[i] = rg ? uu[k0 + 2] : uu[k0];
        dpo[i] = __uint_as_float(dp[i]);
      }
      carry = advance_prefix(zsum, A_t, base, base_c);
      return true;
    };

    // this group's half of the A operand v = R((carry + c0) theta) q_t:
    // dQ launch -> shared memory (and the (cos, sin) staging); dK launch ->
    // tensor memory (the G GEMM's A; copied to shared memory later for C)
    const float th_max = theta_max(s_th, NP);
    auto build_a = [&]() {
      const float bse = carry + kC0;
      const bool mufu_reduce = __all_sync(0xffffffffu, bse * th_max < kMufuReduceMax);
#pragma unroll 1
      for (int g = 0; g < PW / 16; ++g) {
        uint4 qv[4];
        float th[16];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int c = rg * (PW / 4) + 4 * g + cc;  // chunk of the row (4 pairs)
          qv[cc] = lds128(sQ + (c >> 3) * 16384 + sw128_offset(r, c & 7));
          const float4 t4 = lds128f(s_th_u + 16 * c);
          th[4 * cc] = t4.x; th[4 * cc + 1] = t4.y; th[4 * cc + 2] = t4.z; th[4 * cc + 3] = t4.w;
        }
        float rr[16], sn[16], cs[16];
        if (mufu_reduce) {
#pragma unroll
          for (int i = 0; i < 16; ++i) rr[i] = bse * th[i];
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) rr[i] = reduce_2pi(bse * th[i]);
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) __sincosf(rr[i], &sn[i], &cs[i]);
        uint32_t o[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const uint32_t w32 = (i & 3) == 0 ? qv[i >> 2].x : (i & 3) == 1 ? qv[i >> 2].y
                             : (i & 3) == 2 ? qv[i >> 2].z : qv[i >> 2].w;
          const float qe = E::lo(w32), qo = E::hi(w32);
          o[i] = E::pack(qe * cs[i] - qo * sn[i], qe * sn[i] + qo * cs[i]);
        }
        if (MODE == MODE_DQ) {
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const int c = rg * (PW / 4) + 4 * g + cc;
            sts128(sAV + (c >> 3) * 16384 + sw128_offset(r, c & 7),
                   make_uint4(o[4 * cc], o[4 * cc + 1], o[4 * cc + 2], o[4 * cc + 3]));
            // staged for the dQ update
            sts128(s_cs + (4 * g + cc) * 4096,
                   make_uint4(pack_cs(cs[4 * cc], sn[4 * cc]),
                              pack_cs(cs[4 * cc + 1], sn[4 * cc + 1]),
                              pack_cs(cs[4 * cc + 2], sn[4 * cc + 2]),
                              pack_cs(cs[4 * cc + 3], sn[4 * cc + 3])));
          }
        } else {
          tmem_st16(lane_base + tk::AVT + rg * PW + 16 * g, o);
        }
      }
      if (MODE == MODE_DQ) {
        fence_async_smem();
      } else {
        tmem_wait_st();
        tc_fence_before();
      }
      mbar_arrive(&bars[B_AVF]);
    };

    auto load_cs = [&]() {
#pragma unroll
      for (int c = 0; c < PW / 4; ++c) {
        const uint4 v = lds128(s_cs + c * 4096);
        csc[4 * c] = v.x; csc[4 * c + 1] = v.y; csc[4 * c + 2] = v.z; csc[4 * c + 3] = v.w;
      }
    };

    // Clenshaw for this group's 4 keys of a half: logits (log2 units) and
    // their derivative in u.  G columns: 16 c + 8 (m & 1) + key, m = 2 c + (m & 1).
    // All 14 loads are issued before the single wait, after which the G
    // region is released to the next half's GEMM.
    // key pair j runs NPT[j] terms (the chain starts at its first nonzero term)
    auto clenshaw = [&](const float (&uj)[4], float (&f)[4], float (&fd)[4]) {
      constexpr int NPT[2] = {NPT0, NPT1};
      uint32_t g[kM / 2][2][4];
#pragma unroll
      for (int c = 0; c < kM / 2; ++c) {
        tmem_ld4(lane_base + T_G + 16 * c + 4 * rg, g[c][0]);
        tmem_ld4(lane_base + T_G + 16 * c + 8 + 4 * rg, g[c][1]);
      }
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&bars[B_GE]);
      // two keys per packed fp32x2 FMA.  Value: b_m = 2u b_{m+1} + (G_m -
      // b_{m+2}); derivative tracked halved, e = d / 2:
      // e_m = 2u e_{m+1} + (b_{m+1} - e_{m+2}) -- two FMAs per step each
      constexpr bool SGN = MODE == MODE_DQ;
      const float2 neg1 = make_float2(-1.f, -1.f), neg2 = make_float2(-2.f, -2.f);
      const float2 one = make_float2(1.f, 1.f), two = make_float2(2.f, 2.f);
      const float2 nu2[2] = {make_float2(-2.f * uj[0], -2.f * uj[1]),
                             make_float2(-2.f * uj[2], -2.f * uj[3])};
      const float2 u2[2] = {make_float2(2.f * uj[0], 2.f * uj[1]), make_float2(2.f * uj[2], 2.f * uj[3])};
      const float2 u1[2] = {make_float2(uj[0], uj[1]), make_float2(uj[2], uj[3])};
      float2 b1[2], b2[2], e1[2], e2[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        b1[j] = b2[j] = e1[j] = e2[j] = make_float2(0.f, 0.f);
      }
#pragma unroll
      for (int m = kM - 1; m >= 0; --m) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          if (m >= NPT[j]) continue;
          const float2 a = make_float2(__uint_as_float(g[m >> 1][m & 1][2 * j]),
                                       __uint_as_float(g[m >> 1][m & 1][2 * j + 1]));
          if (SGN) {
            // dQ launch: G'_m = s_m G_m (the signs folded into its K^(m)), the
            // basis V_m = s_m T_m with V_{m+1} = a_m V_m + V_{m-1}, a_m = +-2u
            // (minus for odd m): b_m = G'_m + a_m b_{m+1} + b_{m+2},
            // e_m = -+ b_{m+1} + a_m e_{m+1} + e_{m+2} (e = d / 2); then
            // l = G'_0 + u b_1 + b_2 and l' = b_1 + 2u e_1 + 2 e_2
            const float2 t = __ffma2_rn(one, b2[j], a);
            if (m > 0) {
              const float2 al = (m & 1) ? nu2[j] : u2[j];
              const float2 en = __ffma2_rn(al, e1[j], __ffma2_rn((m & 1) ? neg1 : one, b1[j], e2[j]));
              const float2 bn = __ffma2_rn(al, b1[j], t);
              e2[j] = e1[j]; e1[j] = en;
              b2[j] = b1[j]; b1[j] = bn;
            } else {
              const float2 r = __ffma2_rn(u1[j], b1[j], t);
              const float2 rd = __ffma2_rn(u2[j], e1[j], __ffma2_rn(two, e2[j], b1[j]));
              f[2 * j] = r.x; f[2 * j + 1] = r.y;
              fd[2 * j] = rd.x; fd[2 * j + 1] = rd.y;
            }
            continue;
          }
          const float2 t = __ffma2_rn(neg1, b2[j], a);
          if (m > 0) {
            const float2 en = __ffma2_rn(u2[j], e1[j], __ffma2_rn(neg1, e2[j], b1[j]));
            const float2 bn = __ffma2_rn(u2[j], b1[j], t);
            e2[j] = e1[j]; e1[j] = en;
            b2[j] = b1[j]; b1[j] = bn;
          } else {
            const float2 r = __ffma2_rn(u1[j], b1[j], t);
            // l' = u d_1 + b_1 - d_2 = 2 u e_1 + (b_1 - 2 e_2)
            const float2 rd = __ffma2_rn(u2[j], e1[j], __ffma2_rn(neg2, e2[j], b1[j]));
            f[2 * j] = r.x; f[2 * j + 1] = r.y;
            fd[2 * j] = rd.x; fd[2 * j + 1] = rd.y;
          }
        }
      }
    };

    // the two halves of window w
    uint8_t* const hblk0 =
        (MODE == MODE_DQ && P.handoff)
            ? P.handoff + ((int64_t)blockIdx.y * P.blocks_bh + chunk_block0(P.r0, qt)) * kHB
            : nullptr;
    auto halves = [&](int w) -> bool {
      const int j0 = w * kW;
      float da0[4];  // half A's gate gradients, kept for the window's prefix
      uint8_t* const hblk = hblk0 ? hblk0 + (int64_t)w * kHB : nullptr;
      if (MODE == MODE_DK) {
        // the previous window's C GEMMs are done with the A rows and the Y
        // buffer: copy this window's A half from tensor to shared memory
        if (w > 0 && !wwait(bars[B_YFREE], (w - 1) & 1, err, kErrY)) return false;
        tc_fence_after();
#pragma unroll
        for (int g = 0; g < PW / 16; ++g) {
          uint32_t o[16];
          tmem_ld16(lane_base + tk::AVT + rg * PW + 16 * g, o);
          tmem_wait_ld();
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const int c = rg * (PW / 4) + 4 * g + cc;
            sts128(sAV + (c >> 3) * 16384 + sw128_offset(r, c & 7),
                   make_uint4(o[4 * cc], o[4 * cc + 1], o[4 * cc + 2], o[4 * cc + 3]));
          }
        }
      }
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        if (!wwait(bars[B_GF + hh], w & 1, err, kErrG)) return false;
        tc_fence_after();
        float uj[4], zj[4], dpj[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uj[i] = hh ? uo[4 + i] : uo[i];
          zj[i] = hh ? zo[4 + i] : zo[i];
          dpj[i] = hh ? dpo[4 + i] : dpo[i];
        }
        float f[4], fd[4];
        clenshaw(uj, f, fd);
        float dl[4], da[4], pr[4];
        if (diag_window(w)) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int kj = j0 + 4 * hh + 2 * rg + (i & 1) + 8 * (i >> 1);
            const bool valid = row_ok && kj <= t;
            float lg = f[i];
            if (HAS_BIAS && valid) lg = fmaf(P.bias[(int64_t)t * P.bias_rs + kj], kLog2e, lg);
            pr[i] = valid ? exp2f(lg - lse2) : 0.f;
            dl[i] = pr[i] * (dpj[i] - delta);
            da[i] = valid ? dl[i] * (hh ? dac[4 + i] : dac[i]) * fd[i] : 0.f;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int kj = j0 + 4 * hh + 2 * rg + (i & 1) + 8 * (i >> 1);
            float lg = f[i];
            if (HAS_BIAS) lg = fmaf(P.bias[(int64_t)t * P.bias_rs + kj], kLog2e, lg);
            pr[i] = exp2f(lg - lse2);
            dl[i] = pr[i] * (dpj[i] - delta);
            da[i] = dl[i] * (hh ? dac[4 + i] : dac[i]) * fd[i];
          }
        }
        if (hh == 0) {
#pragma unroll
          for (int i = 0; i < 4; ++i) da0[i] = da[i];  // for the window's prefix after half B
        }
        // Y_m = dl T_m(u), packed per term for the group's 4 keys (dQ launch:
        // times ln 2, the base of the logits, so that X and the dq fold carry it)
        uint32_t y[kM][2];
#pragma unroll
        for (int jp = 0; jp < 2; ++jp) {
          // Y_m = dl T_m(u) obeys the Chebyshev recurrence itself,
          // Y_{m+1} = 2u Y_m - Y_{m-1} (Y_0 = dl, Y_1 = dl u).  Stored as
          // V_m = s_m Y_m with s_m = (+, +, -, -, ...): V_m = (-1)^(m+1) 2u
          // V_{m-1} + V_{m-2}, one packed FMA per step for the pair's two keys
          // and no negated operand; the signs are in the dQ launch's K^(m)
          // (its coefficient table) and in the dK launch's combine
          constexpr float ys = MODE == MODE_DQ ? kLn2 : 1.f;
          const float2 u2 = make_float2(2.f * uj[2 * jp], 2.f * uj[2 * jp + 1]);
          const float2 nu2 = make_float2(-2.f * uj[2 * jp], -2.f * uj[2 * jp + 1]);
          float2 v0 = make_float2(ys * dl[2 * jp], ys * dl[2 * jp + 1]);
          float2 v1 = make_float2(v0.x * uj[2 * jp], v0.y * uj[2 * jp + 1]);
          y[0][jp] = E::pack(v0.x, v0.y);
          y[1][jp] = E::pack(v1.x, v1.y);
#pragma unroll
          for (int m = 2; m < kM; ++m) {
            if (m >= (jp ? NPT1 : NPT0)) break;  // the X GEMM's K^(m) rows there are zero
            const float2 v2 = __ffma2_rn((m & 1) ? u2 : nu2, v1, v0);
            v0 = v1;
            v1 = v2;
            y[m][jp] = E::pack(v2.x, v2.y);
          }
        }
        if (MODE == MODE_DQ) {
          // Y half into tensor memory (A operand of X): half A waits until the
          // previous window's GEMMs are done with it, half B until X has
          // consumed half A
          if (hh == 0 && w > 0 && !wwait(bars[B_YTFREE], (w - 1) & 1, err, kErrX)) return false;
          if (hh == 1 && !wwait(bars[B_YDONE], w & 1, err, kErrX)) return false;
          tc_fence_after();
#pragma unroll
          for (int m = 0; m < NPT0; ++m) {
            if (m < NPT1)
              tmem_st2(lane_base + tq::YT + 4 * m + 2 * rg, y[m][0], y[m][1]);
            else
              tmem_st1(lane_base + tq::YT + 4 * m + 2 * rg, y[m][0]);
          }
          if (hh == 0) {
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&bars[B_YA]);
          }
          // P -> chunks 4, 5 of the P | dS rows (B operand of dV^T; keys in
          // order); the previous window's GEMMs are done with them (B_YTFREE above)
          sts32(sDS + sw128_offset(r, 4) + 2 * (4 * hh + 2 * rg), E::pack(pr[0], pr[1]));
          sts32(sDS + sw128_offset(r, 5) + 2 * (4 * hh + 2 * rg), E::pack(pr[2], pr[3]));
        } else {
          // Y rows into shared memory (B operand of the C GEMMs)
          if (hh == 1 && !wwait(bars[B_YDONE], w & 1, err, kErrY)) return false;
#pragma unroll
          for (int m = 0; m < kM; ++m)  // element 8 m + key: chunk m of the row
            sts64(sY + (m >> 3) * 16384 + sw128_offset(r, m & 7) + 8 * rg, y[m][0], y[m][1]);
          fence_async_smem();
          mbar_arrive(&bars[hh ? B_YB : B_YA]);
        }
        if (MODE == MODE_DK) continue;
        if (hblk) {
          const int qd = 2 * hh + rg;
          *reinterpret_cast<uint2*>(hblk + (qd * 128 + r) * 8) =
              make_uint2(pack_dl(dl[0], dl[1]), pack_dl(dl[2], dl[3]));
        }
        if (hh == 0) continue;
        // Gate-gradient prefix over the window's keys in order.  Key pair p
        // (keys 2p, 2p + 1) belongs to group p & 1; this group's pairs in
        // window order are (half 0, keys 0..7), (half 1, 0..7), (half 0,
        // 8..15), (half 1, 8..15).  Each group publishes its four pair sums.
        const float ps[4] = {da0[0] + da0[1], da[0] + da[1], da0[2] + da0[3], da[2] + da[3]};
        sts128f(s_xch + (rg * 128 + r) * 16, make_float4(ps[0], ps[1], ps[2], ps[3]));
        mbar_arrive(&bars[B_XCH]);
        if (!wwait(bars[B_XCH], w & 1, err, kErrXch)) return false;
        const float4 o4 = lds128f(s_xch + ((rg ^ 1) * 128 + r) * 16);
        const float os[4] = {o4.x, o4.y, o4.z, o4.w};
        const float dak[4][2] = {{da0[0], da0[1]}, {da[0], da[1]}, {da0[2], da0[3]}, {da[2], da[3]}};
        const float zk[4][2] = {{zo[0], zo[1]}, {zo[4], zo[5]}, {zo[2], zo[3]}, {zo[6], zo[7]}};
        float ds[4][2];
        float run = da_run;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float pre = run + (rg ? os[k] : 0.f);  // group 1's pair follows group 0's
          ds[k][0] = pre * zk[k][0] * (1.f - zk[k][0]);
          pre += dak[k][0];
          ds[k][1] = pre * zk[k][1] * (1.f - zk[k][1]);
          run += ps[k] + os[k];
        }
        da_run = run;
        // dS -> chunks 6, 7 of the P | dS rows (A operand of dq += dS K,
        // B operand of dK_gate^T); this completes the window's rows
#pragma unroll
        for (int k = 0; k < 4; ++k)
          sts32(sDS + sw128_offset(r, 6 + (k >> 1)) + 2 * (4 * (k & 1) + 2 * rg),
                E::pack(ds[k][0], ds[k][1]));
        fence_async_smem();
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bars[B_YB]);
      }
      return true;
    };

    // dq += R(-(carry + c0) theta) X for this group's 32 pairs (X carries the
    // ln 2 of the logits' base: the dQ launch scales Y by it)
    auto dq_update = [&](int w) -> bool {
      if (!wwait(bars[B_XF], w & 1, err, kErrX)) return false;
      tc_fence_after();
#pragma unroll
      for (int g0 = 0; g0 < PW / 8; g0 += 2) {  // 16 pairs (32 columns) per load round trip
        uint32_t xv[2][16], qv2[2][16];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          tmem_ld16(lane_base + tq::X + 2 * PW * rg + 16 * (g0 + i), xv[i]);
          tmem_ld16(lane_base + tq::DQ + 2 * PW * rg + 16 * (g0 + i), qv2[i]);
        }
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 2; ++i) {
#pragma unroll
          for (int e2 = 0; e2 < 8; ++e2) {
            const float2 cs = unpack_cs(csc[8 * (g0 + i) + e2]);  // cos, sin
            const float xe = __uint_as_float(xv[i][2 * e2]), xo = __uint_as_float(xv[i][2 * e2 + 1]);
            qv2[i][2 * e2] = __float_as_uint(
                fmaf(cs.y, xo, fmaf(cs.x, xe, __uint_as_float(qv2[i][2 * e2]))));
            qv2[i][2 * e2 + 1] = __float_as_uint(
                fmaf(-cs.y, xe, fmaf(cs.x, xo, __uint_as_float(qv2[i][2 * e2 + 1]))));
          }
          tmem_st16(lane_base + tq::DQ + 2 * PW * rg + 16 * (g0 + i), qv2[i]);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars[B_XFREE]);
      return true;
    };

    if (POFF) {
      // the Y columns of terms a key pair does not run are never written:
      // they must hold finite values (zeros) for the X GEMM, whose K^(m) rows
      // there are zero
      tc_fence_after();
#pragma unroll
      for (int m = NPT1; m < NPT0; ++m) tmem_st1(lane_base + tq::YT + 4 * m + 2 * rg + 1, 0u);
      tmem_wait_st();
    }
    if (ok) ok = gates(0);
    if (ok) {
      build_a();
      if (MODE == MODE_DQ) load_cs();
    }
    for (int w = 0; ok && w <= WL; ++w) {
      if (!(ok = halves(w))) break;
      // next window's A operand first, so its G GEMM overlaps the dQ update
      if (w < WL) {
        if (!(ok = gates(w + 1))) break;
        build_a();
      }
      if (MODE == MODE_DQ) {
        if (!(ok = dq_update(w))) break;
        if (w < WL) load_cs();
      }
    }
    if (MODE == MODE_DQ && ok) {
      // all GEMMs into DQ are done (the last window's B_XF was waited above)
      T* dqrow = reinterpret_cast<T*>(P.dq) + b * P.dqs[0] + h * P.dqs[1] +
                 (int64_t)(t - P.r0) * P.dqs[2];
#pragma unroll 1
      for (int c = 0; c < PW / 8; ++c) {
        uint32_t o[16];
        tmem_ld16(lane_base + tq::DQ + 2 * PW * rg + 16 * c, o);
        tmem_wait_ld();
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) pk[i] = E::pack(__uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1]));
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(dqrow + 2 * PW * rg + 16 * c);
          dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
    }
    __syncwarp();
    regs_dec<128>();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------------
// dK launch fed by the dQ launch's hand-off (dl of every (row, key), f16).
// Per window it recomputes the gate scores Q K^T on the tensor cores and, with
// the dQ launch's own arithmetic (window_gates, advance_prefix), the in-window
// positions u and the carry; rebuilds the A rows v = R((carry + c0) theta) q
// and Y_m = dl T_m(u); then runs
//   C^T = v^T Y  (each half; M = head dim, N = 16 terms x 8 keys, K = the 128
//                 query rows)
// on the tensor cores and the per-dimension combine with fp32 atomics into the
// dk accumulator.  dV and the gate part of dK come from the dQ launch.
//
// Roles (512 threads): warps 0-7 two row warpgroups (group g: pairs
// 32g..32g+31 of the A rows, keys 4g..4g+3 of each half); warp 8 TMA (Q once,
// the 16 keys of each window); warp 9 UMMA for C; warp 10 UMMA for the gate
// scores; warps 12-15 combine (one head dim per thread); registers re-split as
// in the dQ launch.  The A rows, the gate scores and the half-A C^T region are
// double-buffered over windows.
namespace k3 {
constexpr int Q = 0, AV = 32768;             // AV: 2 buffers of [NS][128][128 B]
constexpr int YA = AV + 2 * 32768;           // Y half A rows (16 terms x 8 keys)
constexpr int YB = YA + 32768;               // Y half B rows
constexpr int KT = YB + 32768;               // a window's keys: [2 stages][NS][16][128 B]
constexpr int COEF = KT + 2 * NS * 2048;
constexpr int TH = COEF + kMB * NPX * 4;
constexpr int BAR = TH + NPX * 4;
constexpr int SLOT = BAR + 24 * 8;
constexpr int TOTAL = SLOT + 16;
// RDY / YFREE per half: the rows write the next window's half A while the
// tensor core still reads half B of the current one
enum { B_Q = 0, B_RDY = 1, B_AVE = 3, B_YFREE = 5, B_CF = 7, B_CE = 9, B_DRAIN = 11,
       B_CE1 = 12, B_KF = 13, B_KE = 15, B_SF = 17, B_SE = 19, B_DRAIN2 = 21 };
// tensor memory: C^T of half A double-buffered (window parity b at 128 b), C^T
// of half B single (its GEMM waits until the combine has read it), the gate
// scores double-buffered
constexpr uint32_t C0 = 0, C1 = 256, SG = 384;
static_assert(SG + 32 <= 512, "tmem");
}  // namespace k3

template <typename T, int D, bool FIX>
__global__ void __launch_bounds__(kThreads, 1) dk3_kernel(const __grid_constant__ Params P) {
  using E = ElemTraits<T>;
  using namespace sm100;
  constexpr int NP = D / 2, DSL = D / 64, PW = NP / 2, KSTEPS = D / 16;
  constexpr int kM = kMB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + k3::BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + k3::SLOT);
  float* s_coef = reinterpret_cast<float*>(smem + k3::COEF);
  float* s_th = reinterpret_cast<float*>(smem + k3::TH);
  int* err = &g_corope_bwd_error;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qt = gridDim.x - 1 - blockIdx.x;
  const int bh = P.bh0 + blockIdx.y;
  const int h = bh % P.H, b = bh / P.H;
  const int hk = h / (P.H / P.Hkv);
  const int q0 = P.r0 + qt * kBM;  // sequence position of the tile's first row
  const int S = P.r0 + P.S;        // end of this launch's rows (sequence position)
  const int WL = min(S - 1, q0 + kBM - 1) / kW;

  if (tid == 0) {
    mbar_init(&bars[k3::B_Q], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[k3::B_RDY + i], 256);
      mbar_init(&bars[k3::B_YFREE + i], 1);
      mbar_init(&bars[k3::B_AVE + i], 1);
      mbar_init(&bars[k3::B_CF + i], 1);
      mbar_init(&bars[k3::B_CE + i], 128);
      mbar_init(&bars[k3::B_KF + i], 1);
      mbar_init(&bars[k3::B_KE + i], 1);
      mbar_init(&bars[k3::B_SF + i], 1);
      mbar_init(&bars[k3::B_SE + i], 256);
    }
    mbar_init(&bars[k3::B_DRAIN], 1);
    mbar_init(&bars[k3::B_DRAIN2], 1);
    mbar_init(&bars[k3::B_CE1], 128);
    fence_mbar_init();
  }
  for (int i = tid; i < kM * NPX; i += kThreads) s_coef[i] = P.coef[i / NPX][i % NPX];
  for (int p = tid; p < NP; p += kThreads) s_th[p] = theta_at(P.thetas, P.theta, p, D);
  if (DSL == 1) {  // D = 64: the second slab of both A buffers is zero
    for (int i = tid; i < 1024; i += kThreads) {
      reinterpret_cast<uint4*>(smem + k3::AV + 16384)[i] = make_uint4(0u, 0u, 0u, 0u);
      reinterpret_cast<uint4*>(smem + k3::AV + 32768 + 16384)[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    fence_async_smem();
  }
  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t sQ = smem_u32(smem + k3::Q), sAV = smem_u32(smem + k3::AV);
  const uint32_t sYA = smem_u32(smem + k3::YA), sYB = smem_u32(smem + k3::YB);
  const uint32_t sKT = smem_u32(smem + k3::KT);
  const uint32_t s_th_u = smem_u32(s_th);

  if (warp >= 8 && warp < 12) {
    regs_dec<kCtlRegs>();
    named_bar(1, kThreads);
    if (warp == 8 && lane == 0) {
      // ---------------------------------------------------------- TMA
      prefetch_tmap(&P.tm_q);
      prefetch_tmap(&P.tm_k);
      mbar_expect_tx(&bars[k3::B_Q], DSL * 16384);
      for (int s = 0; s < DSL; ++s)
        tma_load_4d(smem + k3::Q + s * 16384, &P.tm_q, &bars[k3::B_Q], 64 * s, q0 - P.r0, h, b);
      int last_use[2] = {-1, -1};
      for (int n = 0; n <= WL; ++n) {  // the keys of window n
        const int st = n & 1, u = n >> 1;
        if (n >= 2 && !mbar_wait(&bars[k3::B_KE + st], (u - 1) & 1, err, kErrKvEmpty)) break;
        mbar_expect_tx(&bars[k3::B_KF + st], DSL * 2048);
        for (int s = 0; s < DSL; ++s)
          tma_load_4d(smem + k3::KT + (st * NS + s) * 2048, &P.tm_k, &bars[k3::B_KF + st],
                      64 * s, kKT * n, hk, b);
        last_use[st] = u;
      }
      // no copy may still be in flight when the CTA exits
      mbar_wait(&bars[k3::B_Q], 0, err, kErrDrain);
      for (int st = 0; st < 2; ++st)
        if (last_use[st] >= 0) mbar_wait(&bars[k3::B_KF + st], last_use[st] & 1, err, kErrDrain);
    } else if (warp == 9 && lane == 0) {
      // ------------------------------------------------- UMMA: C^T = v^T Y
      // half A, then half B; K = the 128 query rows, 16 per step
      const uint32_t id_c = idesc_f16(128, 8 * kM, E::kBf16, true) | (1u << 15);  // A, B MN-major
      bool ok = true;
      for (int w = 0; ok && w <= WL; ++w) {
        const int bf = w & 1;
        const uint32_t av = sAV + 32768 * bf;
        for (int hh = 0; hh < 2 && ok; ++hh) {
          if (!(ok = mbar_wait(&bars[k3::B_RDY + hh], w & 1, err, kErrY))) break;
          if (hh == 0 && w >= 2 &&
              !(ok = mbar_wait(&bars[k3::B_CE + bf], ((w >> 1) - 1) & 1, err, kErrCEmpty)))
            break;
          if (hh == 1 && w >= 1 &&
              !(ok = mbar_wait(&bars[k3::B_CE1], (w - 1) & 1, err, kErrCEmpty)))
            break;
          tc_fence_after();
          const uint32_t yr = hh ? sYB : sYA;
          const uint32_t cacc = tmem + (hh ? k3::C1 : k3::C0 + 128 * bf);
#pragma unroll 1
          for (int s = 0; s < 8; ++s)
            mma_ss(cacc, sdesc_mnmajor(av + 2048 * s, 16384), sdesc_mnmajor(yr + 2048 * s, 16384),
                   id_c, s > 0);
          if (hh == 1) {
            mma_commit(&bars[k3::B_CF + bf]);
            mma_commit(&bars[k3::B_AVE + bf]);
          }
          mma_commit(&bars[k3::B_YFREE + hh]);
        }
      }
      mma_commit(&bars[k3::B_DRAIN]);
      mbar_wait(&bars[k3::B_DRAIN], 0, err, kErrDrain);
    } else if (warp == 10 && lane == 0) {
      // --------------------------------------- UMMA: gate scores Q K^T
      const uint32_t id_gate = idesc_f16(128, 16, E::kBf16, false);
      bool ok = mbar_wait(&bars[k3::B_Q], 0, err, kErrQ);
      for (int w = 0; ok && w <= WL; ++w) {
        const int st = w & 1;
        ok = mbar_wait(&bars[k3::B_KF + st], (w >> 1) & 1, err, kErrKvFull);
        if (ok && w >= 2) ok = mbar_wait(&bars[k3::B_SE + st], ((w >> 1) - 1) & 1, err, kErrSdEmpty);
        if (!ok) break;
        tc_fence_after();
        const uint32_t kt = sKT + st * NS * 2048;
#pragma unroll
        for (int s = 0; s < KSTEPS; ++s)
          mma_ss(tmem + k3::SG + 16 * st, sdesc_kmajor(sQ + (s >> 2) * 16384 + 32 * (s & 3)),
                 sdesc_kmajor(kt + (s >> 2) * 2048 + 32 * (s & 3)), id_gate, s > 0);
        mma_commit(&bars[k3::B_SF + st]);
        mma_commit(&bars[k3::B_KE + st]);
      }
      mma_commit(&bars[k3::B_DRAIN2]);
      mbar_wait(&bars[k3::B_DRAIN2], 0, err, kErrDrain);
    }
    __syncwarp();
    regs_inc<128>();
  } else if (warp >= 12) {
    // ------------------------------------------------------------ combine
    regs_dec<kBldRegs>();
    named_bar(1, kThreads);
    const int gt = tid - 384;  // head dim
    float cm[kM];
    {
      const int p = gt >> 1, e = gt & 1;
#pragma unroll
      for (int m = 0; m < kM; ++m) {
        float sgn;
        switch (m & 3) {
          case 0: sgn = 1.f; break;
          case 1: sgn = e ? 1.f : -1.f; break;
          case 2: sgn = -1.f; break;
          default: sgn = e ? -1.f : 1.f; break;
        }
        // the rows store V_m = s_m Y_m with s_m = -1 for m = 2, 3 mod 4 (their
        // packed recurrence needs no negation): the sign returns here
        if ((m & 3) >= 2) sgn = -sgn;
        cm[m] = kLn2 * s_coef[m * NPX + p] * sgn;  // zero for p >= D / 2
      }
    }
    const uint32_t lane_base = tmem + ((uint32_t)((warp - 12) * 32) << 16);
    const int bhk = b * P.Hkv + hk, BHkv = P.B * P.Hkv;
    for (int w = 0; w <= WL; ++w) {
      const int bf = w & 1;
      if (!wwait(bars[k3::B_CF + bf], (w >> 1) & 1, err, kErrC)) break;
      tc_fence_after();
      float dk[16];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const uint32_t creg = lane_base + (hh ? k3::C1 : k3::C0 + 128 * bf);
        // even terms use this lane's column of C^T; odd terms the partner
        // component's (d ^ 1), whose coefficient for this lane is minus the
        // partner's own: each lane sums its odd terms with -cm and the sums
        // are swapped once per key
        float ev[8], od[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) { ev[j] = 0.f; od[j] = 0.f; }
#pragma unroll
        for (int c0 = 0; c0 < kM / 2; c0 += 2) {  // terms 2c, 2c+1 for the 8 keys
          uint32_t g[2][16];
#pragma unroll
          for (int i = 0; i < 2; ++i)
            if (c0 + i < kM / 2) tmem_ld16(creg + 16 * (c0 + i), g[i]);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int c = c0 + i;
            if (c >= kM / 2) continue;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              ev[j] = fmaf(cm[2 * c], __uint_as_float(g[i][j]), ev[j]);
              od[j] = fmaf(-cm[2 * c + 1], __uint_as_float(g[i][8 + j]), od[j]);
            }
          }
        }
        if (hh == 1) {  // the single half-B region is free for the next window
          tc_fence_before();
          mbar_arrive(&bars[k3::B_CE1]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) dk[8 * hh + j] = ev[j] + __shfl_xor_sync(0xffffffffu, od[j], 1);
      }
      tc_fence_before();
      mbar_arrive(&bars[k3::B_CE + bf]);
      // a window's 16 keys lie in one accumulator chunk (chunks are multiples of 16 keys);
      // dk[8 hh + s] belongs to slot s of half hh
      const int64_t row0 = accum_row(w * kW, bhk, BHkv, P.Sk, P.acc_chunk) * D + gt;
      constexpr bool fixed = FIX;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int key = bwd_slot_key(j >> 3, j & 7);
        if (w * kW + key < P.Sk && gt < D) acc_add(P.dk32, row0 + key * D, dk[j], fixed);
      }
    }
    __syncwarp();
    regs_inc<128>();
  } else {
    // ------------------------------------------------------------ row warps
    regs_inc<kRowRegs>();
    named_bar(1, kThreads);
    const int rg = warp >> 2;
    const int r = tid & 127;
    const int t = q0 + r;
    const bool row_ok = t < S;
    auto diag_window = [&](int w) { return w * kW + kW - 1 > q0 || q0 + kBM > S; };
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const int64_t ri = ((int64_t)b * P.H + h) * P.S + min(t - P.r0, P.S - 1);
    const float A_t = P.a[ri];
    const uint8_t* hb0 =
        P.handoff + ((int64_t)blockIdx.y * P.blocks_bh + chunk_block0(P.r0, qt)) * kHB;
    // dl of this group's 4 keys of each half of window w (f16 pairs)
    auto load = [&](int w, uint2 (&x)[2]) {
      const uint8_t* hb = hb0 + (int64_t)w * kHB;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) x[hh] = ldg64_nc(hb + ((2 * hh + rg) * 128 + r) * 8);
    };
    const float th_max = theta_max(s_th, NP);
    float base = 0.f, base_c = 0.f;  // compensated gate prefix (advance_prefix)
    bool ok = wwait(bars[k3::B_Q], 0, err, kErrQ);
    uint2 cur[2], nxt[2];
    load(0, cur);
    for (int w = 0; ok && w <= WL; ++w) {
      if (w < WL) load(w + 1, nxt);
      // ---- gates and positions of window w (the dQ launch's arithmetic)
      const int st = w & 1;
      if (!(ok = wwait(bars[k3::B_SF + st], (w >> 1) & 1, err, kErrSd))) break;
      tc_fence_after();
      float uo[8];
      float carry;
      {
        uint32_t sraw[16];
        tmem_ld16(lane_base + k3::SG + 16 * st, sraw);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&bars[k3::B_SE + st]);
        float z[16], uu[16];
        const float zsum = diag_window(w) ? window_gates<true>(sraw, w * kW, t, row_ok, z, uu)
                                          : window_gates<false>(sraw, w * kW, t, row_ok, z, uu);
        carry = advance_prefix(zsum, A_t, base, base_c);
#pragma unroll
        for (int i = 0; i < 8; ++i) {  // slot 4 rg + (i & 3) of half i >> 2
          const int k0 = bwd_slot_key(i >> 2, i & 3);
          uo[i] = rg ? uu[k0 + 2] : uu[k0];
        }
      }
      // ---- A rows of this group's slab into buffer w & 1
      if (w >= 2 &&
          !(ok = wwait(bars[k3::B_AVE + (w & 1)], ((w >> 1) - 1) & 1, err, kErrAvEmpty)))
        break;
      {
        const float bse = carry + kC0;
        const bool mufu_reduce = __all_sync(0xffffffffu, bse * th_max < kMufuReduceMax);
        const uint32_t av = sAV + 32768 * (w & 1);
#pragma unroll 1
        for (int g = 0; g < PW / 16; ++g) {
          uint4 qv[4];
          float th[16];
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const int c = rg * (PW / 4) + 4 * g + cc;  // chunk of the row (4 pairs)
            qv[cc] = lds128(sQ + (c >> 3) * 16384 + sw128_offset(r, c & 7));
            const float4 t4 = lds128f(s_th_u + 16 * c);
            th[4 * cc] = t4.x; th[4 * cc + 1] = t4.y; th[4 * cc + 2] = t4.z; th[4 * cc + 3] = t4.w;
          }
          float rr[16], sn[16], cs[16];
          if (mufu_reduce) {
#pragma unroll
            for (int i = 0; i < 16; ++i) rr[i] = bse * th[i];
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) rr[i] = reduce_2pi(bse * th[i]);
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) __sincosf(rr[i], &sn[i], &cs[i]);
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const uint32_t in[4] = {qv[cc].x, qv[cc].y, qv[cc].z, qv[cc].w};
            uint32_t o[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float qe = E::lo(in[i]), qo = E::hi(in[i]);
              const float s_ = sn[4 * cc + i], c_ = cs[4 * cc + i];
              o[i] = E::pack(qe * c_ - qo * s_, qe * s_ + qo * c_);
            }
            const int c = rg * (PW / 4) + 4 * g + cc;
            sts128(av + (c >> 3) * 16384 + sw128_offset(r, c & 7), make_uint4(o[0], o[1], o[2], o[3]));
          }
        }
      }
      // ---- Y_A, then Y_B, each once the previous window's GEMM of that half
      // is done with its rows
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        if (w >= 1 && !(ok = wwait(bars[k3::B_YFREE + hh], (w - 1) & 1, err, kErrY))) break;
        const uint32_t yrow = hh ? sYB : sYA;
        const float2 d01 = unpack_dl(cur[hh].x), d23 = unpack_dl(cur[hh].y);
        const float dl[4] = {d01.x, d01.y, d23.x, d23.y};
        const float uj[4] = {uo[4 * hh], uo[4 * hh + 1], uo[4 * hh + 2], uo[4 * hh + 3]};
        uint32_t y[kM][2];
#pragma unroll
        for (int jp = 0; jp < 2; ++jp) {
          // Y_m = dl T_m(u) obeys the Chebyshev recurrence itself,
          // Y_{m+1} = 2u Y_m - Y_{m-1} (Y_0 = dl, Y_1 = dl u).  Tracked with the
          // signs s_m = (+, +, -, -, ...), V_m = s_m Y_m obeys
          // V_m = (-1)^(m+1) 2u V_{m-1} + V_{m-2}: one packed FMA per step for
          // the pair's two keys, no negated operand (the combine restores s_m)
          const float2 u2 = make_float2(2.f * uj[2 * jp], 2.f * uj[2 * jp + 1]);
          const float2 nu2 = make_float2(-2.f * uj[2 * jp], -2.f * uj[2 * jp + 1]);
          float2 v0 = make_float2(dl[2 * jp], dl[2 * jp + 1]);
          float2 v1 = make_float2(v0.x * uj[2 * jp], v0.y * uj[2 * jp + 1]);
          y[0][jp] = E::pack(v0.x, v0.y);
          y[1][jp] = E::pack(v1.x, v1.y);
#pragma unroll
          for (int m = 2; m < kM; ++m) {
            const float2 v2 = __ffma2_rn((m & 1) ? u2 : nu2, v1, v0);
            v0 = v1;
            v1 = v2;
            y[m][jp] = E::pack(v2.x, v2.y);
          }
        }
#pragma unroll
        for (int m = 0; m < kM; ++m)  // element 8 m + key: chunk m of the row
          sts64(yrow + (m >> 3) * 16384 + sw128_offset(r, m & 7) + 8 * rg, y[m][0], y[m][1]);
        fence_async_smem();
        mbar_arrive(&bars[k3::B_RDY + hh]);
      }
      if (!ok) break;
      cur[0] = nxt[0];
      cur[1] = nxt[1];
    }
    __syncwarp();
    regs_dec<128>();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------------ host
// K^(m) buffer layout and count; returns the dynamic shared memory needed
template <int MODE, int KM>
static int plan(Params& p) {
  using L = SmemTail<MODE, KM>;
  int off = 0, rows = 0;
  for (int s = 0; s < NS; ++s) {
    p.b_slab_off[s] = off;
    off += p.nrow[4 * s] * 128;
  }
  for (int s = 0; s < 8; ++s) rows += p.nrow[s];  // zero beyond the head dim's K steps
  p.max_items = (2 * rows + 127) / 128;  // (term x key row, 8-element chunk) items per builder
  p.bop = (L::ITEMS + p.max_items * 128 * 8 + 1023) & ~1023;
  p.b_buf_bytes = (off + 1023) & ~1023;
  p.nb = (p.bop + 4 * p.b_buf_bytes + 1024 <= kSmemLimit) ? 2 : 1;
  return p.bop + 2 * p.nb * p.b_buf_bytes + 1024;
}

template <typename T, int D, int MODE, bool HAS_BIAS, int KM, bool KMT>
static cudaError_t launch_k(const Params& p, int smem, dim3 grid, cudaStream_t st) {
  auto kern = p.fixed ? bwd_kernel<T, D, MODE, HAS_BIAS, KM, KMT, true>
                      : bwd_kernel<T, D, MODE, HAS_BIAS, KM, KMT, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kSmemLimit);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, smem, st>>>(p);
  return cudaGetLastError();
}

template <typename T, int D, int MODE>
static cudaError_t launch_mode(Params& p, bool bias, int S, int nbh, cudaStream_t st,
                               float theta, float sm_scale) {
  constexpr int KM = kMB;
  tcx::fill_coefficients<KM>(p.coef, p.nrow, D, theta, sm_scale);
  if (MODE == MODE_DQ)  // the per-offset expansions' K extents
    tcx::fill_offset_rows<KM>(p.nrow, D, theta);
  const int smem = plan<MODE, KM>(p);
  if (smem > kSmemLimit) return cudaErrorInvalidValue;
  dim3 grid((S + kBM - 1) / kBM, nbh);
  if (MODE == MODE_DQ && p.km_nhw > 0)  // panels were written for this call
    return bias ? launch_k<T, D, MODE, true, KM, MODE == MODE_DQ>(p, smem, grid, st)
                : launch_k<T, D, MODE, false, KM, MODE == MODE_DQ>(p, smem, grid, st);
  return bias ? launch_k<T, D, MODE, true, KM, false>(p, smem, grid, st)
              : launch_k<T, D, MODE, false, KM, false>(p, smem, grid, st);
}

template <typename T, int D>
static cudaError_t launch_dk3(Params& p, int S, int nbh, cudaStream_t st, float theta,
                              float sm_scale) {
  tcx::fill_coefficients<kMB>(p.coef, p.nrow, D, theta, sm_scale);
  const int smem = k3::TOTAL + 1024;
  dim3 grid((S + kBM - 1) / kBM, nbh);
  auto kern = p.fixed ? dk3_kernel<T, D, true> : dk3_kernel<T, D, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, smem, st>>>(p);
  return cudaGetLastError();
}

// Fewest (b, h) slices per launch of the hand-off pair: 16, or fewer when
// they already make 512 CTAs (about 3.5 waves of 148 SMs; long sequences),
// or all of them.
static int min_slices(int BH, int S) {
  const int qtiles = (S + kBM - 1) / kBM;
  return std::min(std::min(BH, 16), (512 + qtiles - 1) / qtiles);
}

// hand-off blocks of one (b, h): one per (query tile, window)
static int64_t blocks_per_bh(int S, int r0 = 0) {
  int64_t n = 0;
  for (int qt = 0; qt * kBM < S; ++qt) n += (r0 + min(S - 1, qt * kBM + kBM - 1)) / kW + 1;
  return n;
}

template <typename T> constexpr int E_dtype() {
  return ElemTraits<T>::kBf16 ? COROPE_DTYPE_BF16 : COROPE_DTYPE_F16;
}

// Write the dQ launch's K^(m) panels (all Sk keys, the 16-term backward's
// per-offset expansions in its key order) into `panels` and point the
// tensor maps at them.
template <typename T, int D>
static cudaError_t make_panels(Params& p, const BwdArgs& a, void* panels, cudaStream_t st) {
  static tcx::OffsetPanelArgs pa;  // guarded by the caller's lock
  tcx::offset_panel_bytes<kMB>(a.B, a.Hkv, a.Sk, D, a.theta, a.sm_scale, &pa, true, false);
  const int64_t np = tcx::panel_count(a.B, a.Hkv, a.Sk);
  pa.k = a.k;
  for (int i = 0; i < 3; ++i) pa.ks[i] = a.ks[i];
  pa.out[0] = panels;
  pa.out[1] = static_cast<uint8_t*>(panels) + np * pa.rows[0] * 128;
  pa.cf = a.coef;  // written by tc_bwd_launch
  for (int s = 0; s < D / 64; ++s)
    if (!tcx::encode_panels(&p.tm_km[s], pa.out[s], E_dtype<T>(), pa.rows[s], np))
      return cudaErrorInvalidValue;
  p.km_nhw = pa.nhw;
  p.km_rows[0] = pa.rows[0];
  p.km_rows[1] = pa.rows[1];
  tcx::offset_panel_kernel<T, D>
      <<<dim3(tcx::panel_halfwindows_read(a.Sk, a.r0, a.S), a.B * a.Hkv), 128, 0, st>>>(pa);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t launch_all(Params& p, const BwdArgs& a, bool bias, int BH, int S,
                              uint8_t* handoff, size_t handoff_bytes, void* panels,
                              cudaStream_t st, float theta, float sm_scale) {
  if (panels) {
    cudaError_t e = make_panels<T, D>(p, a, panels, st);
    if (e != cudaSuccess) return e;
  }
  const int64_t per_bh = blocks_per_bh(S, p.r0) * kHB;
  int chunk = handoff ? (int)std::min<int64_t>(BH, (int64_t)(handoff_bytes / per_bh)) : 0;
  if (chunk < min_slices(BH, S)) chunk = 0;  // too few CTAs per launch: recompute instead
  cudaError_t e = cudaSuccess;
  if (chunk == 0) {
    p.handoff = nullptr;
    p.bh0 = 0;
    e = launch_mode<T, D, MODE_DQ>(p, bias, S, BH, st, theta, sm_scale);
    if (e == cudaSuccess) e = launch_mode<T, D, MODE_DK>(p, bias, S, BH, st, theta, sm_scale);
    return e;
  }
  p.handoff = handoff;
  p.blocks_bh = blocks_per_bh(S, p.r0);
  for (int bh0 = 0; bh0 < BH && e == cudaSuccess; bh0 += chunk) {
    p.bh0 = bh0;
    const int nbh = std::min(chunk, BH - bh0);
    e = launch_mode<T, D, MODE_DQ>(p, bias, S, nbh, st, theta, sm_scale);
    if (e == cudaSuccess) e = launch_dk3<T, D>(p, S, nbh, st, theta, sm_scale);
  }
  return e;
}

}  // namespace tcb

int64_t tc_bwd_handoff_bytes_per_bh(int S, int r0) { return tcb::blocks_per_bh(S, r0) * tcb::kHB; }

static bool rows16(const void* ptr, const int64_t* st) {
  return (reinterpret_cast<uintptr_t>(ptr) % 16) == 0 && (st[0] * 2) % 16 == 0 &&
         (st[1] * 2) % 16 == 0 && (st[2] * 2) % 16 == 0;
}

bool tc_bwd_supported(const BwdArgs& a, int dtype) {
  if (dtype != COROPE_DTYPE_BF16 && dtype != COROPE_DTYPE_F16) return false;
  // the expansions' term counts assume every frequency theta_p <= 1
  if (!(a.theta >= 1.f)) return false;
  if (a.D != 64 && a.D != 128) return false;
  if (!rows16(a.q, a.qs) || !rows16(a.k, a.ks) || !rows16(a.v, a.vs) ||
      !rows16(a.dout, a.dos) || !rows16(a.dq, a.dqs))
    return false;
  // small theta keeps more Chebyshev terms: the K^(m) buffers must still fit
  using namespace tcb;
  Params p;
  tcx::fill_coefficients<kMB>(p.coef, p.nrow, a.D, a.theta, a.sm_scale);
  if (plan<MODE_DQ, kMB>(p) > tcx::kSmemLimit) return false;
  if (plan<MODE_DK, kMB>(p) > tcx::kSmemLimit) return false;
  return tcx::get_encoder() != nullptr;
}

// Launches the dQ and dK kernels; the caller runs the delta/lse pre-kernel
// before and the fp32 -> dtype conversion of dk/dv after.  With a hand-off
// region large enough for min_slices (b, h) slices the dK launch reads the
// dQ launch's per-pair results (slice by slice through the region); otherwise
// it recomputes them.
size_t tc_bwd_panel_bytes(const BwdArgs& a) {
  return tcx::offset_panel_bytes<tcb::kMB>(a.B, a.Hkv, a.Sk, a.D, a.theta, a.sm_scale, nullptr,
                                           true, false);
}

size_t tc_bwd_coef_bytes() { return tcx::kOffsetCoefBytes;
}

cudaError_t tc_bwd_launch(const BwdArgs& a, int dtype, cudaStream_t st, void* handoff,
                          size_t handoff_bytes, void* panels) {
  using namespace tcb;
  static Params p;
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  std::memset(&p, 0, sizeof(p));
  if (!tcx::encode(&p.tm_q, a.q, dtype, a.B, a.H, a.S, a.D, a.qs, kBM) ||
      !tcx::encode(&p.tm_do, a.dout, dtype, a.B, a.H, a.S, a.D, a.dos, kBM) ||
      !tcx::encode(&p.tm_k, a.k, dtype, a.B, a.Hkv, a.Sk, a.D, a.ks, kKT) ||
      !tcx::encode(&p.tm_v, a.v, dtype, a.B, a.Hkv, a.Sk, a.D, a.vs, kKT))
    return cudaErrorInvalidValue;
  if (!a.coef) return cudaErrorInvalidValue;  // the dQ kernel's coefficients (minimum workspace)
  {
    tcx::OffsetPanelArgs ca;
    tcx::offset_panel_bytes<kMB>(a.B, a.Hkv, a.Sk, a.D, a.theta, a.sm_scale, &ca, true, false);
    ca.cf = a.coef;
    ca.signs = 1;  // the dQ kernel's rows run the signed basis s_m T_m
    tcx::offset_coef_kernel<<<16, 64, 0, st>>>(ca);
  }
  p.cf = a.coef;
  p.r0 = a.r0;
  p.Sk = a.Sk;
  p.dq = a.dq;
  p.dk32 = a.dk32;
  p.dv32 = a.dv32;
  p.fixed = a.fixed;
  p.acc_chunk = a.acc_chunk;
  p.lse = a.lse;
  p.delta = a.delta;
  p.a = a.a;
  p.thetas = a.thetas;
  p.theta = a.theta;
  p.bias = a.bias;
  p.bias_rs = a.bias_rs;
  for (int i = 0; i < 3; ++i) p.dqs[i] = a.dqs[i];
  p.B = a.B; p.H = a.H; p.Hkv = a.Hkv; p.S = a.S;
  const bool bias = a.bias != nullptr;
  uint8_t* hp = static_cast<uint8_t*>(handoff);
  const int BH = a.B * a.H;
  if (dtype == COROPE_DTYPE_BF16)
    return a.D == 64 ? launch_all<__nv_bfloat16, 64>(p, a, bias, BH, a.S, hp, handoff_bytes,
                                                      panels, st, a.theta, a.sm_scale)
                     : launch_all<__nv_bfloat16, 128>(p, a, bias, BH, a.S, hp, handoff_bytes,
                                                       panels, st, a.theta, a.sm_scale);
  return a.D == 64 ? launch_all<__half, 64>(p, a, bias, BH, a.S, hp, handoff_bytes, panels, st,
                                            a.theta, a.sm_scale)
                   : launch_all<__half, 128>(p, a, bias, BH, a.S, hp, handoff_bytes, panels, st,
                                             a.theta, a.sm_scale);
}

}  // namespace corope
