// Tensor-core (tcgen05) CoRoPE forward for sm_100a.
//
// The rotated logit sm * <R(a_tj theta) q_t, k_j> is not a GEMM: the angle
// depends on the (query, key) pair through the contextual position a_tj.
// Keys are processed in windows of W = 16 from the diagonal down.  Inside a
// window the position splits as a_tj = C_t + c0 + c0 * u_tj, where C_t is the
// gate sum of the keys after the window (a per-row carry), c0 = (W-1)/2 and
// u_tj in [-1, 1] is the scaled in-window position.  The rotation by
// (C_t + c0) theta is applied to q_t once per row and window (the A operand
// "v", kept in tensor memory), and the in-window rotation is expanded in
// Chebyshev polynomials (Jacobi-Anger):
//     exp(-i w u) = sum_m eps_m (-i)^m J_m(w) T_m(u),   w = c0 * theta_p,
// so that  logit_tj = sum_m T_m(u_tj) G_m(t, j)  with
//     G_m = v . K^(m),   K^(m)_p(j) = eps_m (-i)^m J_m(c0 theta_p) K_p(j),
// one tensor-core GEMM per window (all m stacked along N).  Fourteen terms
// keep the expansion error below 1.1e-3 at the highest frequency (w = 7.5)
// and far below it elsewhere -- under the rounding of the 16-bit GEMM
// operands; coefficients below 2e-6 are pruned, which shortens the K extent
// of the high-m terms.  With the scaled-key panels each key offset of the
// window has its own expansion (tcx::offset_terms): key o only spans
// positions C_t .. C_t + 15 - o, so later keys need fewer terms (79 instead
// of 112 Clenshaw steps per row thread and window).
//
// Roles per CTA (128 query rows of one (b, h), 512 threads):
//   warps 0-7  two row warpgroups sharing every row (group g: keys 4g..4g+3
//              of each 8-key half, rotation pairs g*D/4 .. and output
//              columns g*D/2 ..): gates, carries, A operand, Chebyshev
//              (Clenshaw) combine, online softmax (stale-max rescaling; the
//              groups agree on each window's row max through shared memory),
//              P, epilogue (row sums combined at the end)
//   warp 8     TMA: Q once, K/V tiles of 64 keys (2 stages)
//   warp 9     UMMA issue of the G GEMM (A operand from tensor memory)
//   warp 10    UMMA issue of the gate GEMM Q K^T and of P V
//   warps 12-15 without panels: build the K^(m) operand of each window in
//              shared memory (double-buffered when it fits); with panels
//              (warp 11 then TMA-loads them): the window's gates, in-window
//              positions and carry, one thread per row, handed to both row
//              groups through shared memory
// Registers are re-balanced with setmaxnreg (rows 176, builders 104, the
// TMA/UMMA warpgroup 56), then a CTA barrier so that no warp returns
// registers to the pool before every warp holds its share.
#include <cmath>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"
#include "tc_common.cuh"

namespace corope {

// First error recorded by a bounded wait of a tensor-core kernel (0: none).
__device__ int g_corope_device_error = 0;

// Read and clear the device error word (synchronises with the device).
int tc_take_device_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_corope_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_corope_device_error, &zero, sizeof(int));
  }
  return v;
}

namespace tc {

using tcx::kW;
using tcx::kM;
constexpr int kBM = 128;     // query rows per CTA
constexpr int kKT = 64;      // keys per K/V tile
constexpr int kThreads = 512;
constexpr int kRowRegs = 176, kBldRegs = 104, kCtlRegs = 56;
static_assert(2 * kRowRegs + kBldRegs + kCtlRegs == 4 * 128, "register split");
using tcx::kC0;
using tcx::kLog2e;
constexpr float kRescale = 8.0f;  // stale-max headroom (log2 units)

// error codes recorded by bounded waits
enum : int {
  kErrQ = 101, kErrKvEmpty, kErrKvFull, kErrSg, kErrG, kErrGEmpty, kErrB, kErrBEmpty, kErrAv,
  kErrP, kErrO, kErrDrain, kErrX
};

struct Params {
  CUtensorMap tm_q, tm_k, tm_v;
  CUtensorMap tm_km[2];  // precomputed K^(m) panels per slab (KMT launches)
  int km_nhw;            // half windows per (b, kv head) in the panels
  int km_rows[2];        // panel rows per slab
  void* o;
  float *m, *l, *a, *lse;
  const float* thetas;
  const float* bias;
  int64_t bias_rs;
  int64_t os[3];
  int B, H, Hkv, S;
  int r0;  // sequence position of row 0 of q / o (a multiple of kBM)
  float theta;
  int nrow[8];          // B-operand rows read by K-step s (multiple of 16, or 0)
  int nb;               // K^(m) buffers per half window (1 or 2)
  int b_slab_off[2];    // byte offset of each 64-element slab in a buffer
  int b_buf_bytes;      // bytes of one buffer (multiple of 1024)
  float coef[kM][64];   // eps_m J_m(c0 theta_p) * sm_scale * log2(e)
};

template <int D>
struct Layout {
  static constexpr int NS = D / 64;  // 64-element (128-byte) slabs
  static constexpr int Q = 0;
  static constexpr int K = Q + NS * 16384;      // [2 stages][NS][64 rows][128 B]
  static constexpr int V = K + 2 * NS * 8192;
  static constexpr int COEF = V + 2 * NS * 8192;
  static constexpr int TH = COEF + kM * (D / 2) * 4;
  static constexpr int BAR = TH + (D / 2) * 4;
  static constexpr int NBAR = 32;
  static constexpr int SLOT = BAR + NBAR * 8;
  // row-group exchange: [2 groups][128 rows] row max, then [2][128] row sums
  static constexpr int XCH = (SLOT + 16 + 15) & ~15;
  // builder work items: [kMaxItems][128 threads] x (uint2); launches with
  // panels use the region for the gate hand-off of warps 12-15 instead:
  // u [2 buffers][2 row groups][2 chunks][128 rows] x float4, then the
  // A-operand carry [2 buffers][128 rows] x float
  static constexpr int MAX_ITEMS = (2 * 8 * 8 * kM + 127) / 128;
  static constexpr int ITEMS = XCH + 4 * 128 * 4;
  static constexpr int GU = ITEMS;
  static constexpr int GC = GU + 2 * 2 * 2 * 128 * 16;
  static constexpr int REGION = MAX_ITEMS * 128 * 8 > GC + 2 * 128 * 4 - ITEMS
                                    ? MAX_ITEMS * 128 * 8 : GC + 2 * 128 * 4 - ITEMS;
  // K^(m) buffers [2 halves][nb][b_buf_bytes] follow, 1024-aligned
  static constexpr int BOP = (ITEMS + REGION + 1023) & ~1023;
  // tensor-memory columns
  static constexpr uint32_t GW = 8 * kM;  // columns of one G half
  static constexpr uint32_t T_O = 0;
  static constexpr uint32_t T_G0 = D;
  static constexpr uint32_t T_G1 = D + GW;
  static constexpr uint32_t T_SG0 = D + 2 * GW;
  static constexpr uint32_t T_SG1 = T_SG0 + 16;
  static constexpr uint32_t T_AV0 = T_SG1 + 16;   // A operand, two buffers
  static constexpr uint32_t T_AV1 = T_AV0 + D / 2;
  static_assert(T_AV1 + D / 2 <= 512, "tensor memory overflow");
};

using tcx::kSmemLimit;

// barrier indices
enum {
  B_Q = 0, B_KVF = 1, B_KVE = 3, B_SG = 5, B_GF = 7, B_GE = 9,
  B_BF = 11,  // [half][buffer] -> B_BF + 2 * half + buffer
  B_BE = 15,  // [half][buffer]
  B_AV = 19, B_P = 20, B_O = 21, B_DRAIN = 22, B_DRAIN2 = 23,
  B_XM = 24, B_XL = 25,  // row-group exchanges: window row max, final row sums
  B_GT = 26              // [buffer]: gates of a window ready (panel launches)
};

using tcx::ElemTraits;
using tcx::sigmoid_f;
using tcx::slot_key;
using tcx::angles16;
using tcx::rotate16;

// Gates of one window for row t (keys j0 .. j0 + 15, descending): the
// in-window positions uu[jj] = (gate sum of the window's keys after jj) / c0
// - 1, and the window's gate sum (returned).  Keys past t have gate 0.
// PER_OFFSET (panel launches): positions scaled by each key offset's own
// half-width, uu[jj] = acc / c_jj - 1.
template <bool PER_OFFSET>
__device__ __forceinline__ float fwd_window_gates(const uint32_t (&sraw)[16], int j0, int t,
                                                  float (&uu)[16]) {
  float acc = 0.f;
#pragma unroll
  for (int jj = 15; jj >= 0; --jj) {
    const float z = (j0 + jj <= t) ? sigmoid_f(__uint_as_float(sraw[jj])) : 0.f;
    uu[jj] = fmaf(acc, PER_OFFSET ? tcx::offset_inv_halfwidth(kM, jj) : 1.0f / kC0, -1.0f);
    acc += z;
  }
  return acc;
}

// KMT: the K^(m) operands come from precomputed panels in global memory
// (tcx::panel_kernel) by TMA, one copy per slab and half window, instead of
// being built from the K tiles by warps 12-15.
template <typename T, int D, bool HAS_BIAS, bool KMT>
__global__ void __launch_bounds__(kThreads, 1) fwd_kernel(const __grid_constant__ Params P) {
  using L = Layout<D>;
  using E = ElemTraits<T>;
  using namespace sm100;
  constexpr int NS = L::NS;
  constexpr int NP = D / 2;
  constexpr int KSTEPS = D / 16;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + L::SLOT);
  float* s_coef = reinterpret_cast<float*>(smem + L::COEF);
  float* s_th = reinterpret_cast<float*>(smem + L::TH);
  int* err = &g_corope_device_error;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qt = gridDim.x - 1 - blockIdx.x;  // longest query tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (P.H / P.Hkv);
  const int q0 = P.r0 + qt * kBM;  // sequence position of the tile's first row
  const int S = P.r0 + P.S;        // end of this launch's rows (sequence position)
  const int W0 = min(S - 1, q0 + kBM - 1) / kW;  // highest window
  const int T0 = W0 / 4;                         // highest K/V tile

  if (tid == 0) {
    mbar_init(&bars[B_Q], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[B_KVF + i], 1);
      mbar_init(&bars[B_KVE + i], KMT ? 1 : 1 + 128);
      mbar_init(&bars[B_SG + i], 1);
      mbar_init(&bars[B_GF + i], 1);
      mbar_init(&bars[B_GE + i], 256);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&bars[B_BF + i], KMT ? 1 : 128);
      mbar_init(&bars[B_BE + i], 1);
    }
    mbar_init(&bars[B_AV], 256);
    mbar_init(&bars[B_P], 256);
    mbar_init(&bars[B_XM], 256);
    mbar_init(&bars[B_XL], 256);
    mbar_init(&bars[B_GT], 128);
    mbar_init(&bars[B_GT + 1], 128);
    mbar_init(&bars[B_O], 1);
    mbar_init(&bars[B_DRAIN], 1);
    mbar_init(&bars[B_DRAIN2], 1);
    fence_mbar_init();
  }
  for (int i = tid; i < kM * NP; i += kThreads) s_coef[i] = P.coef[i / NP][i % NP];
  for (int p = tid; p < NP; p += kThreads) s_th[p] = theta_at(P.thetas, P.theta, p, D);
  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t sQ = smem_u32(smem + L::Q);
  const uint32_t sK = smem_u32(smem + L::K);
  const uint32_t sV = smem_u32(smem + L::V);
  const uint32_t sB = smem_u32(smem + L::BOP);
  const uint32_t s_th_u = smem_u32(s_th);
  const uint32_t s_coef_u = smem_u32(s_coef);
  const int nb = P.nb;

  if (warp >= 8 && warp < 12) {
    regs_dec<kCtlRegs>();
    named_bar(1, kThreads);
    if (warp == 8) {
      // ------------------------------------------------------------ TMA
      if (lane == 0) {
        prefetch_tmap(&P.tm_q);
        prefetch_tmap(&P.tm_k);
        prefetch_tmap(&P.tm_v);
        mbar_expect_tx(&bars[B_Q], NS * 16384);
        for (int s = 0; s < NS; ++s)
          tma_load_4d(smem + L::Q + s * 16384, &P.tm_q, &bars[B_Q], 64 * s, q0 - P.r0, h, b);
        int last_use[2] = {-1, -1};
        for (int n = 0; T0 - n >= 0; ++n) {
          const int tile = T0 - n, st = n & 1, u = n >> 1;
          if (n >= 2 && !mbar_wait(&bars[B_KVE + st], (u - 1) & 1, err, kErrKvEmpty)) break;
          mbar_expect_tx(&bars[B_KVF + st], 2 * NS * 8192);
          for (int s = 0; s < NS; ++s) {
            tma_load_4d(smem + L::K + (st * NS + s) * 8192, &P.tm_k, &bars[B_KVF + st], 64 * s,
                        kKT * tile, hk, b);
            tma_load_4d(smem + L::V + (st * NS + s) * 8192, &P.tm_v, &bars[B_KVF + st], 64 * s,
                        kKT * tile, hk, b);
          }
          last_use[st] = u;
        }
        // no copy may still be in flight when the CTA exits
        for (int st = 0; st < 2; ++st)
          if (last_use[st] >= 0) mbar_wait(&bars[B_KVF + st], last_use[st] & 1, err, kErrDrain);
      }
    } else if (warp == 9) {
      // ------------------------------------------------------ UMMA: G GEMM
      if (lane == 0) {
        bool ok = true;
        for (int w = W0; ok && w >= 0; --w) {
          const int k = W0 - w, buf = k % nb, use = k / nb;
          if (!(ok = mbar_wait(&bars[B_AV], k & 1, err, kErrAv))) break;
          for (int hh = 0; hh < 2 && ok; ++hh) {
            ok = mbar_wait(&bars[B_BF + 2 * hh + buf], use & 1, err, kErrB);
            if (ok && k > 0) ok = mbar_wait(&bars[B_GE + hh], (k - 1) & 1, err, kErrGEmpty);
            if (!ok) break;
            tc_fence_after();
            const uint32_t dst = tmem + (hh ? L::T_G1 : L::T_G0);
            const uint32_t bb = sB + (hh * nb + buf) * P.b_buf_bytes;
  #pragma unroll
            for (int s = 0; s < KSTEPS; ++s) {
              const int nr = P.nrow[s];
              if (nr == 0) break;
              mma_ts(dst, tmem + ((w & 1) ? L::T_AV1 : L::T_AV0) + 8 * s,
                     sdesc_kmajor(bb + P.b_slab_off[s >> 2] + 32 * (s & 3)),
                     idesc_f16(128, nr, E::kBf16, false), s > 0);
            }
            mma_commit(&bars[B_GF + hh]);
            mma_commit(&bars[B_BE + 2 * hh + buf]);
          }
        }
        mma_commit(&bars[B_DRAIN]);
        mbar_wait(&bars[B_DRAIN], 0, err, kErrDrain);
      }
    } else if (warp == 10) {
      // ------------------------------------------- UMMA: gate GEMM and P V
      if (lane == 0) {
        const uint32_t id_gate = idesc_f16(128, 16, E::kBf16, false);
        const uint32_t id_pv = idesc_f16(128, D, E::kBf16, true);
        bool ok = mbar_wait(&bars[B_Q], 0, err, kErrQ);
        tc_fence_after();
        auto gate = [&](int w) -> bool {
          const int n = T0 - w / 4, st = n & 1;
          if (!mbar_wait(&bars[B_KVF + st], (n >> 1) & 1, err, kErrKvFull)) return false;
          tc_fence_after();
          const uint32_t kt = sK + st * NS * 8192 + (w & 3) * kW * 128;
          const uint32_t dst = tmem + ((w & 1) ? L::T_SG1 : L::T_SG0);
  #pragma unroll
          for (int s = 0; s < KSTEPS; ++s)
            mma_ss(dst, sdesc_kmajor(sQ + (s >> 2) * 16384 + 32 * (s & 3)),
                   sdesc_kmajor(kt + (s >> 2) * 8192 + 32 * (s & 3)), id_gate, s > 0);
          mma_commit(&bars[B_SG + (w & 1)]);
          return true;
        };
        if (ok) ok = gate(W0);
        if (ok && W0 >= 1) ok = gate(W0 - 1);
        for (int w = W0; ok && w >= 0; --w) {
          if (!(ok = mbar_wait(&bars[B_P], (W0 - w) & 1, err, kErrP))) break;
          tc_fence_after();
          const int n = T0 - w / 4, st = n & 1;
          const uint32_t vt = sV + st * NS * 8192 + (w & 3) * kW * 128;
          const uint32_t pa = tmem + ((w & 1) ? L::T_SG1 : L::T_SG0);
          mma_ts(tmem + L::T_O, pa, sdesc_mnmajor(vt, 8192), id_pv, w != W0);
          mma_commit(&bars[B_O]);
          if ((w & 3) == 0) mma_commit(&bars[B_KVE + st]);
          // P(w) has been consumed (in issue order) -> its buffer takes gate(w-2)
          if (w >= 2) ok = gate(w - 2);
        }
        mma_commit(&bars[B_DRAIN2]);
        mbar_wait(&bars[B_DRAIN2], 0, err, kErrDrain);
      }
    } else if (warp == 11 && KMT) {
      // ------------------------------------------------- K^(m) panel loads
      if (lane == 0) {
        prefetch_tmap(&P.tm_km[0]);
        if (NS > 1) prefetch_tmap(&P.tm_km[1]);
        const uint32_t bytes = (P.km_rows[0] + (NS > 1 ? P.km_rows[1] : 0)) * 128;
        const int panel0 = (b * P.Hkv + hk) * P.km_nhw;
        int last[4] = {-1, -1, -1, -1};  // [half][buffer]: last use issued
        bool ok = true;
        for (int w = W0; ok && w >= 0; --w) {
          const int k = W0 - w, buf = k % nb, use = k / nb;
          for (int hh = 0; hh < 2; ++hh) {
            const int i = 2 * hh + buf;
            if (use > 0 && !(ok = mbar_wait(&bars[B_BE + i], (use - 1) & 1, err, kErrBEmpty))) break;
            mbar_expect_tx(&bars[B_BF + i], bytes);
            uint8_t* dst = smem + L::BOP + (hh * nb + buf) * P.b_buf_bytes;
            for (int s = 0; s < NS; ++s)
              tma_load_3d(dst + P.b_slab_off[s], &P.tm_km[s], &bars[B_BF + i], 0, 0,
                          panel0 + 2 * w + hh);
            last[i] = use;
          }
        }
        // no copy may still be in flight when the CTA exits
        for (int i = 0; i < 4; ++i)
          if (last[i] >= 0) mbar_wait(&bars[B_BF + i], last[i] & 1, err, kErrDrain);
      }
    }
    __syncwarp();
    regs_inc<128>();
  } else if (warp >= 12 && KMT) {
    regs_dec<kBldRegs>();
    named_bar(1, kThreads);
    // ------------------------------------------------- gates (panel launches)
    // One thread per row: the window's gates and in-window positions and the
    // running carry, handed to both row groups through shared memory (the
    // row groups would otherwise each compute all 16 gates of the row).
    const int r = tid - 384;
    const int t = q0 + r;
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t s_gu = smem_u32(smem + L::GU), s_gc = smem_u32(smem + L::GC);
    float carry = 0.f, carry_c = 0.f;  // compensated, as in the row code
    for (int w = W0; w >= 0; --w) {
      const int buf = w & 1;
      if (!wwait(bars[B_SG + buf], ((W0 - w) >> 1) & 1, err, kErrSg)) break;
      tc_fence_after();
      uint32_t sraw[16];
      tmem_ld16(lane_base + ((w & 1) ? L::T_SG1 : L::T_SG0), sraw);
      tmem_wait_ld();
      float uu[16];
      const float acc = fwd_window_gates<true>(sraw, w * kW, t, uu);
      // group g's keys i -> 8 (i >> 2) + slot_key(4 g + (i & 3)): chunk c = i >> 2
#pragma unroll
      for (int g = 0; g < 2; ++g)
#pragma unroll
        for (int c = 0; c < 2; ++c)
          sts128f(s_gu + (((buf * 2 + g) * 2 + c) * 128 + r) * 16,
                  make_float4(uu[8 * c + slot_key(4 * g)], uu[8 * c + slot_key(4 * g + 1)],
                              uu[8 * c + slot_key(4 * g + 2)], uu[8 * c + slot_key(4 * g + 3)]));
      const float y = acc - carry_c;
      const float carry_next = carry + y;
      carry_c = (carry_next - carry) - y;
      carry = carry_next;
      sts32f(s_gc + (buf * 128 + r) * 4, carry - carry_c);
      tc_fence_before();
      mbar_arrive(&bars[B_GT + buf]);
    }
    __syncwarp();
    regs_inc<128>();
  } else if (warp >= 12) {
    regs_dec<kBldRegs>();
    named_bar(1, kThreads);
    // ------------------------------------------------- K^(m) operand builder
    // Work items are the (K-step s, row, 16-byte chunk) triples the G GEMM
    // reads: rows [0, nrow[s]) x 2 chunks of K-step s, numbered s-major and
    // dealt round-robin over the 128 builder threads.  Each thread's item
    // offsets are fixed for the whole kernel and computed once: the K chunk
    // (without the window/half row offset), the coefficient quad, the
    // destination chunk, and the (-i)^m swap/sign flags.
    constexpr int kMaxItems = L::MAX_ITEMS;
    const int gt = tid - 384;
    uint2* items = reinterpret_cast<uint2*>(smem + L::ITEMS);
    int my_n = 0;
    {
      int item_end[8];
      int acc = 0;
#pragma unroll
      for (int s2 = 0; s2 < 8; ++s2) {
        acc += (s2 < KSTEPS) ? 2 * P.nrow[s2] : 0;
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
          const int r = local >> 1, c = 2 * s2 + (local & 1), m = r >> 3, j = slot_key(r & 7);
          const uint32_t kofs = (c >> 3) * 8192 + j * 128 + (((c & 7) ^ j) << 4);
          const uint32_t cofs = (m * NP + 4 * c) * 4;
          const uint32_t bofs = P.b_slab_off[c >> 3] + sw128_offset(r, c & 7);
          const uint32_t flags = (m & 1) | ((m & 2) ? 2u : 0u) | (((m + 1) & 2) ? 4u : 0u);
          d = make_uint2(kofs | (cofs << 16), bofs | (flags << 16));
          my_n = i + 1;
        }
        items[i * 128 + gt] = d;
      }
    }
    for (int w = W0; w >= 0; --w) {
      const int k = W0 - w, buf = k % nb, use = k / nb;
      const int n = T0 - w / 4, st = n & 1;
      if (!wwait(bars[B_KVF + st], (n >> 1) & 1, err, kErrKvFull)) break;
      bool ok = true;
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        if (use > 0 &&
            !(ok = wwait(bars[B_BE + 2 * hh + buf], (use - 1) & 1, err, kErrBEmpty)))
          break;
        const uint32_t kt = sK + st * NS * 8192 + (2 * (w & 3) + hh) * 1024;
        const uint32_t bt = sB + (hh * nb + buf) * P.b_buf_bytes;
#pragma unroll 1
        for (int i0 = 0; i0 < my_n; i0 += 4) {
          uint2 d[4];
          uint4 kv[4];
          float4 cf[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) d[j] = items[(i0 + j < kMaxItems ? i0 + j : 0) * 128 + gt];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            kv[j] = lds128(kt + (d[j].x & 0xffffu));
            cf[j] = lds128f(s_coef_u + (d[j].x >> 16));
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (i0 + j < my_n) {
              // (-i)^m: odd terms swap the pair's components (one byte
              // permute), terms 2, 3 mod 4 negate one or both (a sign-bit xor)
              const uint32_t fl = d[j].y >> 16;
              const uint32_t sel = (fl & 1u) ? 0x1032u : 0x3210u;
              const uint32_t sgn = ((fl & 2u) ? 0x8000u : 0u) | ((fl & 4u) ? 0x80000000u : 0u);
              const uint32_t in[4] = {kv[j].x, kv[j].y, kv[j].z, kv[j].w};
              const float cfa[4] = {cf[j].x, cf[j].y, cf[j].z, cf[j].w};
              uint32_t out[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const uint32_t wv = __byte_perm(in[e], 0u, sel) ^ sgn;
                out[e] = E::pack(cfa[e] * E::lo(wv), cfa[e] * E::hi(wv));
              }
              sts128(bt + (d[j].y & 0xffffu), make_uint4(out[0], out[1], out[2], out[3]));
            }
          }
        }
        fence_async_smem();
        mbar_arrive(&bars[B_BF + 2 * hh + buf]);
      }
      if (!ok) break;
      if ((w & 3) == 0) mbar_arrive(&bars[B_KVE + st]);
    }
    __syncwarp();
    regs_inc<128>();
  } else {
    // ------------------------------------------------------------ row warps
    regs_inc<kRowRegs>();
    named_bar(1, kThreads);
    const int rg = warp >> 2;  // row group
    const int r = tid & 127;
    const int t = q0 + r;
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t s_xch = smem_u32(smem + L::XCH);
    // gate sum of keys after the window, compensated (Kahan): it reaches ~S/2,
    // where fp32 steps are 2^-10 at S = 32768, and a plain running sum over
    // S/16 windows drifts by ~1e-2 (an angle error of that size in the fastest
    // rotation).  carry - carry_c is the sum to ~1 ulp.
    float carry = 0.f, carry_c = 0.f;
    float a_total = 0.f;  // gate sum of all keys (the saved A)
    const uint32_t s_gu = smem_u32(smem + L::GU), s_gc = smem_u32(smem + L::GC);
    float m_used = -1e30f, m_true = -INFINITY;
    float lsum = 0.f;                      // this group's keys
    bool ok = wwait(bars[B_Q], 0, err, kErrQ);

    // This group's half of the A operand of one window, v = R((carry + c0)
    // theta) q_t, into tensor memory (angles reduced to [-pi, pi] on the FMA
    // pipe, sine/cosine on MUFU).
    const float th_max = theta_max(s_th, NP);
    auto build_a = [&](float cw, uint32_t av_col) {
      const float base = cw + kC0;
      const bool mufu_reduce = __all_sync(0xffffffffu, base * th_max < kMufuReduceMax);
#pragma unroll 1
      for (int g = 0; g < NP / 32; ++g) {
        // 16 independent pairs, advanced stage by stage (instruction-level
        // parallelism across pairs instead of one long chain per pair)
        const int p0 = rg * (NP / 2) + 16 * g;
        uint4 qv[4];
        float th[16];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int c = p0 / 4 + cc;  // 16-byte chunk of the row (4 pairs)
          qv[cc] = lds128(sQ + (c >> 3) * 16384 + sw128_offset(r, c & 7));
          const float4 t4 = lds128f(s_th_u + 16 * c);
          th[4 * cc] = t4.x; th[4 * cc + 1] = t4.y; th[4 * cc + 2] = t4.z; th[4 * cc + 3] = t4.w;
        }
        float rr[16], sn[16], cs[16];
        angles16(base, th, rr);
        if (!mufu_reduce) {
#pragma unroll
          for (int i = 0; i < 16; ++i) rr[i] = reduce_2pi(rr[i]);
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) __sincosf(rr[i], &sn[i], &cs[i]);
        uint32_t regs[16];
        rotate16<E>(qv, sn, cs, regs);
        tmem_st16(lane_base + av_col + p0, regs);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars[B_AV]);
    };

    // Clenshaw combine of this group's 4 keys (slots 4 rg + j) of G half HH:
    // f_j = sum_m T_m(u_j) G_m, G columns 16 c + 8 (m & 1) + slot (m = 2c + (m & 1)).
    // Position j runs NT(j) terms: all kM, or with the panels' per-offset
    // expansions the larger count of the two groups' keys at that position.
    // All loads go out before one wait; the half's G region is then released.
    auto combine = [&](auto hh_tag, uint32_t gcol, const float (&uj)[4], float (&f)[4],
                       int ge_bar) {
      constexpr int HH = decltype(hh_tag)::value;
      constexpr int NT0 = KMT ? tcx::position_terms(kM, HH, 0) : kM;
      constexpr int NT1 = KMT ? tcx::position_terms(kM, HH, 1) : kM;
      constexpr int NT2 = KMT ? tcx::position_terms(kM, HH, 2) : kM;
      constexpr int NT3 = KMT ? tcx::position_terms(kM, HH, 3) : kM;
      constexpr int NT[4] = {NT0, NT1, NT2, NT3};
      constexpr int NMAX = NT0 > NT1 ? (NT0 > NT2 ? (NT0 > NT3 ? NT0 : NT3) : (NT2 > NT3 ? NT2 : NT3))
                                     : (NT1 > NT2 ? (NT1 > NT3 ? NT1 : NT3) : (NT2 > NT3 ? NT2 : NT3));
      uint32_t g[kM / 2][2][4];
#pragma unroll
      for (int c = 0; c < (NMAX + 1) / 2; ++c) {
        tmem_ld4(lane_base + gcol + 16 * c + 4 * rg, g[c][0]);
        if (2 * c + 1 < NMAX) tmem_ld4(lane_base + gcol + 16 * c + 8 + 4 * rg, g[c][1]);
      }
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&bars[ge_bar]);
      float b1[4], b2[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) { b1[j] = 0.f; b2[j] = 0.f; }
#pragma unroll
      for (int m = NMAX - 1; m >= 0; --m) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (m >= NT[j]) continue;
          const float a = __uint_as_float(g[m >> 1][m & 1][j]);
          if (m > 0) {
            const float bn = fmaf(2.0f * uj[j], b1[j], a - b2[j]);
            b2[j] = b1[j];
            b1[j] = bn;
          } else {
            f[j] = fmaf(uj[j], b1[j], a - b2[j]);
          }
        }
      }
    };

    if (ok) {
      tc_fence_after();
      build_a(0.f, (W0 & 1) ? L::T_AV1 : L::T_AV0);
    }
    for (int w = W0; ok && w >= 0; --w) {
      const int k = W0 - w;
      const int j0 = w * kW;
      const uint32_t sg = (w & 1) ? L::T_SG1 : L::T_SG0;
      // gates of the window: this group's keys i -> key 8 (i >> 2) + slot_key(4 rg + (i & 3))
      float uo[8];
      float carry_a;  // gate sum of the keys after the next window (its A operand)
      if (KMT) {
        // from warps 12-15
        const int buf = w & 1;
        if (!(ok = wwait(bars[B_GT + buf], ((W0 - w) >> 1) & 1, err, kErrSg))) break;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const float4 v = lds128f(s_gu + (((buf * 2 + rg) * 2 + c) * 128 + r) * 16);
          uo[4 * c] = v.x; uo[4 * c + 1] = v.y; uo[4 * c + 2] = v.z; uo[4 * c + 3] = v.w;
        }
        carry_a = lds32f(s_gc + (buf * 128 + r) * 4);
      } else {
        if (!(ok = wwait(bars[B_SG + (w & 1)], ((W0 - w) >> 1) & 1, err, kErrSg))) break;
        tc_fence_after();
        uint32_t sraw[16];
        tmem_ld16(lane_base + sg, sraw);
        tmem_wait_ld();
        float uu[16];
        const float acc = fwd_window_gates<false>(sraw, j0, t, uu);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          uo[i] = rg ? uu[8 * (i >> 2) + slot_key(4 + (i & 3))] : uu[8 * (i >> 2) + slot_key(i & 3)];
        const float y = acc - carry_c;
        const float carry_next = carry + y;
        carry_c = (carry_next - carry) - y;
        carry = carry_next;
        carry_a = carry - carry_c;
      }
      // A operand of the next window (its buffer was last read by G(w+1),
      // which completed before this row group loaded G(w+1))
      if (w > 0) build_a(carry_a, ((w - 1) & 1) ? L::T_AV1 : L::T_AV0);
      float lg[8];
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        if (!(ok = wwait(bars[B_GF + hh], k & 1, err, kErrG))) break;
        tc_fence_after();
        float uj[4], f[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) uj[j] = hh ? uo[4 + j] : uo[j];
        if (hh == 0)
          combine(std::integral_constant<int, 0>(), L::T_G0, uj, f, B_GE);
        else
          combine(std::integral_constant<int, 1>(), L::T_G1, uj, f, B_GE + 1);
        if (hh == 0) {
#pragma unroll
          for (int j = 0; j < 4; ++j) lg[j] = f[j];
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) lg[4 + j] = f[j];
        }
      }
      if (!ok) break;
      // online softmax (log2 units) with stale-max rescaling; the row max
      // of the window is agreed between the two groups
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int kj = j0 + 8 * (i >> 2) + (rg ? slot_key(4 + (i & 3)) : slot_key(i & 3));
        if (HAS_BIAS && kj <= t) lg[i] = fmaf(P.bias[(int64_t)t * P.bias_rs + kj], kLog2e, lg[i]);
        lg[i] = (kj <= t) ? lg[i] : -INFINITY;
        mx = fmaxf(mx, lg[i]);
      }
      sts32f(s_xch + (rg * 128 + r) * 4, mx);
      mbar_arrive(&bars[B_XM]);
      if (!(ok = wwait(bars[B_XM], k & 1, err, kErrX))) break;
      mx = fmaxf(mx, lds32f(s_xch + ((rg ^ 1) * 128 + r) * 4));
      m_true = fmaxf(m_true, mx);
      if (k > 0) {
        if (!(ok = wwait(bars[B_O], (k - 1) & 1, err, kErrO))) break;
        tc_fence_after();
      }
      const bool resc = mx > m_used + kRescale;
      const float alpha = resc ? exp2f(m_used - mx) : 1.0f;
      if (resc) m_used = mx;
      lsum *= alpha;
      if (k > 0 && __any_sync(0xffffffffu, resc)) {
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {  // this group's half of the O columns
          const uint32_t oc = lane_base + L::T_O + rg * (D / 2) + 16 * c;
          uint32_t o[16];
          tmem_ld16(oc, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st16(oc, o);
        }
      }
      uint32_t pk[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float p0 = exp2f(lg[2 * i] - m_used), p1 = exp2f(lg[2 * i + 1] - m_used);
        lsum += p0 + p1;
        pk[i] = E::pack(p0, p1);
      }
      // P over the gate columns (keys 2i, 2i+1 in word i): this group's key
      // pairs are slots (4 rg, 4 rg + 1) and (4 rg + 2, 4 rg + 3) of each half
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int key = 8 * (i >> 1) + (rg ? slot_key(4 + 2 * (i & 1)) : slot_key(2 * (i & 1)));
        tmem_st1(lane_base + sg + key / 2, pk[i]);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars[B_P]);
      a_total = carry_a;
    }
    // epilogue: row sum of both groups, then this group's output columns
    if (ok) ok = wwait(bars[B_O], W0 & 1, err, kErrO);
    sts32f(s_xch + (256 + rg * 128 + r) * 4, lsum);
    mbar_arrive(&bars[B_XL]);
    if (ok) ok = wwait(bars[B_XL], 0, err, kErrX);
    if (ok) {
      tc_fence_after();
      const float ltot = lsum + lds32f(s_xch + (256 + (rg ^ 1) * 128 + r) * 4);
      const float inv = 1.0f / ltot;
      T* orow = reinterpret_cast<T*>(P.o) + b * P.os[0] + h * P.os[1] +
                (int64_t)(t - P.r0) * P.os[2] +
                rg * (D / 2);
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[16];
        tmem_ld16(lane_base + L::T_O + rg * (D / 2) + 16 * c, o);
        tmem_wait_ld();
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          pk[i] = E::pack(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
        if (t < S) {
          uint4* dst = reinterpret_cast<uint4*>(orow + 16 * c);
          dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
      if (t < S && rg == 0) {
        const int64_t ri = ((int64_t)b * P.H + h) * P.S + (t - P.r0);
        const float M = m_true * 0.6931471805599453f;
        const float Lv = ltot * exp2f(m_used - m_true);
        if (P.m) P.m[ri] = M;
        if (P.l) P.l[ri] = Lv;
        if (P.a) P.a[ri] = a_total;
        if (P.lse) P.lse[ri] = M + logf(Lv);
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

// ------------------------------------------------------------------ host
using tcx::encode;
using tcx::get_encoder;

static void fill_coefficients(Params& p, int D, float theta, float sm_scale) {
  tcx::fill_coefficients(p.coef, p.nrow, D, theta, sm_scale);
}

// Lay out the K^(m) buffers (rows actually read per slab) and choose double
// buffering when it fits in shared memory.  Returns the dynamic smem bytes.
template <int D>
static int plan_buffers(Params& p) {
  using L = Layout<D>;
  int off = 0;
  for (int s = 0; s < L::NS; ++s) {
    p.b_slab_off[s] = off;
    off += p.nrow[4 * s] * 128;
  }
  p.b_buf_bytes = (off + 1023) & ~1023;
  p.nb = (L::BOP + 4 * p.b_buf_bytes + 1024 <= kSmemLimit) ? 2 : 1;
  return L::BOP + 2 * p.nb * p.b_buf_bytes + 1024;
}

template <typename T> constexpr int E_dtype() {
  return ElemTraits<T>::kBf16 ? COROPE_DTYPE_BF16 : COROPE_DTYPE_F16;
}

template <typename T, int D, bool HAS_BIAS, bool KMT>
static cudaError_t launch_k(const Params& p, int smem, dim3 grid, cudaStream_t st) {
  auto kern = fwd_kernel<T, D, HAS_BIAS, KMT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kSmemLimit);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, smem, st>>>(p);
  return cudaGetLastError();
}

// With a workspace of tcx::offset_panel_bytes<kM> bytes the K^(m) operands
// are written once by tcx::offset_panel_kernel (per-offset expansions, from
// the coefficients tcx::offset_coef_kernel puts behind them) and loaded by
// TMA; without one the forward kernel's builder warps make them from the K
// tiles (one expansion per window).
template <typename T, int D>
static cudaError_t launch_t(Params& p, const FwdArgs& a, cudaStream_t st, void* ws,
                            size_t ws_bytes) {
  static tcx::OffsetPanelArgs pa;  // guarded by the caller's lock
  const size_t need = tcx::offset_panel_bytes<kM>(a.B, a.Hkv, a.Sk, D, a.theta, a.sm_scale, &pa);
  const bool kmt = ws && need > 0 && ws_bytes >= need;
  if (kmt)  // the per-offset expansions' K extents
    for (int s = 0; s < 8; ++s) p.nrow[s] = pa.nrow[s];
  const int smem = plan_buffers<D>(p);
  if (smem > kSmemLimit) return cudaErrorInvalidValue;
  dim3 grid((a.S + kBM - 1) / kBM, a.H, a.B);
  if (kmt) {
    const int64_t np = tcx::panel_count(a.B, a.Hkv, a.Sk);
    pa.k = a.k;
    for (int i = 0; i < 3; ++i) pa.ks[i] = a.ks[i];
    pa.out[0] = ws;
    pa.out[1] = static_cast<uint8_t*>(ws) + np * pa.rows[0] * 128;
    // the coefficient table behind both slabs' panels (16-byte aligned: rows are 128 B)
    pa.cf = reinterpret_cast<float2*>(static_cast<uint8_t*>(ws) + np * (pa.rows[0] + pa.rows[1]) * 128);
    for (int s = 0; s < D / 64; ++s)
      if (!tcx::encode_panels(&p.tm_km[s], pa.out[s], E_dtype<T>(), pa.rows[s], np))
        return cudaErrorInvalidValue;
    p.km_nhw = pa.nhw;
    p.km_rows[0] = pa.rows[0];
    p.km_rows[1] = pa.rows[1];
    tcx::offset_coef_kernel<<<16, 64, 0, st>>>(pa);
    tcx::offset_panel_kernel<T, D>
        <<<dim3(tcx::panel_halfwindows_read(a.Sk, a.r0, a.S), a.B * a.Hkv), 128, 0, st>>>(pa);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  if (a.bias)
    return kmt ? launch_k<T, D, true, true>(p, smem, grid, st)
               : launch_k<T, D, true, false>(p, smem, grid, st);
  return kmt ? launch_k<T, D, false, true>(p, smem, grid, st)
             : launch_k<T, D, false, false>(p, smem, grid, st);
}

}  // namespace tc

static bool rows_ok(const void* ptr, const int64_t* st) {
  return (reinterpret_cast<uintptr_t>(ptr) % 16) == 0 && (st[0] * 2) % 16 == 0 &&
         (st[1] * 2) % 16 == 0 && (st[2] * 2) % 16 == 0;
}

bool tc_fwd_supported(const FwdArgs& a, int dtype) {
  if (dtype != COROPE_DTYPE_BF16 && dtype != COROPE_DTYPE_F16) return false;
  // the expansions' term counts assume every frequency theta_p <= 1
  if (!(a.theta >= 1.f)) return false;
  if (a.D != 64 && a.D != 128) return false;
  if (!rows_ok(a.q, a.qs) || !rows_ok(a.k, a.ks) || !rows_ok(a.v, a.vs) || !rows_ok(a.o, a.os))
    return false;
  if (a.bias && (reinterpret_cast<uintptr_t>(a.bias) % 4) != 0) return false;
  return tc::get_encoder() != nullptr;
}

size_t tc_fwd_workspace_bytes(const FwdArgs& a) {
  return tcx::offset_panel_bytes<tc::kM>(a.B, a.Hkv, a.Sk, a.D, a.theta, a.sm_scale);
}

cudaError_t tc_fwd_launch(const FwdArgs& a, int dtype, cudaStream_t st, void* ws,
                          size_t ws_bytes) {
  using namespace tc;
  static Params p;  // large (>4 KB); filled per call under a lock
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  std::memset(&p, 0, sizeof(p));
  if (!encode(&p.tm_q, a.q, dtype, a.B, a.H, a.S, a.D, a.qs, kBM) ||
      !encode(&p.tm_k, a.k, dtype, a.B, a.Hkv, a.Sk, a.D, a.ks, kKT) ||
      !encode(&p.tm_v, a.v, dtype, a.B, a.Hkv, a.Sk, a.D, a.vs, kKT))
    return cudaErrorInvalidValue;
  p.r0 = a.r0;
  p.o = a.o;
  p.m = a.m; p.l = a.l; p.a = a.a; p.lse = a.lse;
  p.thetas = a.thetas; p.theta = a.theta;
  p.bias = a.bias; p.bias_rs = a.bias_rs;
  for (int i = 0; i < 3; ++i) p.os[i] = a.os[i];
  p.B = a.B; p.H = a.H; p.Hkv = a.Hkv; p.S = a.S;
  fill_coefficients(p, a.D, a.theta, a.sm_scale);
  const bool bf = dtype == COROPE_DTYPE_BF16;
  if (a.D == 64)
    return bf ? launch_t<__nv_bfloat16, 64>(p, a, st, ws, ws_bytes)
              : launch_t<__half, 64>(p, a, st, ws, ws_bytes);
  return bf ? launch_t<__nv_bfloat16, 128>(p, a, st, ws, ws_bytes)
            : launch_t<__half, 128>(p, a, st, ws, ws_bytes);
}

}  // namespace corope
