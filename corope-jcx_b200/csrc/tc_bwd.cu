// Tensor-core (tcgen05) CoRoPE backward for sm_100a, head_dim 128.
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
//   dQ launch:  X = Y . K^(m) (K = 14 terms x 16 keys) and dq_t +=
//               ln2 R(-(C_t + c0) theta) X_t  (per-row rotation after the GEMM),
//               plus the gate part dq += dS K (UMMA straight into TMEM).
//   dK launch:  C^T = v^T . Y (M = head dim, N = 14 terms x 8 keys, K = the 128
//               query rows), then per head dim a combine over the 14 terms
//               with the coefficients and the (i)^m pair rotation; plus
//               dV^T = dO^T P and dK_gate^T = Q^T dS; fp32 atomics into the
//               dk/dv accumulators of the workspace (query tiles race on keys).
//
// Roles per CTA (128 query rows of one (b, h), 384 threads): warps 0-3 row
// work; warp 4 TMA; warp 5 UMMA for the gate, dP and G GEMMs; warp 6 UMMA
// for the mode's GEMMs; warps 8-11 build K^(m) (and, in the dK launch, run
// the per-dimension combine).  Every wait is bounded as in the forward.
#include <cstring>

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
using tcx::kM;
using tcx::kSmemLimit;
using tcx::kW;
using tcx::sigmoid_f;

constexpr int D = 128;
constexpr int NS = 2;        // 64-element slabs of the head dim
constexpr int NP = 64;       // rotation pairs
constexpr int KSTEPS = 8;    // 16-element K steps over the head dim
constexpr int kBM = 128;     // query rows per CTA
constexpr int kKT = 32;      // keys per K/V tile (2 windows)
constexpr int kThreads = 384;
constexpr int MODE_DQ = 0, MODE_DK = 1;

enum : int {
  kErrQ = 201, kErrKvEmpty, kErrKvFull, kErrSd, kErrSdEmpty, kErrAv, kErrAvEmpty, kErrB,
  kErrBEmpty, kErrG, kErrGEmpty, kErrY, kErrX, kErrXFree, kErrC, kErrCEmpty, kErrDrain
};

struct Params {
  CUtensorMap tm_q, tm_k, tm_v, tm_do;
  void* dq;              // dQ launch output, element type of q
  float *dk32, *dv32;    // dK launch accumulators [B, Hkv, S, D]
  const float *lse, *delta, *a;  // [B, H, S]
  const float* thetas;
  const float* bias;
  int64_t bias_rs;
  int64_t dqs[3];
  int B, H, Hkv, S;
  float theta;
  int nrow[8];
  int nb;
  int b_slab_off[2];
  int b_buf_bytes;
  float coef[kM][64];
};

// shared memory (bytes from the 1024-aligned base)
constexpr int S_Q = 0;                       // [NS][128 rows][128 B]
constexpr int S_DO = S_Q + NS * 16384;
constexpr int S_K = S_DO + NS * 16384;       // [2 stages][NS][32 rows][128 B]
constexpr int S_V = S_K + 2 * NS * 4096;
constexpr int S_AV = S_V + 2 * NS * 4096;    // A operand rows [NS][128][128 B]
constexpr int S_Y = S_AV + NS * 16384;       // dK launch: Y | P | dS rows [NS][128][128 B]
template <int MODE> struct SmemTail {
  static constexpr int COEF = (MODE == MODE_DK) ? S_Y + NS * 16384 : S_Y;
  static constexpr int TH = COEF + kM * NP * 4;
  static constexpr int BAR = TH + NP * 4;
  static constexpr int NBAR = 40;
  static constexpr int SLOT = BAR + NBAR * 8;
  static constexpr int MAX_ITEMS = (2 * 8 * 8 * kM + 127) / 128;
  static constexpr int ITEMS = (SLOT + 16 + 15) & ~15;
  static constexpr int BOP = (ITEMS + MAX_ITEMS * 128 * 8 + 1023) & ~1023;
};

// tensor memory columns
namespace tq {  // dQ launch
constexpr uint32_t X = 0, DQ = 128, G = 256, SG0 = 368, SG1 = 384, DP0 = 400, DP1 = 416,
                   YT = 432;  // Y (56 cols) | dS (8 cols)
static_assert(YT + 64 <= 512, "tmem");
}  // namespace tq
namespace tk {  // dK launch
constexpr uint32_t G = 0, SG0 = 112, SG1 = 128, DP0 = 144, DP1 = 160, C0 = 176, C1 = 320;
// C region: [0,112) C^T terms x keys, [112,128) dO^T (P | dS), [128,144) Q^T (P | dS)
static_assert(C1 + 144 <= 512, "tmem");
}  // namespace tk

enum {
  B_Q = 0, B_KVF = 1, B_KVE = 3, B_SDF = 5, B_SDE = 7, B_AVF = 9, B_AVE = 10,
  B_BF = 11,  // [half][buf]
  B_BE = 15,  // [half][buf]
  B_GF = 19,  // [half]
  B_GE = 21,
  B_YA = 22, B_YDONE = 23, B_YB = 24,
  B_XF = 25, B_XFREE = 26, B_YTFREE = 27,        // dQ launch
  B_CF = 28, B_CE = 30, B_YFREE = 32,            // dK launch: [half] x 2
  B_DRAIN5 = 34, B_DRAIN6 = 35
};

__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t (&r)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3])
               : "memory");
}

template <typename T, int MODE, bool HAS_BIAS>
__global__ void __launch_bounds__(kThreads, 1) bwd_kernel(const __grid_constant__ Params P) {
  using E = ElemTraits<T>;
  using L = SmemTail<MODE>;
  using namespace sm100;

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
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (P.H / P.Hkv);
  const int q0 = qt * kBM;
  const int S = P.S;
  const int WL = min(S - 1, q0 + kBM - 1) / kW;  // last (highest) window
  const int nb = P.nb;

  if (tid == 0) {
    mbar_init(&bars[B_Q], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[B_KVF + i], 1);
      mbar_init(&bars[B_KVE + i], 2 + 128);  // two UMMA issuers + the builders
      mbar_init(&bars[B_SDF + i], 1);
      mbar_init(&bars[B_SDE + i], 128);
      mbar_init(&bars[B_GF + i], 1);
      mbar_init(&bars[B_CF + i], 1);
      mbar_init(&bars[B_CE + i], 128);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&bars[B_BF + i], 128);
      mbar_init(&bars[B_BE + i], MODE == MODE_DQ ? 2 : 1);  // G (+ X) done with K^(m)
    }
    mbar_init(&bars[B_AVF], 128);
    mbar_init(&bars[B_AVE], 1);
    mbar_init(&bars[B_GE], 128);
    mbar_init(&bars[B_YA], 128);
    mbar_init(&bars[B_YDONE], 1);
    mbar_init(&bars[B_YB], 128);
    mbar_init(&bars[B_XF], 1);
    mbar_init(&bars[B_XFREE], 128);
    mbar_init(&bars[B_YTFREE], 1);
    mbar_init(&bars[B_YFREE], 1);
    mbar_init(&bars[B_DRAIN5], 1);
    mbar_init(&bars[B_DRAIN6], 1);
    fence_mbar_init();
  }
  for (int i = tid; i < kM * NP; i += kThreads) s_coef[i] = P.coef[i / NP][i % NP];
  for (int p = tid; p < NP; p += kThreads) s_th[p] = theta_at(P.thetas, P.theta, p, D);
  // The K^(m) buffers start at zero: the builders skip the pruned (term,
  // head-dim) entries, which the dQ launch's X GEMM still reads densely.
  {
    uint4* kb = reinterpret_cast<uint4*>(smem + L::BOP);
    const int n16 = (2 * P.nb * P.b_buf_bytes) / 16;
    for (int i = tid; i < n16; i += kThreads) kb[i] = make_uint4(0u, 0u, 0u, 0u);
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
  const uint32_t sB = smem_u32(smem + L::BOP);
  const uint32_t s_th_u = smem_u32(s_th), s_coef_u = smem_u32(s_coef);
  const uint32_t T_SG0 = MODE == MODE_DQ ? tq::SG0 : tk::SG0;
  const uint32_t T_SG1 = MODE == MODE_DQ ? tq::SG1 : tk::SG1;
  const uint32_t T_DP0 = MODE == MODE_DQ ? tq::DP0 : tk::DP0;
  const uint32_t T_DP1 = MODE == MODE_DQ ? tq::DP1 : tk::DP1;
  const uint32_t T_G = MODE == MODE_DQ ? tq::G : tk::G;

  if (warp == 4) {
    // ------------------------------------------------------------ TMA
    if (lane == 0) {
      prefetch_tmap(&P.tm_q);
      prefetch_tmap(&P.tm_k);
      prefetch_tmap(&P.tm_v);
      prefetch_tmap(&P.tm_do);
      mbar_expect_tx(&bars[B_Q], 2 * NS * 16384);
      for (int s = 0; s < NS; ++s) {
        tma_load_4d(smem + S_Q + s * 16384, &P.tm_q, &bars[B_Q], 64 * s, q0, h, b);
        tma_load_4d(smem + S_DO + s * 16384, &P.tm_do, &bars[B_Q], 64 * s, q0, h, b);
      }
      const int TL = WL / 2;  // last K/V tile
      int last_use[2] = {-1, -1};
      for (int n = 0; n <= TL; ++n) {
        const int st = n & 1, u = n >> 1;
        if (n >= 2 && !mbar_wait(&bars[B_KVE + st], (u - 1) & 1, err, kErrKvEmpty)) break;
        mbar_expect_tx(&bars[B_KVF + st], 2 * NS * 4096);
        for (int s = 0; s < NS; ++s) {
          tma_load_4d(smem + S_K + (st * NS + s) * 4096, &P.tm_k, &bars[B_KVF + st], 64 * s,
                      kKT * n, hk, b);
          tma_load_4d(smem + S_V + (st * NS + s) * 4096, &P.tm_v, &bars[B_KVF + st], 64 * s,
                      kKT * n, hk, b);
        }
        last_use[st] = u;
      }
      for (int st = 0; st < 2; ++st)
        if (last_use[st] >= 0) mbar_wait(&bars[B_KVF + st], last_use[st] & 1, err, kErrDrain);
    }
  } else if (warp == 5) {
    // ---------------------------------- UMMA: gate, dP and G GEMMs
    if (lane == 0) {
      const uint32_t id_n16 = idesc_f16(128, 16, E::kBf16, false);
      bool ok = mbar_wait(&bars[B_Q], 0, err, kErrQ);
      tc_fence_after();
      // gate scores Q K^T and dP = dO V^T of window w into buffer w & 1
      auto sd = [&](int w) -> bool {
        const int n = w >> 1, st = n & 1;
        if (!mbar_wait(&bars[B_KVF + st], (n >> 1) & 1, err, kErrKvFull)) return false;
        if (w >= 2 && !mbar_wait(&bars[B_SDE + (w & 1)], ((w >> 1) - 1) & 1, err, kErrSdEmpty))
          return false;
        tc_fence_after();
        const uint32_t kt = sK + st * NS * 4096 + (w & 1) * kW * 128;
        const uint32_t vt = sV + st * NS * 4096 + (w & 1) * kW * 128;
        const uint32_t dsg = tmem + ((w & 1) ? T_SG1 : T_SG0);
        const uint32_t ddp = tmem + ((w & 1) ? T_DP1 : T_DP0);
#pragma unroll
        for (int s = 0; s < KSTEPS; ++s) {
          const uint32_t off = (s >> 2) * 16384 + 32 * (s & 3);
          const uint32_t koff = (s >> 2) * 4096 + 32 * (s & 3);
          mma_ss(dsg, sdesc_kmajor(sQ + off), sdesc_kmajor(kt + koff), id_n16, s > 0);
          mma_ss(ddp, sdesc_kmajor(sDO + off), sdesc_kmajor(vt + koff), id_n16, s > 0);
        }
        mma_commit(&bars[B_SDF + (w & 1)]);
        if (w & 1) mma_commit(&bars[B_KVE + st]);  // last window of the tile
        return true;
      };
      if (ok) ok = sd(0);
      if (ok && WL >= 1) ok = sd(1);
      for (int w = 0; ok && w <= WL; ++w) {
        const int buf = w % nb, use = w / nb;
        if (!(ok = mbar_wait(&bars[B_AVF], w & 1, err, kErrAv))) break;
        for (int hh = 0; hh < 2 && ok; ++hh) {
          ok = mbar_wait(&bars[B_BF + 2 * hh + buf], use & 1, err, kErrB);
          // the single G region: the rows have consumed the previous half
          const int prev = 2 * w + hh - 1;
          if (ok && prev >= 0) ok = mbar_wait(&bars[B_GE], prev & 1, err, kErrGEmpty);
          if (!ok) break;
          tc_fence_after();
          const uint32_t bb = sB + (hh * nb + buf) * P.b_buf_bytes;
#pragma unroll
          for (int s = 0; s < KSTEPS; ++s) {
            const int nr = P.nrow[s];
            if (nr == 0) break;
            mma_ss(tmem + T_G, sdesc_kmajor(sAV + (s >> 2) * 16384 + 32 * (s & 3)),
                   sdesc_kmajor(bb + P.b_slab_off[s >> 2] + 32 * (s & 3)),
                   idesc_f16(128, nr, E::kBf16, false), s > 0);
          }
          mma_commit(&bars[B_GF + hh]);
          mma_commit(&bars[B_BE + 2 * hh + buf]);
        }
        if (!ok) break;
        if (w + 2 <= WL) ok = sd(w + 2);
      }
      mma_commit(&bars[B_DRAIN5]);
      mbar_wait(&bars[B_DRAIN5], 0, err, kErrDrain);
    }
  } else if (warp == 6) {
    // ---------------------------------- UMMA: the launch's own GEMMs
    if (lane == 0) {
      bool ok = mbar_wait(&bars[B_Q], 0, err, kErrQ);
      tc_fence_after();
      if (MODE == MODE_DQ) {
        const uint32_t id_x = idesc_f16(128, 64, E::kBf16, true);   // B = K^(m), MN-major
        const uint32_t id_g = idesc_f16(128, D, E::kBf16, true);    // B = K tile, MN-major
        for (int w = 0; ok && w <= WL; ++w) {
          const int buf = w % nb;
          const int n = w >> 1, st = n & 1;
          for (int hh = 0; hh < 2 && ok; ++hh) {
            ok = mbar_wait(&bars[hh ? B_YB : B_YA], w & 1, err, kErrY);
            // X is free once the rows have folded the previous window into dq
            if (ok && hh == 0 && w > 0) ok = mbar_wait(&bars[B_XFREE], (w - 1) & 1, err, kErrXFree);
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
          // gate part: dq += dS K_w  (A = dS from tensor memory, B = K tile)
          if (!(ok = mbar_wait(&bars[B_KVF + st], (n >> 1) & 1, err, kErrKvFull))) break;
          mma_ts(tmem + tq::DQ, tmem + tq::YT + 56,
                 sdesc_mnmajor(sK + st * NS * 4096 + (w & 1) * kW * 128, 4096), id_g, w > 0);
          mma_commit(&bars[B_XF]);
          mma_commit(&bars[B_YTFREE]);
          if (w & 1) mma_commit(&bars[B_KVE + st]);
        }
      } else {
        const uint32_t id_c = idesc_f16(128, 112, E::kBf16, true) | (1u << 15);  // A, B MN-major
        const uint32_t id_s = idesc_f16(128, 16, E::kBf16, true) | (1u << 15);
        for (int w = 0; ok && w <= WL; ++w) {
          for (int hh = 0; hh < 2 && ok; ++hh) {
            ok = mbar_wait(&bars[hh ? B_YB : B_YA], w & 1, err, kErrY);
            if (ok && w > 0) ok = mbar_wait(&bars[B_CE + hh], (w - 1) & 1, err, kErrCEmpty);
            if (!ok) break;
            tc_fence_after();
            const uint32_t creg = tmem + (hh ? tk::C1 : tk::C0);
#pragma unroll 1
            for (int s = 0; s < 8; ++s) {  // K = 128 query rows, 16 per step
              const uint32_t ko = 2048 * s;
              // C^T = v^T Y: A = v^T (M = head dim), B = Y^T (N = term x key)
              mma_ss(creg, sdesc_mnmajor(sAV + ko, 16384), sdesc_mnmajor(sY + ko, 16384), id_c,
                     s > 0);
              // dO^T (P | dS) and Q^T (P | dS): B = elements 112..127 of the rows
              mma_ss(creg + 112, sdesc_mnmajor(sDO + ko, 16384),
                     sdesc_mnmajor(sY + 16384 + ko + 96, 16384), id_s, s > 0);
              mma_ss(creg + 128, sdesc_mnmajor(sQ + ko, 16384),
                     sdesc_mnmajor(sY + 16384 + ko + 96, 16384), id_s, s > 0);
            }
            mma_commit(&bars[B_CF + hh]);
            mma_commit(&bars[hh ? B_YFREE : B_YDONE]);
            if (hh == 1) mma_commit(&bars[B_AVE]);
          }
          if (!ok) break;
          if (w & 1) mma_commit(&bars[B_KVE + ((w >> 1) & 1)]);
        }
      }
      mma_commit(&bars[B_DRAIN6]);
      mbar_wait(&bars[B_DRAIN6], 0, err, kErrDrain);
    }
  } else if (warp >= 8) {
    // ------------------------- K^(m) builder (+ per-dimension combine, dK launch)
    constexpr int kMaxItems = L::MAX_ITEMS;
    const int gt = tid - 256;
    uint2* items = reinterpret_cast<uint2*>(smem + L::ITEMS);
    int my_n = 0;
    {
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
          const int r = local >> 1, c = 2 * s2 + (local & 1), m = r >> 3, j = r & 7;
          const uint32_t kofs = (c >> 3) * 4096 + j * 128 + (((c & 7) ^ j) << 4);
          const uint32_t cofs = (m * NP + 4 * c) * 4;
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
        cm[m] = kLn2 * s_coef[m * NP + p] * sgn;
      }
    }
    const uint32_t lane_base = tmem + ((uint32_t)((warp - 8) * 32) << 16);
    float* dk32 = P.dk32 + ((int64_t)b * P.Hkv + hk) * S * D;
    float* dv32 = P.dv32 + ((int64_t)b * P.Hkv + hk) * S * D;

    auto build = [&](int w) -> bool {
      const int buf = w % nb, use = w / nb;
      const int n = w >> 1, st = n & 1;
      if (!mbar_wait(&bars[B_KVF + st], (n >> 1) & 1, err, kErrKvFull)) return false;
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        if (use > 0 && !mbar_wait(&bars[B_BE + 2 * hh + buf], (use - 1) & 1, err, kErrBEmpty))
          return false;
        const uint32_t kt = sK + st * NS * 4096 + (2 * (w & 1) + hh) * 1024;
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
              const uint32_t fl = d[j].y >> 16;
              const bool swp = fl & 1u;
              const float sre = (fl & 2u) ? -1.f : 1.f, sim = (fl & 4u) ? -1.f : 1.f;
              const uint32_t in[4] = {kv[j].x, kv[j].y, kv[j].z, kv[j].w};
              const float cfa[4] = {cf[j].x, cf[j].y, cf[j].z, cf[j].w};
              uint32_t out[4];
#pragma unroll
              for (int e2 = 0; e2 < 4; ++e2) {
                const float ke = E::lo(in[e2]), ko = E::hi(in[e2]);
                const float a = swp ? ko : ke, bq = swp ? ke : ko;
                out[e2] = E::pack(sre * cfa[e2] * a, sim * cfa[e2] * bq);
              }
              sts128(bt + (d[j].y & 0xffffu), make_uint4(out[0], out[1], out[2], out[3]));
            }
          }
        }
        fence_async_smem();
        mbar_arrive(&bars[B_BF + 2 * hh + buf]);
      }
      if (w & 1) mbar_arrive(&bars[B_KVE + st]);
      return true;
    };

    auto combine = [&](int w) -> bool {
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        if (!mbar_wait(&bars[B_CF + hh], w & 1, err, kErrC)) return false;
        tc_fence_after();
        const uint32_t creg = lane_base + (hh ? tk::C1 : tk::C0);
        float dk[8], dv[8];
        {
          uint32_t g[16];
          tmem_ld16(creg + 112, g);  // dO^T P (0..7) | dO^T dS (8..15)
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j) dv[j] = __uint_as_float(g[j]);
          tmem_ld16(creg + 128, g);  // Q^T P | Q^T dS (8..15)
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j) dk[j] = __uint_as_float(g[8 + j]);
        }
#pragma unroll
        for (int c = 0; c < kM / 2; ++c) {  // terms 2c, 2c+1 for the 8 keys
          uint32_t g[16];
          tmem_ld16(creg + 16 * c, g);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float own = __uint_as_float(g[j]);
            const float odd = __uint_as_float(g[8 + j]);
            const float partner = __shfl_xor_sync(0xffffffffu, odd, 1);
            dk[j] = fmaf(cm[2 * c], own, dk[j]);
            dk[j] = fmaf(cm[2 * c + 1], partner, dk[j]);
          }
        }
        tc_fence_before();
        mbar_arrive(&bars[B_CE + hh]);
        const int d = gt;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int key = w * kW + hh * 8 + j;
          if (key < S) {
            atomicAdd(dk32 + (int64_t)key * D + d, dk[j]);
            atomicAdd(dv32 + (int64_t)key * D + d, dv[j]);
          }
        }
      }
      return true;
    };

    bool ok = build(0);
    for (int w = 0; ok && w <= WL; ++w) {
      if (w + 1 <= WL) ok = build(w + 1);
      if (ok && MODE == MODE_DK) ok = combine(w);
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------ row warps
    const int r = tid;
    const int t = q0 + r;
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    const int64_t ri = ((int64_t)b * P.H + h) * S + min(t, S - 1);
    const float A_t = P.a[ri];
    const float lse2 = P.lse[ri] * kLog2e;
    const float delta = P.delta[ri];
    float base = 0.f;    // gate prefix before the window
    float da_run = 0.f;  // prefix of da before the current key
    bool ok = mbar_wait(&bars[B_Q], 0, err, kErrQ);

    // sin/cos of (carry + c0) theta for 16 pairs starting at pair 16 g
    auto angles = [&](float cw, int g, float (&sn)[16], float (&cs)[16]) {
      const float bse = cw + kC0;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const float4 t4 = lds128f(s_th_u + 16 * (g * 4 + cc));
        const float th[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float rr = reduce_2pi(bse * th[i]);
          __sincosf(rr, &sn[4 * cc + i], &cs[4 * cc + i]);
        }
      }
    };

    // A operand rows v = R((carry + c0) theta) q_t into shared memory
    auto build_a = [&](float cw) {
#pragma unroll 1
      for (int g = 0; g < NP / 16; ++g) {
        float sn[16], cs[16];
        angles(cw, g, sn, cs);
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int c = g * 4 + cc;
          const uint4 qv = lds128(sQ + (c >> 3) * 16384 + sw128_offset(r, c & 7));
          const uint32_t in[4] = {qv.x, qv.y, qv.z, qv.w};
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float qe = E::lo(in[i]), qo = E::hi(in[i]);
            const float s_ = sn[4 * cc + i], c_ = cs[4 * cc + i];
            o[i] = E::pack(qe * c_ - qo * s_, qe * s_ + qo * c_);
          }
          sts128(sAV + (c >> 3) * 16384 + sw128_offset(r, c & 7), make_uint4(o[0], o[1], o[2], o[3]));
        }
      }
      fence_async_smem();
      mbar_arrive(&bars[B_AVF]);
    };

    // Clenshaw: logits (log2 units) and their derivative in u for 8 keys
    auto clenshaw = [&](const float* uj, float* f, float* fd) {
      float b1[8], b2[8], d1[8], d2[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) { b1[j] = b2[j] = d1[j] = d2[j] = 0.f; }
#pragma unroll
      for (int c0 = kM / 2 - 1; c0 >= 0; c0 -= 2) {
        uint32_t g[2][16];
#pragma unroll
        for (int i = 0; i < 2; ++i)
          if (c0 - i >= 0) tmem_ld16(lane_base + T_G + 16 * (c0 - i), g[i]);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int c = c0 - i;
          if (c < 0) continue;
#pragma unroll
          for (int mm = 1; mm >= 0; --mm) {
            const int m = 2 * c + mm;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float a = __uint_as_float(g[i][mm * 8 + j]);
              const float u2 = 2.0f * uj[j];
              if (m > 0) {
                const float dn = fmaf(u2, d1[j], fmaf(2.0f, b1[j], -d2[j]));
                const float bn = fmaf(u2, b1[j], a - b2[j]);
                d2[j] = d1[j]; d1[j] = dn;
                b2[j] = b1[j]; b1[j] = bn;
              } else {
                f[j] = fmaf(uj[j], b1[j], a - b2[j]);
                fd[j] = fmaf(uj[j], d1[j], b1[j] - d2[j]);
              }
            }
          }
        }
      }
    };

    for (int w = 0; ok && w <= WL; ++w) {
      const int j0 = w * kW;
      // ---- gates, positions
      if (!(ok = mbar_wait(&bars[B_SDF + (w & 1)], (w >> 1) & 1, err, kErrSd))) break;
      tc_fence_after();
      float z[16], uu[16];
      {
        uint32_t sraw[16];
        tmem_ld16(lane_base + ((w & 1) ? T_SG1 : T_SG0), sraw);
        tmem_wait_ld();
        float zsum = 0.f;
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
          z[jj] = (j0 + jj <= t) ? sigmoid_f(__uint_as_float(sraw[jj])) : 0.f;
          zsum += z[jj];
        }
        float suf = 0.f;  // in-window suffix after key jj
#pragma unroll
        for (int jj = 15; jj >= 0; --jj) {
          uu[jj] = fmaf(suf, 1.0f / kC0, -1.0f);
          suf += z[jj];
        }
        base += zsum;
      }
      const float carry = A_t - base;  // gate sum of the keys after the window
      // ---- A operand (its buffer is free: the previous window's GEMMs that
      // read it have completed)
      if (MODE == MODE_DK && w > 0 && !(ok = mbar_wait(&bars[B_AVE], (w - 1) & 1, err, kErrAvEmpty)))
        break;
      build_a(carry);
      // ---- the two halves of the window
      float dpv[16];
      {
        uint32_t dr[16];
        tmem_ld16(lane_base + ((w & 1) ? T_DP1 : T_DP0), dr);
        tmem_wait_ld();
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) dpv[jj] = __uint_as_float(dr[jj]);
      }
      tc_fence_before();
      mbar_arrive(&bars[B_SDE + (w & 1)]);
      uint32_t dspk[8];  // dS (bf16 pairs) for the 16 keys
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        if (!(ok = mbar_wait(&bars[B_GF + hh], w & 1, err, kErrG))) break;
        tc_fence_after();
        float uj[8], f[8], fd[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) uj[j] = hh ? uu[8 + j] : uu[j];
        clenshaw(uj, f, fd);
        tc_fence_before();
        mbar_arrive(&bars[B_GE]);
        float dl[8], ds[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int jj = hh * 8 + j;
          const bool valid = j0 + jj <= t;
          float lg = f[j];
          if (HAS_BIAS && valid) lg = fmaf(P.bias[(int64_t)t * P.bias_rs + j0 + jj], kLog2e, lg);
          const float pr = valid ? exp2f(lg - lse2) : 0.f;
          dl[j] = pr * ((hh ? dpv[8 + j] : dpv[j]) - delta);
          const float da = dl[j] * (kLn2 / kC0) * fd[j];
          const float zj = hh ? z[8 + j] : z[j];
          ds[j] = valid ? da_run * zj * (1.f - zj) : 0.f;
          da_run += valid ? da : 0.f;
          f[j] = pr;  // keep P for the dK launch
        }
        // Y_m = dl T_m(u), packed per term for the 8 keys
        uint32_t y[kM][4];
#pragma unroll
        for (int jp = 0; jp < 4; ++jp) {
          float ta0 = 1.f, tb0 = 1.f;
          float ta1 = uj[2 * jp], tb1 = uj[2 * jp + 1];
          y[0][jp] = E::pack(dl[2 * jp], dl[2 * jp + 1]);
          y[1][jp] = E::pack(dl[2 * jp] * ta1, dl[2 * jp + 1] * tb1);
#pragma unroll
          for (int m = 2; m < kM; ++m) {
            const float ta2 = fmaf(2.f * uj[2 * jp], ta1, -ta0);
            const float tb2 = fmaf(2.f * uj[2 * jp + 1], tb1, -tb0);
            ta0 = ta1; ta1 = ta2; tb0 = tb1; tb1 = tb2;
            y[m][jp] = E::pack(dl[2 * jp] * ta2, dl[2 * jp + 1] * tb2);
          }
        }
#pragma unroll
        for (int jp = 0; jp < 4; ++jp) dspk[hh * 4 + jp] = E::pack(ds[2 * jp], ds[2 * jp + 1]);
        if (MODE == MODE_DQ) {
          // Y half into tensor memory (A operand of X); half B waits until X
          // has consumed half A, half A until the previous window's GEMMs are done
          if (hh == 0 && w > 0 && !(ok = mbar_wait(&bars[B_YTFREE], (w - 1) & 1, err, kErrX))) break;
          if (hh == 1 && !(ok = mbar_wait(&bars[B_YDONE], w & 1, err, kErrX))) break;
          tc_fence_after();
#pragma unroll
          for (int q = 0; q < 3; ++q) {
            uint32_t v16[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) v16[i] = y[(16 * q + i) >> 2][i & 3];
            tmem_st16(lane_base + tq::YT + 16 * q, v16);
          }
          {
            uint32_t v8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v8[i] = y[(48 + i) >> 2][i & 3];
            tmem_st8(lane_base + tq::YT + 48, v8);
          }
          if (hh == 1) {
            uint32_t v8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v8[i] = dspk[i];
            tmem_st8(lane_base + tq::YT + 56, v8);
          }
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(&bars[hh ? B_YB : B_YA]);
        } else {
          // Y | P | dS rows into shared memory (B operand of the C GEMMs)
          if (hh == 0 && w > 0 && !(ok = mbar_wait(&bars[B_YFREE], (w - 1) & 1, err, kErrY))) break;
          if (hh == 1 && !(ok = mbar_wait(&bars[B_YDONE], w & 1, err, kErrY))) break;
#pragma unroll
          for (int m = 0; m < kM; ++m)  // element m*8 + jj: chunk m of the row
            sts128(sY + (m >> 3) * 16384 + sw128_offset(r, m & 7),
                   make_uint4(y[m][0], y[m][1], y[m][2], y[m][3]));
          sts128(sY + 16384 + sw128_offset(r, 6),
                 make_uint4(E::pack(f[0], f[1]), E::pack(f[2], f[3]), E::pack(f[4], f[5]),
                            E::pack(f[6], f[7])));
          sts128(sY + 16384 + sw128_offset(r, 7),
                 make_uint4(dspk[hh * 4], dspk[hh * 4 + 1], dspk[hh * 4 + 2], dspk[hh * 4 + 3]));
          fence_async_smem();
          mbar_arrive(&bars[hh ? B_YB : B_YA]);
        }
      }
      if (!ok) break;
      if (MODE == MODE_DQ) {
        // ---- dq += ln2 R(-(carry + c0) theta) X   (X and the gate UMMA done)
        if (!(ok = mbar_wait(&bars[B_XF], w & 1, err, kErrX))) break;
        tc_fence_after();
#pragma unroll 1
        for (int g = 0; g < NP / 16; ++g) {
          float sn[16], cs[16];
          angles(carry, g, sn, cs);
          uint32_t xv[2][16], qv2[2][16];
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            tmem_ld16(lane_base + tq::X + 32 * g + 16 * i, xv[i]);
            tmem_ld16(lane_base + tq::DQ + 32 * g + 16 * i, qv2[i]);
          }
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 2; ++i) {
#pragma unroll
            for (int e2 = 0; e2 < 8; ++e2) {
              const int pl = 8 * i + e2;  // pair within the group
              const float xe = __uint_as_float(xv[i][2 * e2]), xo = __uint_as_float(xv[i][2 * e2 + 1]);
              const float c_ = cs[pl] * kLn2, s_ = sn[pl] * kLn2;
              qv2[i][2 * e2] = __float_as_uint(__uint_as_float(qv2[i][2 * e2]) + fmaf(c_, xe, s_ * xo));
              qv2[i][2 * e2 + 1] =
                  __float_as_uint(__uint_as_float(qv2[i][2 * e2 + 1]) + fmaf(c_, xo, -s_ * xe));
            }
            tmem_st16(lane_base + tq::DQ + 32 * g + 16 * i, qv2[i]);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bars[B_XFREE]);
      }
    }
    if (MODE == MODE_DQ && ok) {
      // all GEMMs into DQ are done (the last window's B_XF was waited above)
      T* dqrow = reinterpret_cast<T*>(P.dq) + b * P.dqs[0] + h * P.dqs[1] + (int64_t)t * P.dqs[2];
#pragma unroll 1
      for (int c = 0; c < D / 16; ++c) {
        uint32_t o[16];
        tmem_ld16(lane_base + tq::DQ + 16 * c, o);
        tmem_wait_ld();
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) pk[i] = E::pack(__uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1]));
        if (t < S) {
          uint4* dst = reinterpret_cast<uint4*>(dqrow + 16 * c);
          dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------------ host
template <int MODE>
static int plan(Params& p) {
  using L = SmemTail<MODE>;
  int off = 0;
  for (int s = 0; s < NS; ++s) {
    p.b_slab_off[s] = off;
    off += p.nrow[4 * s] * 128;
  }
  p.b_buf_bytes = (off + 1023) & ~1023;
  p.nb = (L::BOP + 4 * p.b_buf_bytes + 1024 <= kSmemLimit) ? 2 : 1;
  return L::BOP + 2 * p.nb * p.b_buf_bytes + 1024;
}

template <typename T, int MODE>
static cudaError_t launch_mode(Params& p, bool bias, int B, int H, int S, cudaStream_t st) {
  const int smem = plan<MODE>(p);
  if (smem > kSmemLimit) return cudaErrorInvalidValue;
  dim3 grid((S + kBM - 1) / kBM, H, B);
  cudaError_t e;
  if (bias) {
    auto kern = bwd_kernel<T, MODE, true>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) return e;
    kern<<<grid, kThreads, smem, st>>>(p);
  } else {
    auto kern = bwd_kernel<T, MODE, false>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) return e;
    kern<<<grid, kThreads, smem, st>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace tcb

static bool rows16(const void* ptr, const int64_t* st) {
  return (reinterpret_cast<uintptr_t>(ptr) % 16) == 0 && (st[0] * 2) % 16 == 0 &&
         (st[1] * 2) % 16 == 0 && (st[2] * 2) % 16 == 0;
}

bool tc_bwd_supported(const BwdArgs& a, int dtype) {
  if (dtype != COROPE_DTYPE_BF16 && dtype != COROPE_DTYPE_F16) return false;
  if (a.D != 128) return false;
  if (!rows16(a.q, a.qs) || !rows16(a.k, a.ks) || !rows16(a.v, a.vs) ||
      !rows16(a.dout, a.dos) || !rows16(a.dq, a.dqs))
    return false;
  return tcx::get_encoder() != nullptr;
}

// Launches the dQ and dK kernels; the caller runs the delta/lse pre-kernel
// before and the fp32 -> dtype conversion of dk/dv after.
cudaError_t tc_bwd_launch(const BwdArgs& a, int dtype, cudaStream_t st) {
  using namespace tcb;
  static Params p;
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  std::memset(&p, 0, sizeof(p));
  if (!tcx::encode(&p.tm_q, a.q, dtype, a.B, a.H, a.S, a.D, a.qs, kBM) ||
      !tcx::encode(&p.tm_do, a.dout, dtype, a.B, a.H, a.S, a.D, a.dos, kBM) ||
      !tcx::encode(&p.tm_k, a.k, dtype, a.B, a.Hkv, a.S, a.D, a.ks, kKT) ||
      !tcx::encode(&p.tm_v, a.v, dtype, a.B, a.Hkv, a.S, a.D, a.vs, kKT))
    return cudaErrorInvalidValue;
  p.dq = a.dq;
  p.dk32 = a.dk32;
  p.dv32 = a.dv32;
  p.lse = a.lse;
  p.delta = a.delta;
  p.a = a.a;
  p.thetas = a.thetas;
  p.theta = a.theta;
  p.bias = a.bias;
  p.bias_rs = a.bias_rs;
  for (int i = 0; i < 3; ++i) p.dqs[i] = a.dqs[i];
  p.B = a.B; p.H = a.H; p.Hkv = a.Hkv; p.S = a.S;
  tcx::fill_coefficients(p.coef, p.nrow, a.D, a.theta, a.sm_scale);
  const bool bias = a.bias != nullptr;
  cudaError_t e;
  if (dtype == COROPE_DTYPE_BF16) {
    e = launch_mode<__nv_bfloat16, MODE_DQ>(p, bias, a.B, a.H, a.S, st);
    if (e == cudaSuccess) e = launch_mode<__nv_bfloat16, MODE_DK>(p, bias, a.B, a.H, a.S, st);
  } else {
    e = launch_mode<__half, MODE_DQ>(p, bias, a.B, a.H, a.S, st);
    if (e == cudaSuccess) e = launch_mode<__half, MODE_DK>(p, bias, a.B, a.H, a.S, st);
  }
  return e;
}

}  // namespace corope
