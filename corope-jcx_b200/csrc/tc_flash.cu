// Plain (softmax) attention forward on the tcgen05 pipeline of the CoRoPE
// kernels -- the baseline that measures what the contextual positions cost.
// Same TMA staging, tensor-memory accumulators and bounded waits as the
// CoRoPE forward, without the gates, positions and rotation:
//     S = sm_scale * Q K^T,  P = softmax(S) (causal or not),  O = P V.
//
// Per CTA: 128 query rows of one (b, h), 320 threads.
//   warps 0-7  two softmax warpgroups; group g owns keys 64g .. 64g+63 of
//              every 128-key tile for all 128 rows (one row per thread),
//              with its own running max, row sum and O accumulator in tensor
//              memory, so the groups never wait for each other inside the
//              key loop; the two partial results are merged once at the end
//   warp 8     TMA: Q once, K/V tiles of 128 keys (2 stages, 128B swizzle)
//   warp 9     UMMA: S_j = Q K_j^T into one of two S buffers, then
//              O_g += P_g V_j per group (P_g in bf16/f16 over the group's own S
//              columns, read from tensor memory)
// Tensor memory (512 columns): S0, S1 (128 each), O_0, O_1 (D each).
// Softmax in log2 units with stale-max rescaling: O_g is rescaled only when
// the group's row max grows by more than 2^8.
#include <cmath>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "sm100.cuh"
#include "tc_common.cuh"

namespace corope {

// First error recorded by a bounded wait of the plain attention kernel.
__device__ int g_corope_flash_error = 0;

int tcf_take_device_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_corope_flash_error, sizeof(int)) != cudaSuccess) return -1;
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_corope_flash_error, &zero, sizeof(int));
  }
  return v;
}

namespace tcf {

using tcx::ElemTraits;
using tcx::kLog2e;
constexpr int kBM = 128;   // query rows per CTA
constexpr int kBN = 128;   // keys per tile
constexpr int kThreads = 320;
constexpr float kRescale = 8.0f;  // stale-max headroom (log2 units)

enum : int { kErrQ = 301, kErrKvFull, kErrKvEmpty, kErrS, kErrP, kErrPv, kErrX, kErrDrain };

struct Params {
  CUtensorMap tm_q, tm_k, tm_v;
  void* o;
  float *m, *lse;
  int64_t os[3];
  int B, H, Hkv, S, Sk;
  float scale2;  // sm_scale * log2(e)
  float sm_scale;
};

template <int D>
struct Layout {
  static constexpr int NS = D / 64;               // 64-element slabs
  static constexpr int Q = 0;                     // [NS][128 rows][128 B]
  static constexpr int K = Q + NS * 16384;        // [2 stages][NS][128 keys][128 B]
  static constexpr int V = K + 2 * NS * 16384;
  static constexpr int BAR = V + 2 * NS * 16384;
  static constexpr int SLOT = BAR + 16 * 8;
  static constexpr int XCH = SLOT + 16;           // [3 values][2 groups][128 rows] fp32
  static constexpr int TOTAL = XCH + 3 * 2 * 128 * 4;
  // tensor-memory columns
  static constexpr uint32_t T_S0 = 0, T_S1 = 128, T_O0 = 256, T_O1 = 256 + D;
  static_assert(T_O1 + D <= 512, "tensor memory");
};

enum { B_Q = 0, B_KVF = 1, B_KVE = 3, B_SF = 5, B_PF = 7 /* [buf][group] */, B_PVD = 11,
       B_X = 13, B_DRAIN = 14 };

template <typename T, int D, bool CAUSAL>
__global__ void __launch_bounds__(kThreads, 1) flash_fwd_kernel(const __grid_constant__ Params P) {
  using L = Layout<D>;
  using E = ElemTraits<T>;
  using namespace sm100;
  constexpr int NS = L::NS;
  constexpr int KSTEPS = D / 16;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + L::SLOT);
  float* xch = reinterpret_cast<float*>(smem + L::XCH);
  int* err = &g_corope_flash_error;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qt = gridDim.x - 1 - blockIdx.x;  // longest query tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (P.H / P.Hkv);
  const int q0 = qt * kBM;
  // key tiles: up to the diagonal (causal) or all keys
  const int last_key = CAUSAL ? min(P.Sk, q0 + kBM) - 1 : P.Sk - 1;
  const int NT = last_key / kBN + 1;

  if (tid == 0) {
    mbar_init(&bars[B_Q], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[B_KVF + i], 1);
      mbar_init(&bars[B_KVE + i], 1);
      mbar_init(&bars[B_SF + i], 1);
      mbar_init(&bars[B_PVD + i], 1);
      mbar_init(&bars[B_PF + 2 * i], 128);
      mbar_init(&bars[B_PF + 2 * i + 1], 128);
    }
    mbar_init(&bars[B_X], 256);
    mbar_init(&bars[B_DRAIN], 1);
    fence_mbar_init();
  }
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

  if (warp == 8) {
    // -------------------------------------------------------------- TMA
    if (lane == 0) {
      prefetch_tmap(&P.tm_q);
      prefetch_tmap(&P.tm_k);
      prefetch_tmap(&P.tm_v);
      mbar_expect_tx(&bars[B_Q], NS * 16384);
      for (int s = 0; s < NS; ++s)
        tma_load_4d(smem + L::Q + s * 16384, &P.tm_q, &bars[B_Q], 64 * s, q0, h, b);
      int last_use[2] = {-1, -1};
      for (int j = 0; j < NT; ++j) {
        const int st = j & 1, u = j >> 1;
        if (j >= 2 && !mbar_wait(&bars[B_KVE + st], (u - 1) & 1, err, kErrKvEmpty)) break;
        mbar_expect_tx(&bars[B_KVF + st], 2 * NS * 16384);
        for (int s = 0; s < NS; ++s) {
          tma_load_4d(smem + L::K + (st * NS + s) * 16384, &P.tm_k, &bars[B_KVF + st], 64 * s,
                      kBN * j, hk, b);
          tma_load_4d(smem + L::V + (st * NS + s) * 16384, &P.tm_v, &bars[B_KVF + st], 64 * s,
                      kBN * j, hk, b);
        }
        last_use[st] = u;
      }
      // no copy may still be in flight when the CTA exits
      mbar_wait(&bars[B_Q], 0, err, kErrDrain);
      for (int st = 0; st < 2; ++st)
        if (last_use[st] >= 0) mbar_wait(&bars[B_KVF + st], last_use[st] & 1, err, kErrDrain);
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------- UMMA
    if (lane == 0) {
      const uint32_t id_s = idesc_f16(128, kBN, E::kBf16, false);
      const uint32_t id_pv = idesc_f16(128, D, E::kBf16, true);  // B = V tile, MN-major
      // O_g += P_g V_j: A = P_g (group g's 64 keys, 16-bit, over its S
      // columns), B = rows 64g.. of the V tile, K = 16 keys per step
      auto pv = [&](int j) -> bool {
        const int sb = j & 1, st = j & 1;
        const uint32_t sreg = tmem + (sb ? L::T_S1 : L::T_S0);
        for (int g = 0; g < 2; ++g) {
          if (!mbar_wait(&bars[B_PF + 2 * sb + g], (j >> 1) & 1, err, kErrP)) return false;
          tc_fence_after();
          const uint32_t vt = sV + st * NS * 16384 + g * 8192;
#pragma unroll
          for (int s = 0; s < 4; ++s)
            mma_ts(tmem + (g ? L::T_O1 : L::T_O0), sreg + 64 * g + 8 * s,
                   sdesc_mnmajor(vt + 2048 * s, 16384), id_pv, (j > 0 || s > 0) ? 1u : 0u);
        }
        mma_commit(&bars[B_PVD + sb]);
        mma_commit(&bars[B_KVE + st]);
        return true;
      };
      bool ok = mbar_wait(&bars[B_Q], 0, err, kErrQ);
      for (int j = 0; ok && j < NT; ++j) {
        const int st = j & 1, sb = j & 1;
        ok = mbar_wait(&bars[B_KVF + st], (j >> 1) & 1, err, kErrKvFull);
        // the S buffer's previous P has been read by its PV GEMMs
        if (ok && j >= 2) ok = mbar_wait(&bars[B_PVD + sb], ((j >> 1) - 1) & 1, err, kErrPv);
        if (!ok) break;
        tc_fence_after();
        const uint32_t kt = sK + st * NS * 16384;
#pragma unroll
        for (int s = 0; s < KSTEPS; ++s)
          mma_ss(tmem + (sb ? L::T_S1 : L::T_S0), sdesc_kmajor(sQ + (s >> 2) * 16384 + 32 * (s & 3)),
                 sdesc_kmajor(kt + (s >> 2) * 16384 + 32 * (s & 3)), id_s, s > 0);
        mma_commit(&bars[B_SF + sb]);
        if (j >= 1) ok = pv(j - 1);
      }
      if (ok) pv(NT - 1);
      mma_commit(&bars[B_DRAIN]);
      mbar_wait(&bars[B_DRAIN], 0, err, kErrDrain);
    }
  } else {
    // ----------------------------------------------------- softmax rows
    const int g = warp >> 2;  // group: keys 64g .. 64g+63 of each tile
    const int r = tid & 127;
    const int t = q0 + r;
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t t_o = g ? L::T_O1 : L::T_O0;
    float m_used = -INFINITY, m_true = -INFINITY, lsum = 0.f;
    bool ok = true;
    for (int j = 0; ok && j < NT; ++j) {
      const int sb = j & 1;
      const uint32_t sreg = lane_base + (sb ? L::T_S1 : L::T_S0) + 64 * g;
      if (!(ok = wwait(bars[B_SF + sb], (j >> 1) & 1, err, kErrS))) break;
      tc_fence_after();
      uint32_t s[64];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld16(sreg + 16 * c, *reinterpret_cast<uint32_t(*)[16]>(s + 16 * c));
      tmem_wait_ld();
      const int k0 = kBN * j + 64 * g;  // this group's first key of the tile
      // keys past the row (causal) or past the sequence are masked
      const bool masked = (CAUSAL && k0 + 63 > q0) || k0 + 63 >= P.Sk;
      float mx = -INFINITY;
      if (masked) {
        const int lim = CAUSAL ? min(t, P.Sk - 1) : P.Sk - 1;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          if (k0 + i > lim) s[i] = __float_as_uint(-INFINITY);
          mx = fmaxf(mx, __uint_as_float(s[i]));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) mx = fmaxf(mx, __uint_as_float(s[i]));
      }
      const float mx2 = mx * P.scale2;
      m_true = fmaxf(m_true, mx2);
      const bool resc = mx2 > m_used + kRescale;
      const float m_new = resc ? mx2 : m_used;
      if (__any_sync(0xffffffffu, resc) && j > 0) {
        // O_g must not be in flight: the previous tile's PV GEMMs are done
        if (!(ok = wwait(bars[B_PVD + ((j - 1) & 1)], ((j - 1) >> 1) & 1, err, kErrPv))) break;
        tc_fence_after();
        const float alpha = exp2f(m_used - m_new);
#pragma unroll 1
        for (int c = 0; c < D / 16; ++c) {
          uint32_t o[16];
          tmem_ld16(lane_base + t_o + 16 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st16(lane_base + t_o + 16 * c, o);
        }
        lsum *= alpha;
      }
      m_used = m_new;
      // P = 2^(s * scale2 - m) as 16-bit pairs over this group's first 32 S
      // columns (its own scores, already read).  A row that has seen no key
      // yet (m = -inf) has only masked scores here: subtract 0, not -inf.
      const float msub = m_used == -INFINITY ? 0.f : m_used;
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float p0 = exp2f(fmaf(__uint_as_float(s[2 * i]), P.scale2, -msub));
        const float p1 = exp2f(fmaf(__uint_as_float(s[2 * i + 1]), P.scale2, -msub));
        lsum += p0 + p1;
        pk[i] = E::pack(p0, p1);
      }
      tmem_st16(sreg, *reinterpret_cast<uint32_t(*)[16]>(pk));
      tmem_st16(sreg + 16, *reinterpret_cast<uint32_t(*)[16]>(pk + 16));
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars[B_PF + 2 * sb + g]);
    }
    // ---- epilogue: merge the two groups' partial results
    if (ok) ok = wwait(bars[B_PVD + ((NT - 1) & 1)], ((NT - 1) >> 1) & 1, err, kErrPv);
    xch[(0 * 2 + g) * 128 + r] = m_used;
    xch[(1 * 2 + g) * 128 + r] = lsum;
    xch[(2 * 2 + g) * 128 + r] = m_true;
    mbar_arrive(&bars[B_X]);
    if (ok) ok = wwait(bars[B_X], 0, err, kErrX);
    if (ok) {
      tc_fence_after();
      const float mu[2] = {xch[0 * 128 + r], xch[1 * 128 + r]};
      const float ls[2] = {xch[2 * 128 + r], xch[3 * 128 + r]};
      const float mt = fmaxf(xch[4 * 128 + r], xch[5 * 128 + r]);
      const float m = fmaxf(mu[0], mu[1]);
      const float f0 = mu[0] == -INFINITY ? 0.f : exp2f(mu[0] - m);
      const float f1 = mu[1] == -INFINITY ? 0.f : exp2f(mu[1] - m);
      const float ltot = ls[0] * f0 + ls[1] * f1;
      const float inv = 1.0f / ltot;
      const float c0 = f0 * inv, c1 = f1 * inv;
      T* orow = reinterpret_cast<T*>(P.o) + b * P.os[0] + h * P.os[1] + (int64_t)t * P.os[2] +
                g * (D / 2);
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {  // this group's half of the output columns
        const int col = g * (D / 2) + 16 * c;
        uint32_t a[16], bb[16];
        tmem_ld16(lane_base + L::T_O0 + col, a);
        tmem_ld16(lane_base + L::T_O1 + col, bb);
        tmem_wait_ld();
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          pk[i] = E::pack(fmaf(__uint_as_float(a[2 * i]), c0, __uint_as_float(bb[2 * i]) * c1),
                          fmaf(__uint_as_float(a[2 * i + 1]), c0,
                               __uint_as_float(bb[2 * i + 1]) * c1));
        if (t < P.S) {
          uint4* dst = reinterpret_cast<uint4*>(orow + 16 * c);
          dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
      if (t < P.S && g == 0) {
        const int64_t ri = ((int64_t)b * P.H + h) * P.S + t;
        const float M = mt / kLog2e;  // row max of sm_scale * q.k
        if (P.m) P.m[ri] = M;
        if (P.lse) P.lse[ri] = M + logf(ltot * exp2f(m - mt));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

template <typename T, int D, bool CAUSAL>
static cudaError_t launch(const Params& p, dim3 grid, cudaStream_t st) {
  constexpr int smem = Layout<D>::TOTAL + 1024;
  auto kern = flash_fwd_kernel<T, D, CAUSAL>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, smem, st>>>(p);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t launch_d(const Params& p, bool causal, dim3 grid, cudaStream_t st) {
  return causal ? launch<T, D, true>(p, grid, st) : launch<T, D, false>(p, grid, st);
}

}  // namespace tcf

static bool rows16(const void* ptr, const int64_t* st) {
  return (reinterpret_cast<uintptr_t>(ptr) % 16) == 0 && (st[0] * 2) % 16 == 0 &&
         (st[1] * 2) % 16 == 0 && (st[2] * 2) % 16 == 0;
}

bool tc_flash_supported(const FwdArgs& a, int dtype) {
  if (dtype != COROPE_DTYPE_BF16 && dtype != COROPE_DTYPE_F16) return false;
  if (a.D != 64 && a.D != 128) return false;
  if (!rows16(a.q, a.qs) || !rows16(a.k, a.ks) || !rows16(a.v, a.vs) || !rows16(a.o, a.os))
    return false;
  return tcx::get_encoder() != nullptr;
}

cudaError_t tc_flash_launch(const FwdArgs& a, int dtype, bool causal, cudaStream_t st) {
  using namespace tcf;
  static Params p;  // holds three tensor maps; filled per call under a lock
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  std::memset(&p, 0, sizeof(p));
  if (!tcx::encode(&p.tm_q, a.q, dtype, a.B, a.H, a.S, a.D, a.qs, kBM) ||
      !tcx::encode(&p.tm_k, a.k, dtype, a.B, a.Hkv, a.Sk, a.D, a.ks, kBN) ||
      !tcx::encode(&p.tm_v, a.v, dtype, a.B, a.Hkv, a.Sk, a.D, a.vs, kBN))
    return cudaErrorInvalidValue;
  p.o = a.o;
  p.m = a.m;
  p.lse = a.lse;
  for (int i = 0; i < 3; ++i) p.os[i] = a.os[i];
  p.B = a.B; p.H = a.H; p.Hkv = a.Hkv; p.S = a.S; p.Sk = a.Sk;
  p.sm_scale = a.sm_scale;
  p.scale2 = a.sm_scale * kLog2e;
  dim3 grid((a.S + kBM - 1) / kBM, a.H, a.B);
  const bool bf = dtype == COROPE_DTYPE_BF16;
  if (a.D == 64)
    return bf ? launch_d<__nv_bfloat16, 64>(p, causal, grid, st)
              : launch_d<__half, 64>(p, causal, grid, st);
  return bf ? launch_d<__nv_bfloat16, 128>(p, causal, grid, st)
            : launch_d<__half, 128>(p, causal, grid, st);
}

}  // namespace corope
