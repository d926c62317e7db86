// Pieces shared by the tensor-core CoRoPE kernels (forward and backward):
// the windowed Chebyshev expansion constants, 16-bit element helpers, and the
// host-side tensor-map encoding and expansion coefficients.
#pragma once

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "sm100.cuh"

namespace corope {
namespace tcx {

constexpr int kW = 16;       // keys per window
constexpr int kM = 14;       // Chebyshev terms
constexpr float kC0 = 7.5f;  // (kW - 1) / 2: window centre
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kSmemLimit = 232448;  // opt-in dynamic shared memory per block

// Key slots of a half window.  The G GEMM's columns, the scaled-key panels and
// the row groups see the 8 keys of a half window in slot order: slot s holds
// key slot_key(s) of the half, and row group g takes slots 4g .. 4g + 3 --
// key pairs (0, 1) and (6, 7) for group 0, (2, 3) and (4, 5) for group 1 --
// so that with the per-offset term counts below both groups and both key
// pairs of a group run similar numbers of terms.
__host__ __device__ constexpr int slot_key(int s) { return s < 2 ? s : s < 4 ? s + 4 : s - 2; }

// Per-offset expansions (launches with scaled-key panels).  Key o of a window
// (0 .. 15, ascending) sits at a_tj = C_t + s_o with s_o, the gate sum of the
// window's keys after it, in [0, 15 - o]: its expansion is centred at
// C_t + c_o with half-width c_o = (15 - o) / 2 instead of the window's c0, so
// it needs fewer terms the later the key.  The term counts keep the
// truncation error of the value (and, for the 16-term backward, of its
// position derivative, for which the last key keeps c = 1/2) at or below that
// of the uniform expansion at c0.  The shift from the window centre,
// exp(i (c0 - c_o) theta_p), is folded into the panels.
__host__ __device__ constexpr int offset_terms(int km, int o) {
  return km == 16 ? (o < 2 ? 16 : o == 2 ? 15 : o < 5 ? 14 : o == 5 ? 13 : o < 8 ? 12
                     : o == 8 ? 11 : o == 9 ? 10 : o == 10 ? 9 : o == 11 ? 8 : o == 12 ? 7
                     : o == 13 ? 6 : 5)
                  : (o < 2 ? 14 : o < 4 ? 13 : o == 4 ? 12 : o < 7 ? 11 : o == 7 ? 10
                     : o == 8 ? 9 : o < 11 ? 8 : o == 11 ? 7 : o == 12 ? 6 : o == 13 ? 5
                     : o == 14 ? 4 : 1);
}
__host__ __device__ constexpr float offset_halfwidth(int km, int o) {
  return km == 16 && o == 15 ? 0.5f : 0.5f * (15 - o);
}
__host__ __device__ constexpr float offset_inv_halfwidth(int km, int o) {
  return offset_halfwidth(km, o) > 0.f ? 1.0f / offset_halfwidth(km, o) : 0.f;
}
// The backward's key slots: slot s of half hh holds window key
// bwd_slot_key(hh, s) = (s & 1) + 2 (s >> 2) + 4 hh + 8 ((s >> 1) & 1), so row
// group g takes key pairs (4 hh + 2 g, +1) and (8 + 4 hh + 2 g, +1): both
// halves of a window see the same offsets' term counts (the pairs of keys
// 0..7 and of keys 8..15), one instance of the per-pair code serves both.
__host__ __device__ constexpr int bwd_slot_key(int hh, int s) {
  return (s & 1) + 2 * (s >> 2) + 4 * hh + 8 * ((s >> 1) & 1);
}

// Terms a row group runs for position j (0..3) of half hh: the larger count
// of the two groups' keys there (the smaller one's extra terms are zero).
__host__ __device__ constexpr int position_terms(int km, int hh, int j) {
  return offset_terms(km, 8 * hh + slot_key(j)) > offset_terms(km, 8 * hh + slot_key(4 + j))
             ? offset_terms(km, 8 * hh + slot_key(j))
             : offset_terms(km, 8 * hh + slot_key(4 + j));
}

template <typename T> struct ElemTraits;
template <> struct ElemTraits<__nv_bfloat16> {
  static constexpr bool kBf16 = true;
  __device__ static float lo(uint32_t x) { return __uint_as_float(x << 16); }
  __device__ static float hi(uint32_t x) { return __uint_as_float(x & 0xffff0000u); }
  // -hi(x): the sign flip folded into the same logic operation
  __device__ static float nhi(uint32_t x) { return __uint_as_float((x & 0xffff0000u) ^ 0x80000000u); }
  __device__ static uint32_t pack(float a, float b) { return sm100::pack_bf16(a, b); }
};
template <> struct ElemTraits<__half> {
  static constexpr bool kBf16 = false;
  __device__ static float lo(uint32_t x) {
    return __half2float(__ushort_as_half((unsigned short)(x & 0xffffu)));
  }
  __device__ static float hi(uint32_t x) {
    return __half2float(__ushort_as_half((unsigned short)(x >> 16)));
  }
  __device__ static float nhi(uint32_t x) {
    return __half2float(__ushort_as_half((unsigned short)((x >> 16) ^ 0x8000u)));
  }
  __device__ static uint32_t pack(float a, float b) { return sm100::pack_f16(a, b); }
};

// Angles a * th[i] of 16 rotation pairs, two per packed fp32x2 multiply (the
// same single rounding as a scalar product).
__device__ __forceinline__ void angles16(float a, const float (&th)[16], float (&rr)[16]) {
  const float2 a2 = make_float2(a, a);
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    const float2 x = __fmul2_rn(a2, make_float2(th[i], th[i + 1]));
    rr[i] = x.x;
    rr[i + 1] = x.y;
  }
}

// The A operand's rotation of 16 pairs: pair i of the row, the 16-bit word
// (q_e, q_o) at word i of qv, becomes (q_e c - q_o s, q_e s + q_o c) with
// s, c = sn[i], cs[i], rounded to 16 bits.  Two pairs per packed fp32x2
// multiply and FMA (each component one product then one FMA, as the scalar
// form rounds); -q_o comes from its own unpack, so no operand is negated.
template <typename E>
__device__ __forceinline__ void rotate16(const uint4 (&qv)[4], const float (&sn)[16],
                                         const float (&cs)[16], uint32_t (&o)[16]) {
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    const uint4& v = qv[i >> 2];
    const uint32_t w0 = (i & 3) == 0 ? v.x : v.z;
    const uint32_t w1 = (i & 3) == 0 ? v.y : v.w;
    const float2 qe = make_float2(E::lo(w0), E::lo(w1));
    const float2 qo = make_float2(E::hi(w0), E::hi(w1));
    const float2 nqo = make_float2(E::nhi(w0), E::nhi(w1));
    const float2 c = make_float2(cs[i], cs[i + 1]);
    const float2 sv = make_float2(sn[i], sn[i + 1]);
    const float2 x = __ffma2_rn(nqo, sv, __fmul2_rn(qe, c));
    const float2 y = __ffma2_rn(qo, c, __fmul2_rn(qe, sv));
    o[i] = E::pack(x.x, y.x);
    o[i + 1] = E::pack(x.y, y.y);
  }
}

__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + __expf(-x)); }

// ------------------------------------------------------------------ host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn get_encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// [B, H, S, D] 16-bit tensor (element strides) -> 4-D map, {64, rows} box,
// 128-byte swizzle
inline bool encode(CUtensorMap* m, const void* ptr, int dtype, int B, int H, int S, int D,
                   const int64_t* st, int box_rows) {
  EncodeTiledFn enc = get_encoder();
  if (!enc) return false;
  const cuuint64_t es = 2;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)st[2] * es, (cuuint64_t)st[1] * es,
                           (cuuint64_t)st[0] * es};
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, dtype == COROPE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   4, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// K^(m) panels [npanels][rows][64] (16-bit, contiguous) -> 3-D map with a
// {64, rows, 1} box and 128-byte swizzle: one load fills one slab of a
// B-operand buffer exactly as the in-kernel builders lay it out.
inline bool encode_panels(CUtensorMap* m, const void* ptr, int dtype, int rows, int64_t npanels) {
  EncodeTiledFn enc = get_encoder();
  if (!enc || rows <= 0 || rows > 256) return false;
  cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)npanels};
  cuuint64_t strides[2] = {128, (cuuint64_t)rows * 128};
  cuuint32_t box[3] = {64, (cuuint32_t)rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, dtype == COROPE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Bessel function of the first kind, integer order, by its power series
// (|x| <= 8 here, where the series converges quickly in double precision).
__host__ __device__ inline double bessel_j(int m, double x) {
  double term = 1.0;
  for (int i = 1; i <= m; ++i) term *= (x / 2.0) / i;
  double sum = term;
  const double q = -(x * x) / 4.0;
  for (int k = 1; k < 80; ++k) {
    term *= q / (k * (double)(k + m));
    sum += term;
    if (fabs(term) < 1e-18 * fabs(sum) + 1e-300) break;
  }
  return sum;
}

// Chebyshev coefficients eps_m J_m(c0 theta_p) * sm_scale * log2(e) of the
// first KM terms and the pruned K extent of each term: nrow[s] = rows of the K^(m) operand that
// K-step s (16 head dims) reads (8 keys per term, rounded to 16 rows).
template <int KM = kM>
inline void fill_coefficients(float (*coef)[64], int* nrow, int D, float theta, float sm_scale) {
  // KM x D/2 Bessel functions per call (tens of microseconds of host time,
  // several times per backward call): kept per (KM, D, theta, sm_scale)
  struct Entry { int D; float theta, sm_scale; int nrow[8]; float coef[KM][64]; };
  static std::mutex mu;
  static Entry cache[8];
  static int ncache = 0;
  {
    std::lock_guard<std::mutex> g(mu);
    for (int i = 0; i < ncache; ++i)
      if (cache[i].D == D && cache[i].theta == theta && cache[i].sm_scale == sm_scale) {
        std::memcpy(nrow, cache[i].nrow, sizeof(cache[i].nrow));
        std::memcpy(coef, cache[i].coef, sizeof(cache[i].coef));
        return;
      }
  }
  const int NP = D / 2;
  int kd[KM];
  for (int m = 0; m < KM; ++m) {
    int need = 0;
    for (int q = 0; q < NP; ++q) {
      const double th = 1.0 / std::pow((double)theta, (double)(2 * q) / (double)D);
      const double beta = (m == 0 ? 1.0 : 2.0) * bessel_j(m, kC0 * th);
      coef[m][q] = (float)(beta * sm_scale * kLog2e);
      if (std::fabs(beta) > 2e-6) need = q + 1;
    }
    for (int q = NP; q < 64; ++q) coef[m][q] = 0.f;
    kd[m] = std::max(1, (2 * need + 15) / 16);
  }
  for (int m = KM - 2; m >= 0; --m) kd[m] = std::max(kd[m], kd[m + 1]);
  for (int s = 0; s < 8; ++s) {
    int nm = 0;
    for (int m = 0; m < KM; ++m) nm += kd[m] > s;
    nm = (nm + 1) & ~1;
    nrow[s] = (s < D / 16) ? 8 * nm : 0;
  }
  std::lock_guard<std::mutex> g(mu);
  Entry& e = cache[ncache < 8 ? ncache++ : 7];
  e.D = D;
  e.theta = theta;
  e.sm_scale = sm_scale;
  std::memcpy(e.nrow, nrow, sizeof(e.nrow));
  std::memcpy(e.coef, coef, sizeof(e.coef));
}

// The same K extents for the per-offset expansions of the panels: term m of
// key offset o has coefficient eps_m J_m(c_o theta_p) for m below the
// offset's count, zero above.
// The scan evaluates 16 x KM x D/2 Bessel functions (about a millisecond of
// host time), so its result is kept per (KM, D, theta).
template <int KM>
inline void fill_offset_rows(int* nrow, int D, float theta) {
  struct Entry { int D; float theta; int nrow[8]; };
  static std::mutex mu;
  static Entry cache[16];
  static int ncache = 0;
  {
    std::lock_guard<std::mutex> g(mu);
    for (int i = 0; i < ncache; ++i)
      if (cache[i].D == D && cache[i].theta == theta) {
        std::memcpy(nrow, cache[i].nrow, sizeof(cache[i].nrow));
        return;
      }
  }
  const int NP = D / 2;
  int kd[KM];
  for (int m = 0; m < KM; ++m) {
    int need = 0;
    for (int o = 0; o < 16; ++o) {
      if (m >= offset_terms(KM, o)) continue;
      for (int q = 0; q < NP; ++q) {
        const double th = 1.0 / std::pow((double)theta, (double)(2 * q) / (double)D);
        const double beta =
            (m == 0 ? 1.0 : 2.0) * bessel_j(m, (double)offset_halfwidth(KM, o) * th);
        if (std::fabs(beta) > 2e-6) need = std::max(need, q + 1);
      }
    }
    kd[m] = std::max(1, (2 * need + 15) / 16);
  }
  for (int m = KM - 2; m >= 0; --m) kd[m] = std::max(kd[m], kd[m + 1]);
  for (int s = 0; s < 8; ++s) {
    int nm = 0;
    for (int m = 0; m < KM; ++m) nm += kd[m] > s;
    nm = (nm + 1) & ~1;
    nrow[s] = (s < D / 16) ? 8 * nm : 0;
  }
  std::lock_guard<std::mutex> g(mu);
  Entry& e = cache[ncache < 16 ? ncache++ : 15];
  e.D = D;
  e.theta = theta;
  std::memcpy(e.nrow, nrow, sizeof(e.nrow));
}

// ------------------------------------------------------------------
// K^(m) panels in global memory.  The scaled keys K^(m)_j (term m, key j)
// depend on the keys alone, so every query tile of a (b, kv head) -- and for
// MQA every query head -- reads the same B operands.  One launch writes them
// once per call, in the row order the kernels use (row 8 m + j of a half
// window's 8 keys), as [b * Hkv + hk][half window][slab rows][64] panels per
// 64-element slab; the kernels then load each half window's operand with one
// 3-D TMA copy per slab instead of rebuilding it in every CTA.
constexpr int kPanelTerms = 16;  // most terms any kernel uses

struct PanelArgs {
  const void* k;
  int64_t ks[3];
  int B, Hkv, S;
  int nhw;          // half windows per (b, hk): 2 * ceil(S / 16)
  int rows[2];      // panel rows per slab (the slab's first K step's count)
  int nrow[8];      // rows each K step reads (multiples of 16)
  void* out[2];     // slab panels
  float coef[kPanelTerms][64];
};

inline int64_t panel_count(int B, int Hkv, int S) {
  return (int64_t)B * Hkv * 2 * ((S + kW - 1) / kW);
}

// Row r of K step s (16 elements = two 16-byte chunks) holds term m = r / 8 of
// key j = r % 8: coef_m(p) times the key's pair p, swapped for odd m and with
// the signs of (-i)^m, exactly as the in-kernel builders compute it; rows a K
// step does not read (past nrow[s]) and keys past S are zero.
template <typename T, int D>
__global__ void __launch_bounds__(128) panel_kernel(const __grid_constant__ PanelArgs A) {
  using E = ElemTraits<T>;
  const int hw = blockIdx.x, bh = blockIdx.y;
  const int b = bh / A.Hkv, hk = bh % A.Hkv;
  const T* kb = static_cast<const T*>(A.k) + b * A.ks[0] + hk * A.ks[1];
#pragma unroll
  for (int s = 0; s < D / 64; ++s) {
    const int rows = A.rows[s];
    uint4* out = static_cast<uint4*>(A.out[s]) + ((int64_t)bh * A.nhw + hw) * rows * 8;
    for (int it = threadIdx.x; it < rows * 8; it += 128) {
      const int r = it >> 3, c = it & 7, m = r >> 3, j = r & 7;
      const int key = 8 * hw + j;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (r < A.nrow[4 * s + (c >> 1)] && key < A.S && m < kPanelTerms) {
        const uint4 kv = *reinterpret_cast<const uint4*>(kb + (int64_t)key * A.ks[2] + 64 * s + 8 * c);
        const uint32_t sel = (m & 1) ? 0x1032u : 0x3210u;
        const uint32_t sgn = ((m & 2) ? 0x8000u : 0u) | (((m + 1) & 2) ? 0x80000000u : 0u);
        const uint32_t in[4] = {kv.x, kv.y, kv.z, kv.w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float cf = A.coef[m][32 * s + 4 * c + e];
          const uint32_t wv = __byte_perm(in[e], 0u, sel) ^ sgn;
          o[e] = E::pack(cf * E::lo(wv), cf * E::hi(wv));
        }
        v = make_uint4(o[0], o[1], o[2], o[3]);
      }
      out[it] = v;
    }
  }
}

// Fill the panel arguments for KM terms (coefficients and row counts from
// fill_coefficients) and return the panel bytes of both slabs (0 when the
// head dim has none).
template <int KM>
inline size_t panel_bytes(int B, int Hkv, int S, int D, float theta, float sm_scale,
                          PanelArgs* a = nullptr) {
  PanelArgs local;
  PanelArgs& p = a ? *a : local;
  std::memset(&p, 0, sizeof(p));
  float coef[kPanelTerms][64];
  fill_coefficients<KM>(coef, p.nrow, D, theta, sm_scale);
  for (int m = 0; m < kPanelTerms; ++m)
    for (int q = 0; q < 64; ++q) p.coef[m][q] = m < KM ? coef[m][q] : 0.f;
  p.rows[0] = p.nrow[0];
  p.rows[1] = D == 128 ? p.nrow[4] : 0;
  p.B = B; p.Hkv = Hkv; p.S = S;
  p.nhw = 2 * ((S + kW - 1) / kW);
  return (size_t)panel_count(B, Hkv, S) * (p.rows[0] + p.rows[1]) * 128;
}


// ------------------------------------------------------------------
// Scaled-key panels of the per-offset expansions (the forward's).  Term m
// of the key at offset o of its window is
//   eps_m J_m(c_o theta_p) * sm_scale * log2(e) * (-i)^m * exp(i (c0 - c_o) theta_p)
// times the key's pair p (zero from the offset's term count on).  Those
// complex coefficients depend on the call's theta and scale only: one small
// launch writes them, [16 offsets][16 terms][64 pairs] x float2, behind the
// panels in the workspace, and the panel launch reads them from there.
constexpr size_t kOffsetCoefBytes = (size_t)16 * kPanelTerms * 64 * 8;

struct OffsetPanelArgs {
  const void* k;
  int64_t ks[3];
  int B, Hkv, S;
  int nhw;          // half windows per (b, hk): 2 * ceil(S / 16)
  int rows[2];      // panel rows per slab (the slab's first K step's count)
  int nrow[8];      // rows each K step reads (multiples of 16)
  void* out[2];     // slab panels
  float2* cf;       // [16][kPanelTerms][64] complex coefficients
  int km;           // most terms of any offset
  int bwd_order;    // key slots: tcx::bwd_slot_key (else 8 hh + slot_key)
  int signs;        // coefficients times s_m = (+, +, -, -, ...) (the dQ kernel's basis)
  float scale;      // sm_scale * log2(e)
  double th[64];    // theta_p
};

// J_0(x) .. J_{n-1}(x) (n <= 16, 0 <= x <= 8) by Miller's backward recurrence
// J_{k-1} = (2k / x) J_k - J_{k+1} from k = 32, normalised by
// J_0 + 2 (J_2 + J_4 + ...) = 1.
__device__ inline void bessel_j_all(double x, int n, double* out) {
  if (x == 0.0) {
    for (int m = 0; m < n; ++m) out[m] = m == 0 ? 1.0 : 0.0;
    return;
  }
  const double r = 2.0 / x;
  double jp = 0.0, j = 1e-30, norm = 0.0;
  for (int k = 32; k >= 1; --k) {
    const double jm = k * r * j - jp;  // J_{k-1}
    jp = j;
    j = jm;
    if (k - 1 < n) out[k - 1] = j;
    if (((k - 1) & 1) == 0) norm += (k - 1 == 0 ? 1.0 : 2.0) * j;
    if (fabs(j) > 1e200) {  // keep the unnormalised values in range
      j *= 1e-200; jp *= 1e-200; norm *= 1e-200;
      for (int m = k - 1; m < n; ++m) out[m] *= 1e-200;
    }
  }
  const double inv = 1.0 / norm;
  for (int m = 0; m < n; ++m) out[m] *= inv;
}

// The scaled key of one pair: (k_lo + i k_hi) (cr + i ci), rounded once to
// the 16-bit type; the panel kernel and the dQ kernel's builders share it so
// that both give the same bits.
template <typename E>
__device__ __forceinline__ uint32_t cmul_pack(uint32_t kw, float cr, float ci) {
  const float kl = E::lo(kw), kh = E::hi(kw);
  return E::pack(__fmaf_rn(kl, cr, __fmul_rn(-kh, ci)), __fmaf_rn(kl, ci, __fmul_rn(kh, cr)));
}

// One thread per (offset o = blockIdx.x, pair p = threadIdx.x).
static __global__ void __launch_bounds__(64) offset_coef_kernel(const __grid_constant__ OffsetPanelArgs A) {
  const int o = blockIdx.x, p = threadIdx.x;
  const double c = offset_halfwidth(A.km, o);
  const int n = offset_terms(A.km, o);
  double jv[kPanelTerms];
  bessel_j_all(c * A.th[p], n, jv);
  double sn, cs;
  sincos((kC0 - c) * A.th[p], &sn, &cs);
  for (int m = 0; m < kPanelTerms; ++m) {
    const double be = (m < n ? (m == 0 ? 1.0 : 2.0) * jv[m] * A.scale : 0.0) *
                      (A.signs && (m & 3) >= 2 ? -1.0 : 1.0);
    // (-i)^m exp(i phi) = exp(i (phi - m pi / 2))
    double re, im;
    switch (m & 3) {
      case 0: re = cs; im = sn; break;
      case 1: re = sn; im = -cs; break;
      case 2: re = -cs; im = -sn; break;
      default: re = -sn; im = cs; break;
    }
    A.cf[((size_t)o * kPanelTerms + m) * 64 + p] = make_float2((float)(be * re), (float)(be * im));
  }
}

// Row r of K step s (16 elements = two 16-byte chunks) of half window hw
// holds term m = r / 8 of the key in slot r % 8 (window key 8 (hw & 1) +
// slot_key(r % 8), or bwd_slot_key(hw & 1, r % 8) in the backward's order):
// its complex coefficient times the key's pair.  Rows a K step does not read
// (past nrow[s]) and keys past S are zero.
template <typename T, int D>
__global__ void __launch_bounds__(128) offset_panel_kernel(const __grid_constant__ OffsetPanelArgs A) {
  using E = ElemTraits<T>;
  const int hw = blockIdx.x, bh = blockIdx.y;
  const int b = bh / A.Hkv, hk = bh % A.Hkv;
  const T* kb = static_cast<const T*>(A.k) + b * A.ks[0] + hk * A.ks[1];
  const int hh = hw & 1;
#pragma unroll
  for (int s = 0; s < D / 64; ++s) {
    const int rows = A.rows[s];
    uint4* out = static_cast<uint4*>(A.out[s]) + ((int64_t)bh * A.nhw + hw) * rows * 8;
    for (int it = threadIdx.x; it < rows * 8; it += 128) {
      const int r = it >> 3, c = it & 7, m = r >> 3, slot = r & 7;
      const int kk = A.bwd_order ? bwd_slot_key(hh, slot) : 8 * hh + slot_key(slot);  // window offset
      const int key = 16 * (hw >> 1) + kk;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (r < A.nrow[4 * s + (c >> 1)] && key < A.S && m < kPanelTerms) {
        const uint4 kv =
            *reinterpret_cast<const uint4*>(kb + (int64_t)key * A.ks[2] + 64 * s + 8 * c);
        const float4* cp = reinterpret_cast<const float4*>(
            A.cf + ((size_t)kk * kPanelTerms + m) * 64 + 32 * s + 4 * c);
        const float4 c01 = __ldg(cp), c23 = __ldg(cp + 1);
        v = make_uint4(cmul_pack<E>(kv.x, c01.x, c01.y), cmul_pack<E>(kv.y, c01.z, c01.w),
                       cmul_pack<E>(kv.z, c23.x, c23.y), cmul_pack<E>(kv.w, c23.z, c23.w));
      }
      out[it] = v;
    }
  }
}

// Half windows of panels a launch reads: its rows r0 .. r0 + S - 1 see keys
// below r0 + S only (causal), so a query chunk of a longer key sequence needs
// the panels of those keys alone; the panel layout keeps the stride of all Sk.
inline int panel_halfwindows_read(int Sk, int r0, int S) {
  return 2 * ((std::min(Sk, r0 + S) + kW - 1) / kW);
}

// Fill the arguments of the per-offset panels (KM: most terms of any
// offset) and return the workspace bytes they take: both slabs' panels, then
// (own_table) the coefficient table (0 when the head dim has none).
template <int KM>
inline size_t offset_panel_bytes(int B, int Hkv, int S, int D, float theta, float sm_scale,
                                 OffsetPanelArgs* a = nullptr, bool bwd_order = false,
                                 bool own_table = true) {
  OffsetPanelArgs local;
  OffsetPanelArgs& p = a ? *a : local;
  std::memset(&p, 0, sizeof(p));
  fill_offset_rows<KM>(p.nrow, D, theta);
  p.rows[0] = p.nrow[0];
  p.rows[1] = D == 128 ? p.nrow[4] : 0;
  p.B = B; p.Hkv = Hkv; p.S = S;
  p.nhw = 2 * ((S + kW - 1) / kW);
  p.km = KM;
  p.bwd_order = bwd_order ? 1 : 0;
  p.scale = sm_scale * kLog2e;
  for (int q = 0; q < 64; ++q)
    p.th[q] = q < D / 2 ? 1.0 / std::pow((double)theta, (double)(2 * q) / (double)D) : 0.0;
  const size_t panels = (size_t)panel_count(B, Hkv, S) * (p.rows[0] + p.rows[1]) * 128;
  return panels > 0 ? panels + (own_table ? kOffsetCoefBytes : 0) : 0;
}

}  // namespace tcx
}  // namespace corope
