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

template <typename T> struct ElemTraits;
template <> struct ElemTraits<__nv_bfloat16> {
  static constexpr bool kBf16 = true;
  __device__ static float lo(uint32_t x) { return __uint_as_float(x << 16); }
  __device__ static float hi(uint32_t x) { return __uint_as_float(x & 0xffff0000u); }
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
  __device__ static uint32_t pack(float a, float b) { return sm100::pack_f16(a, b); }
};

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
inline double bessel_j(int m, double x) {
  double term = 1.0;
  for (int i = 1; i <= m; ++i) term *= (x / 2.0) / i;
  double sum = term;
  const double q = -(x * x) / 4.0;
  for (int k = 1; k < 80; ++k) {
    term *= q / (k * (double)(k + m));
    sum += term;
    if (std::fabs(term) < 1e-18 * std::fabs(sum) + 1e-300) break;
  }
  return sum;
}

// Chebyshev coefficients eps_m J_m(c0 theta_p) * sm_scale * log2(e) of the
// first KM terms and the pruned K extent of each term: nrow[s] = rows of the K^(m) operand that
// K-step s (16 head dims) reads (8 keys per term, rounded to 16 rows).
template <int KM = kM>
inline void fill_coefficients(float (*coef)[64], int* nrow, int D, float theta, float sm_scale) {
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

}  // namespace tcx
}  // namespace corope
