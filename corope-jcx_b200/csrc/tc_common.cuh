// Pieces shared by the tensor-core CoRoPE kernels (forward and backward):
// the windowed Chebyshev expansion constants, 16-bit element helpers, and the
// host-side tensor-map encoding and expansion coefficients.
#pragma once

#include <algorithm>
#include <cmath>
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

}  // namespace tcx
}  // namespace corope
