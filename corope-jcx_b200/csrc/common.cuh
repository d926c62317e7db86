// Shared device helpers for the CoRoPE kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/corope.h"

namespace corope {

// ---- element conversion -------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// ---- angles ---------------------------------------------------------------
// sin/cos of x = a * theta (radians, |x| up to ~1e5).  The product is
// rounded once to fp32, as the reference's `freq = a * thetas` is
// (check.py:68-72), then reduced to [-pi, pi] with a two-constant
// Cody-Waite split of 2*pi (the hi part has 8 significant bits, so k*hi is
// exact in fp32 for |k| < 2^16, i.e. |x| < 4e5; lo carries the rest), and
// evaluated with the hardware approximation, which is accurate on [-pi, pi].
__device__ __forceinline__ void sincos_reduced(float x, float* s, float* c) {
  const float kInv2Pi = 0.15915494309189535f;
  const float k2PiHi = 6.28125f;                 // 2*pi rounded to 8 bits
  const float k2PiLo = 1.9353071795864769e-3f;   // 2*pi - k2PiHi
  float k = rintf(x * kInv2Pi);
  float r = fmaf(-k, k2PiHi, x);
  r = fmaf(-k, k2PiLo, r);
  __sincosf(r, s, c);
}

// Below this many radians MUFU's own range reduction keeps sin/cos within
// 5.5e-4 of the fp32 angle's (measured maximum up to 4096 rad), under half a
// bf16 ulp of a unit-scale rotated value: the tensor-core kernels, whose
// rotated operands are rounded to 16-bit floats, skip the explicit reduction
// when a whole warp's angles are below it.
constexpr float kMufuReduceMax = 4096.f;

// Largest |theta_p| of a frequency table of n entries in shared memory.
__device__ __forceinline__ float theta_max(const float* th, int n) {
  float m = 0.f;
  for (int p = 0; p < n; ++p) m = fmaxf(m, fabsf(th[p]));
  return m;
}

// Reduce x (radians) to r in [-pi, pi]: k = nearest integer to x / 2pi by
// the round-to-nearest of adding 1.5 * 2^23 (|x| / 2pi < 2^22), then the same
// two-constant Cody-Waite subtraction as sincos_reduced.  FMA pipe only.
__device__ __forceinline__ float reduce_2pi(float x) {
  const float kInv2Pi = 0.15915494309189535f;
  const float kMagic = 12582912.0f;
  const float k = fmaf(x, kInv2Pi, kMagic) - kMagic;
  float r = fmaf(-k, 6.28125f, x);
  return fmaf(-k, 1.9353071795864769e-3f, r);
}

__device__ __forceinline__ float sigmoidf_fast(float x) {
  return 1.0f / (1.0f + __expf(-x));
}

// theta_p = 1 / theta^(2p/D) in fp32, the reference's table
// (CoROPE/forward.py:130-133, without the repeat_interleave), or the
// caller's table when one is given.
__device__ __forceinline__ float theta_at(const float* table, float theta, int p, int D) {
  return table ? table[p] : 1.0f / powf(theta, (float)(2 * p) / (float)D);
}

// Arguments shared by the forward kernels (element strides; D stride 1).
struct FwdArgs {
  const void *q, *k, *v;
  void* o;
  float *m, *l, *a, *lse;
  const float* thetas;  // [D/2] or NULL: theta^(-2p/D) from `theta`
  const float* bias;
  int64_t bias_rs;
  int64_t qs[3], ks[3], vs[3], os[3];
  int B, H, Hkv, S, D;
  float sm_scale, theta;
  // query chunk: q, o, m, l, a, lse hold the S rows at sequence positions
  // r0 .. r0 + S - 1 (r0 a multiple of 128); k, v hold Sk >= r0 + S rows
  // from position 0.  A whole sequence is r0 = 0, Sk = S.
  int r0, Sk;
};

struct BwdArgs {
  const void *q, *k, *v, *o, *dout;
  const float *m, *l, *a;
  const float* thetas;
  const float* bias;
  int64_t bias_rs;
  void *dq, *dk, *dv;
  int64_t qs[3], ks[3], vs[3], os[3], dos[3], dqs[3], dks[3], dvs[3];
  int B, H, Hkv, S, D;
  float sm_scale, theta;
  // query chunk, as in FwdArgs: q, o, dO, dq, m, l, a, delta, lse hold rows
  // r0 .. r0 + S - 1; k, v, dk32, dv32 (and dk, dv) hold Sk rows
  int r0, Sk;
  // workspace views
  float* delta;  // [B,H,S]  rowsum(dO * O)
  float* lse;    // [B,H,S]  m + log(l)
  float* dk32;   // [B,Hkv,Sk,D] fp32 accumulators (or the owner-major chunk
  float* dv32;   // layout, acc_chunk > 0: see accum_row)
  int acc_chunk; // 0, or the chunk rows C of the owner-major layout
  float2* coef;  // tensor-core path: the dQ kernel's per-offset expansion
                 // coefficients [16][16][64] (complex), written per call
  int fixed;     // 1: dk32 / dv32 hold 64-bit fixed-point sums (acc_add)
};

// Deterministic accumulation: each contribution is rounded to a multiple of
// 2^-36 and added as a 64-bit integer.  Integer addition is associative, so
// the sums do not depend on the order in which the query tiles' atomics land
// (fp32 atomics do); sums must stay below 2^27 in magnitude.
constexpr float kFixScale = 68719476736.f;       // 2^36
constexpr float kFixUnit = 1.4551915228366852e-11f;  // 2^-36

// Adds v to element i of an accumulator: fp32 atomics, or with `fixed` the
// fixed-point sum of the same element count viewed as 64-bit words.
__device__ __forceinline__ void acc_add(float* base, int64_t i, float v, bool fixed) {
  if (fixed)
    atomicAdd(reinterpret_cast<unsigned long long*>(base) + i,
              static_cast<unsigned long long>(__float2ll_rn(v * kFixScale)));
  else
    atomicAdd(base + i, v);
}

// Element i of an accumulator as fp32 (acc_add's two layouts).
__device__ __forceinline__ float acc_get(const float* base, int64_t i, bool fixed) {
  if (fixed) return __ll2float_rn(reinterpret_cast<const long long*>(base)[i]) * kFixUnit;
  return base[i];
}

// Row (in units of D elements) of key `key` of (b, kv head) `bhk` in the fp32
// dk / dv accumulators: [B*Hkv][Sk] rows, or, with C = acc_chunk > 0, the
// zig-zag owner-major layout [2][N][B*Hkv][C] of a sequence of 2N chunks of C
// rows (Sk = 2 N C): chunk c < N at [0][c], chunk c >= N at [1][2N-1-c].
__device__ __forceinline__ int64_t accum_row(int key, int bhk, int BHkv, int Sk, int C) {
  if (C == 0) return (int64_t)bhk * Sk + key;
  const int n = Sk / (2 * C);  // ranks
  const int c = key / C;
  const int pos = c < n ? c : 3 * n - 1 - c;
  return ((int64_t)pos * BHkv + bhk) * C + (key - c * C);
}

}  // namespace corope
