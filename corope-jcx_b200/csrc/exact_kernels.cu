// Exact-math CoRoPE kernels on CUDA cores (sm_100a).
//
// Every (query t, key j, pair p) angle a_tj * theta_p gets its own sine and
// cosine, as in the reference definition (check.py:65-95).  These kernels are
// the precision anchor of the library (COROPE_ALGO_EXACT) and cover every
// shape; the tensor-core kernels in tc_fwd.cu are the fast path.
//
// Work split: one CTA owns BM = 64 query rows of one (b, h); each row is
// owned by TPR consecutive threads, each holding an interleaved subset of the
// D/2 rotation pairs (pair p belongs to thread p % TPR, which keeps the
// shared-memory reads of a key row bank-conflict free).  Keys are staged in
// shared memory as fp32 tiles of BN = 32.
#include "common.cuh"

namespace corope {

constexpr int kBM = 64;
constexpr int kBN = 32;

template <typename T>
__device__ __forceinline__ float2 load_pair(const T* base, int64_t off) {
  return make_float2(to_f32<T>(base[off]), to_f32<T>(base[off + 1]));
}

// Load keys [j0, j0 + kBN) of one head into shared memory as fp32 pairs
// (rows past the sequence end are zero).
template <typename T, int D>
__device__ __forceinline__ void stage_rows(float2* dst, const T* src, int64_t seq_stride,
                                           int j0, int S, int nthreads) {
  constexpr int P = D / 2;
  for (int idx = threadIdx.x; idx < kBN * P; idx += nthreads) {
    int r = idx / P, p = idx % P;
    int j = j0 + r;
    dst[idx] = (j < S) ? load_pair<T>(src, (int64_t)j * seq_stride + 2 * p) : make_float2(0.f, 0.f);
  }
}

template <int TPR>
__device__ __forceinline__ float group_sum(float x) {
#pragma unroll
  for (int off = 1; off < TPR; off <<= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

// ---------------------------------------------------------------------------
// Forward.  Keys are walked from the diagonal down to 0 (as the reference
// kernel does, CoROPE/forward.py:57-78) so the contextual position
// a_tj = sum_{i=j+1..t} z_ti is a running suffix sum per row.
// ---------------------------------------------------------------------------
template <typename T, int D, int TPR, bool HAS_BIAS>
__global__ void __launch_bounds__(kBM * TPR)
exact_fwd_kernel(FwdArgs args) {
  constexpr int P = D / 2;
  constexpr int NP = P / TPR;       // pairs per thread
  constexpr int NT = kBM * TPR;
  constexpr int CH = 8;             // keys per online-softmax update
  __shared__ float2 Ks[kBN * P];
  __shared__ float2 Vs[kBN * P];
  __shared__ float th_s[P];

  const int qtile = gridDim.x - 1 - blockIdx.x;   // longest rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (args.H / args.Hkv);
  const int rl = threadIdx.x / TPR, sub = threadIdx.x % TPR;
  const int tl = qtile * kBM + rl;  // row of q / o
  const int t = args.r0 + tl;       // its sequence position
  const int S = args.S;

  const T* qb = (const T*)args.q + b * args.qs[0] + h * args.qs[1];
  const T* kb = (const T*)args.k + b * args.ks[0] + hk * args.ks[1];
  const T* vb = (const T*)args.v + b * args.vs[0] + hk * args.vs[1];

  for (int p = threadIdx.x; p < P; p += NT) th_s[p] = theta_at(args.thetas, args.theta, p, D);

  float2 qp[NP], op[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    int p = i * TPR + sub;
    qp[i] = (tl < S) ? load_pair<T>(qb, (int64_t)tl * args.qs[2] + 2 * p) : make_float2(0.f, 0.f);
    op[i] = make_float2(0.f, 0.f);
  }
  float m_run = -1e30f, l_run = 0.f;
  // suffix gate sum, compensated (Kahan; a_run - a_cmp is the sum to ~1 ulp):
  // a plain fp32 running sum over tens of thousands of keys drifts by ~1e-2
  float a_run = 0.f, a_cmp = 0.f;
  float lg[CH];
  const float sm = args.sm_scale;

  const int last_row = args.r0 + min(S - 1, qtile * kBM + kBM - 1);  // sequence position
  for (int j0 = (last_row / kBN) * kBN; j0 >= 0; j0 -= kBN) {
    __syncthreads();
    stage_rows<T, D>(Ks, kb, args.ks[2], j0, args.Sk, NT);
    stage_rows<T, D>(Vs, vb, args.vs[2], j0, args.Sk, NT);
    __syncthreads();
#pragma unroll 1
    for (int c0 = kBN - CH; c0 >= 0; c0 -= CH) {
#pragma unroll
      for (int u = CH - 1; u >= 0; --u) {
        const int jj = c0 + u;
        const int j = j0 + jj;
        const bool valid = (j <= t) && (tl < S);
        const float2* kr = Ks + jj * P;
        float g = 0.f;
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          float2 kk = kr[i * TPR + sub];
          g = fmaf(qp[i].x, kk.x, fmaf(qp[i].y, kk.y, g));
        }
        g = group_sum<TPR>(g);
        const float z = valid ? sigmoidf_fast(g) : 0.f;
        const float a_tj = a_run - a_cmp;
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          float2 kk = kr[i * TPR + sub];
          float s, c;
          sincos_reduced(a_tj * th_s[i * TPR + sub], &s, &c);
          float Cp = fmaf(qp[i].x, kk.x, qp[i].y * kk.y);
          float Sp = fmaf(qp[i].x, kk.y, -qp[i].y * kk.x);
          acc = fmaf(c, Cp, fmaf(s, Sp, acc));
        }
        acc = group_sum<TPR>(acc);
        float logit = acc * sm;
        if (HAS_BIAS && valid) logit += args.bias[(int64_t)t * args.bias_rs + j];
        lg[u] = valid ? logit : -INFINITY;
        {
          const float y = z - a_cmp;
          const float s2 = a_run + y;
          a_cmp = (s2 - a_run) - y;
          a_run = s2;
        }
      }
      // online softmax over the CH keys just scored
      float mx = m_run;
#pragma unroll
      for (int u = 0; u < CH; ++u) mx = fmaxf(mx, lg[u]);
      const float alpha = __expf(m_run - mx);
      l_run *= alpha;
#pragma unroll
      for (int i = 0; i < NP; ++i) { op[i].x *= alpha; op[i].y *= alpha; }
#pragma unroll
      for (int u = 0; u < CH; ++u) {
        const float pr = __expf(lg[u] - mx);
        l_run += pr;
        const float2* vr = Vs + (c0 + u) * P;
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          float2 vv = vr[i * TPR + sub];
          op[i].x = fmaf(pr, vv.x, op[i].x);
          op[i].y = fmaf(pr, vv.y, op[i].y);
        }
      }
      m_run = mx;
    }
  }

  if (tl < S) {
    T* ob = (T*)args.o + b * args.os[0] + h * args.os[1] + (int64_t)tl * args.os[2];
    const float inv = 1.0f / l_run;
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      int p = i * TPR + sub;
      ob[2 * p] = from_f32<T>(op[i].x * inv);
      ob[2 * p + 1] = from_f32<T>(op[i].y * inv);
    }
    if (sub == 0) {
      const int64_t r = ((int64_t)b * args.H + h) * S + tl;
      if (args.m) args.m[r] = m_run;
      if (args.l) args.l[r] = l_run;
      if (args.a) args.a[r] = a_run - a_cmp;
      if (args.lse) args.lse[r] = m_run + logf(l_run);
    }
  }
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------
// delta_t = sum_d dO_td * O_td and lse_t = m_t + log(l_t); one warp per row.
// VEC: 16-bit rows with 8-byte aligned starts and D a multiple of 4 -- each
// lane reads 4 consecutive elements of o and dO per 8-byte load.
template <typename T, bool VEC>
__global__ void exact_bwd_pre_kernel(BwdArgs args) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)args.B * args.H * args.S;
  if (warp >= rows) return;
  const int t = warp % args.S;
  const int bh = warp / args.S;
  const int h = bh % args.H, b = bh / args.H;
  const T* ob = (const T*)args.o + b * args.os[0] + h * args.os[1] + (int64_t)t * args.os[2];
  const T* db = (const T*)args.dout + b * args.dos[0] + h * args.dos[1] + (int64_t)t * args.dos[2];
  float s = 0.f;
  if constexpr (VEC) {
    for (int d = 4 * lane; d < args.D; d += 128) {
      const uint2 ov = *reinterpret_cast<const uint2*>(ob + d);
      const uint2 dv = *reinterpret_cast<const uint2*>(db + d);
      const T* o4 = reinterpret_cast<const T*>(&ov);
      const T* d4 = reinterpret_cast<const T*>(&dv);
#pragma unroll
      for (int e = 0; e < 4; ++e) s = fmaf(to_f32<T>(o4[e]), to_f32<T>(d4[e]), s);
    }
  } else {
    for (int d = lane; d < args.D; d += 32) s = fmaf(to_f32<T>(ob[d]), to_f32<T>(db[d]), s);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) {
    args.delta[warp] = s;
    args.lse[warp] = args.m[warp] + logf(args.l[warp]);
  }
}

// Query-stationary backward.  For each key tile (ascending) the row owners
// recompute gates, positions a_tj = A_t - sum_{i<=j} z_ti, logits, P, dP and
// the position/gate chain (exclusive prefix sum of da along keys), update dq,
// and leave the per-pair scalars (P, dlogit*sm, dgate, a) in shared memory;
// then the same threads re-partition by key and reduce dk, dv over the
// tile's 64 rows, adding the partial sums to fp32 accumulators in global
// memory.
template <typename T, int D, int TPR, bool HAS_BIAS>
__global__ void __launch_bounds__(kBM * TPR)
exact_bwd_kernel(BwdArgs args) {
  constexpr int P = D / 2;
  constexpr int NP = P / TPR;
  constexpr int NT = kBM * TPR;
  constexpr int TPK = NT / kBN;                    // threads per key in phase 2
  constexpr int NP2 = (P + TPK - 1) / TPK;
  constexpr int PB = kBN + 1;                      // padded pair-buffer row
  extern __shared__ float4 smem_f4[];
  float2* Ks = reinterpret_cast<float2*>(smem_f4);
  float2* Vs = Ks + kBN * P;
  float2* Qs = Vs + kBN * P;
  float2* Ds = Qs + kBM * P;
  float* bufP = reinterpret_cast<float*>(Ds + kBM * P);
  float* bufW = bufP + kBM * PB;
  float* bufG = bufW + kBM * PB;
  float* bufA = bufG + kBM * PB;
  float* th_s = bufA + kBM * PB;

  const int qtile = gridDim.x - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (args.H / args.Hkv);
  const int rl = threadIdx.x / TPR, sub = threadIdx.x % TPR;
  const int q0 = qtile * kBM;        // first row of the tile in q / dO / dq
  const int tl = q0 + rl;
  const int t = args.r0 + tl;        // sequence position of row tl
  const int S = args.S;
  const float sm = args.sm_scale;

  const T* qb = (const T*)args.q + b * args.qs[0] + h * args.qs[1];
  const T* kb = (const T*)args.k + b * args.ks[0] + hk * args.ks[1];
  const T* vb = (const T*)args.v + b * args.vs[0] + hk * args.vs[1];
  const T* db = (const T*)args.dout + b * args.dos[0] + h * args.dos[1];

  for (int p = threadIdx.x; p < P; p += NT) th_s[p] = theta_at(args.thetas, args.theta, p, D);
  for (int idx = threadIdx.x; idx < kBM * P; idx += NT) {
    int r = idx / P, p = idx % P;
    int tt = q0 + r;
    Qs[idx] = (tt < S) ? load_pair<T>(qb, (int64_t)tt * args.qs[2] + 2 * p) : make_float2(0.f, 0.f);
    Ds[idx] = (tt < S) ? load_pair<T>(db, (int64_t)tt * args.dos[2] + 2 * p) : make_float2(0.f, 0.f);
  }
  __syncthreads();

  float2 qp[NP], dop[NP], dqp[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    qp[i] = Qs[rl * P + i * TPR + sub];
    dop[i] = Ds[rl * P + i * TPR + sub];
    dqp[i] = make_float2(0.f, 0.f);
  }
  const int64_t rix = ((int64_t)b * args.H + h) * S + tl;
  const float A_t = (tl < S) ? args.a[rix] : 0.f;
  const float lse_t = (tl < S) ? args.lse[rix] : 0.f;
  const float dlt_t = (tl < S) ? args.delta[rix] : 0.f;
  // gate prefix, compensated (Kahan; c_run - c_cmp is the prefix to ~1 ulp)
  float c_run = 0.f, c_cmp = 0.f, da_run = 0.f;

  // phase-2 mapping
  const int kj = threadIdx.x / TPK, sub2 = threadIdx.x % TPK;
  const int bhk = b * args.Hkv + hk;
  const int BHkv = args.B * args.Hkv;

  const int last_row = args.r0 + min(S - 1, q0 + kBM - 1);  // sequence position
  for (int j0 = 0; j0 <= last_row; j0 += kBN) {
    __syncthreads();
    stage_rows<T, D>(Ks, kb, args.ks[2], j0, args.Sk, NT);
    stage_rows<T, D>(Vs, vb, args.vs[2], j0, args.Sk, NT);
    __syncthreads();
    // ---- phase 1: row owners --------------------------------------------
#pragma unroll 1
    for (int jj = 0; jj < kBN; ++jj) {
      const int j = j0 + jj;
      const bool valid = (j <= t) && (tl < S);
      const float2* kr = Ks + jj * P;
      const float2* vr = Vs + jj * P;
      float g = 0.f;
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        float2 kk = kr[i * TPR + sub];
        g = fmaf(qp[i].x, kk.x, fmaf(qp[i].y, kk.y, g));
      }
      g = group_sum<TPR>(g);
      const float z = valid ? sigmoidf_fast(g) : 0.f;
      {
        const float y = z - c_cmp;
        const float s2 = c_run + y;
        c_cmp = (s2 - c_run) - y;
        c_run = s2;
      }
      const float a = valid ? ((A_t - c_run) + c_cmp) : 0.f;
      float cs[NP], sn[NP];
      float acc = 0.f, dacc = 0.f, dpp = 0.f;
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        const int p = i * TPR + sub;
        float2 kk = kr[p];
        float2 vv = vr[p];
        sincos_reduced(a * th_s[p], &sn[i], &cs[i]);
        float Cp = fmaf(qp[i].x, kk.x, qp[i].y * kk.y);
        float Sp = fmaf(qp[i].x, kk.y, -qp[i].y * kk.x);
        acc = fmaf(cs[i], Cp, fmaf(sn[i], Sp, acc));
        dacc = fmaf(th_s[p], fmaf(cs[i], Sp, -sn[i] * Cp), dacc);
        dpp = fmaf(dop[i].x, vv.x, fmaf(dop[i].y, vv.y, dpp));
      }
      acc = group_sum<TPR>(acc);
      dacc = group_sum<TPR>(dacc);
      dpp = group_sum<TPR>(dpp);
      float logit = acc * sm;
      if (HAS_BIAS && valid) logit += args.bias[(int64_t)t * args.bias_rs + j];
      const float pr = valid ? __expf(logit - lse_t) : 0.f;
      const float w = pr * (dpp - dlt_t) * sm;      // d logit * sm_scale
      const float da = w * dacc;
      const float ds = valid ? da_run * z * (1.f - z) : 0.f;   // exclusive prefix
      da_run += valid ? da : 0.f;
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        float2 kk = kr[i * TPR + sub];
        // w * R(-phi) k + ds * k
        dqp[i].x += w * fmaf(kk.x, cs[i], kk.y * sn[i]) + ds * kk.x;
        dqp[i].y += w * fmaf(kk.y, cs[i], -kk.x * sn[i]) + ds * kk.y;
      }
      if (sub == 0) {
        bufP[rl * PB + jj] = pr;
        bufW[rl * PB + jj] = valid ? w : 0.f;
        bufG[rl * PB + jj] = ds;
        bufA[rl * PB + jj] = a;
      }
    }
    __syncthreads();
    // ---- phase 2: key owners --------------------------------------------
    {
      const int j = j0 + kj;
      float2 dkp[NP2], dvp[NP2];
#pragma unroll
      for (int i = 0; i < NP2; ++i) { dkp[i] = make_float2(0.f, 0.f); dvp[i] = dkp[i]; }
#pragma unroll 1
      for (int r = 0; r < kBM; ++r) {
        const float pr = bufP[r * PB + kj];
        const float w = bufW[r * PB + kj];
        const float ds = bufG[r * PB + kj];
        const float a = bufA[r * PB + kj];
#pragma unroll
        for (int i = 0; i < NP2; ++i) {
          const int p = i * TPK + sub2;
          if (p < P) {
            float s, c;
            sincos_reduced(a * th_s[p], &s, &c);
            float2 qq = Qs[r * P + p];
            float2 dd = Ds[r * P + p];
            // w * R(phi) q + ds * q
            dkp[i].x += w * fmaf(qq.x, c, -qq.y * s) + ds * qq.x;
            dkp[i].y += w * fmaf(qq.x, s, qq.y * c) + ds * qq.y;
            dvp[i].x = fmaf(pr, dd.x, dvp[i].x);
            dvp[i].y = fmaf(pr, dd.y, dvp[i].y);
          }
        }
      }
      if (j < args.Sk) {
        const int64_t row = accum_row(j, bhk, BHkv, args.Sk, args.acc_chunk) * D;
#pragma unroll
        for (int i = 0; i < NP2; ++i) {
          const int p = i * TPK + sub2;
          if (p < P) {
            const bool fixed = args.fixed != 0;
            acc_add(args.dk32, row + 2 * p, dkp[i].x, fixed);
            acc_add(args.dk32, row + 2 * p + 1, dkp[i].y, fixed);
            acc_add(args.dv32, row + 2 * p, dvp[i].x, fixed);
            acc_add(args.dv32, row + 2 * p + 1, dvp[i].y, fixed);
          }
        }
      }
    }
  }

  if (tl < S) {
    T* dqb = (T*)args.dq + b * args.dqs[0] + h * args.dqs[1] + (int64_t)tl * args.dqs[2];
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      int p = i * TPR + sub;
      dqb[2 * p] = from_f32<T>(dqp[i].x);
      dqb[2 * p + 1] = from_f32<T>(dqp[i].y);
    }
  }
}

// two floats -> one word of 16-bit values, rounded to nearest (as from_f32)
template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Four consecutive fixed-point accumulator elements (acc_add) from i, a
// multiple of 4: two 16-byte loads.
__device__ __forceinline__ float4 fix4(const float* base, int64_t i) {
  const longlong2* p = reinterpret_cast<const longlong2*>(base) + i / 2;
  const longlong2 a = p[0], b = p[1];
  return make_float4(__ll2float_rn(a.x) * kFixUnit, __ll2float_rn(a.y) * kFixUnit,
                     __ll2float_rn(b.x) * kFixUnit, __ll2float_rn(b.y) * kFixUnit);
}

// fp32 (or fixed-point) dk/dv accumulators -> output dtype and strides.  VEC: 16-bit outputs
// with 16-byte aligned rows and D a multiple of 8 -- each thread converts 8
// consecutive elements (two 16-byte loads per accumulator, one 16-byte store
// per output) and derives the row once for them.
template <typename T, bool VEC>
__global__ void exact_bwd_post_kernel(BwdArgs args) {
  if constexpr (VEC) {
    const int d8 = args.D / 8;
    const int64_t n8 = (int64_t)args.B * args.Hkv * args.Sk * d8;
    for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < n8;
         g += (int64_t)gridDim.x * blockDim.x) {
      const int64_t r = g / d8;
      const int d0 = (int)(g - r * d8) * 8;
      const int j = (int)(r % args.Sk);
      const int64_t bh = r / args.Sk;
      const int hk = (int)(bh % args.Hkv), b = (int)(bh / args.Hkv);
      float4 ka, kb, va, vb;
      if (args.fixed) {
        ka = fix4(args.dk32, g * 8); kb = fix4(args.dk32, g * 8 + 4);
        va = fix4(args.dv32, g * 8); vb = fix4(args.dv32, g * 8 + 4);
      } else {
        const float4* k4 = reinterpret_cast<const float4*>(args.dk32 + g * 8);
        const float4* v4 = reinterpret_cast<const float4*>(args.dv32 + g * 8);
        ka = k4[0]; kb = k4[1]; va = v4[0]; vb = v4[1];
      }
      uint4 ko, vo;
      ko.x = pack2<T>(ka.x, ka.y); ko.y = pack2<T>(ka.z, ka.w);
      ko.z = pack2<T>(kb.x, kb.y); ko.w = pack2<T>(kb.z, kb.w);
      vo.x = pack2<T>(va.x, va.y); vo.y = pack2<T>(va.z, va.w);
      vo.z = pack2<T>(vb.x, vb.y); vo.w = pack2<T>(vb.z, vb.w);
      *reinterpret_cast<uint4*>((T*)args.dk + b * args.dks[0] + hk * args.dks[1] +
                                (int64_t)j * args.dks[2] + d0) = ko;
      *reinterpret_cast<uint4*>((T*)args.dv + b * args.dvs[0] + hk * args.dvs[1] +
                                (int64_t)j * args.dvs[2] + d0) = vo;
    }
    return;
  }
  const int64_t n = (int64_t)args.B * args.Hkv * args.Sk * args.D;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int d = i % args.D;
    int64_t r = i / args.D;
    const int j = r % args.Sk;
    r /= args.Sk;
    const int hk = r % args.Hkv;
    const int b = r / args.Hkv;
    const bool fixed = args.fixed != 0;
    ((T*)args.dk)[b * args.dks[0] + hk * args.dks[1] + (int64_t)j * args.dks[2] + d] =
        from_f32<T>(acc_get(args.dk32, i, fixed));
    ((T*)args.dv)[b * args.dvs[0] + hk * args.dvs[1] + (int64_t)j * args.dvs[2] + d] =
        from_f32<T>(acc_get(args.dv32, i, fixed));
  }
}

// The vectorised conversion applies to 16-bit outputs whose rows start on
// 16-byte boundaries, with D a multiple of 8.
template <typename T>
static bool post_vec_ok(const BwdArgs& a) {
  if (sizeof(T) != 2 || a.D % 8 != 0) return false;
  const int64_t* st[2] = {a.dks, a.dvs};
  const void* p[2] = {a.dk, a.dv};
  for (int i = 0; i < 2; ++i) {
    if (reinterpret_cast<uintptr_t>(p[i]) % 16 != 0) return false;
    for (int k = 0; k < 3; ++k)
      if ((st[i][k] * 2) % 16 != 0) return false;
  }
  return true;
}
template <typename T>
static cudaError_t launch_post(const BwdArgs& a, cudaStream_t st) {
  if constexpr (sizeof(T) == 2) {
    if (post_vec_ok<T>(a)) {
      exact_bwd_post_kernel<T, true><<<148 * 8, 256, 0, st>>>(a);
      return cudaGetLastError();
    }
  }
  exact_bwd_post_kernel<T, false><<<148 * 8, 256, 0, st>>>(a);
  return cudaGetLastError();
}
// The vectorised delta reads apply to 16-bit rows starting on 8-byte
// boundaries, with D a multiple of 4.
template <typename T>
static void launch_pre(const BwdArgs& a, cudaStream_t st) {
  const int64_t rows = (int64_t)a.B * a.H * a.S;
  const unsigned grid = (unsigned)((rows * 32 + 255) / 256);
  if constexpr (sizeof(T) == 2) {
    bool vec = a.D % 4 == 0 && reinterpret_cast<uintptr_t>(a.o) % 8 == 0 &&
               reinterpret_cast<uintptr_t>(a.dout) % 8 == 0;
    for (int k = 0; k < 3; ++k) vec = vec && (a.os[k] * 2) % 8 == 0 && (a.dos[k] * 2) % 8 == 0;
    if (vec) {
      exact_bwd_pre_kernel<T, true><<<grid, 256, 0, st>>>(a);
      return;
    }
  }
  exact_bwd_pre_kernel<T, false><<<grid, 256, 0, st>>>(a);
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
template <int D> constexpr int tpr_for() { return D >= 8 ? 4 : 2; }

template <typename T, int D>
static cudaError_t launch_fwd_d(const FwdArgs& a, cudaStream_t st) {
  constexpr int TPR = tpr_for<D>();
  dim3 grid((a.S + kBM - 1) / kBM, a.H, a.B);
  if (a.bias)
    exact_fwd_kernel<T, D, TPR, true><<<grid, kBM * TPR, 0, st>>>(a);
  else
    exact_fwd_kernel<T, D, TPR, false><<<grid, kBM * TPR, 0, st>>>(a);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_fwd_t(const FwdArgs& a, cudaStream_t st) {
  switch (a.D) {
    case 4: return launch_fwd_d<T, 4>(a, st);
    case 8: return launch_fwd_d<T, 8>(a, st);
    case 16: return launch_fwd_d<T, 16>(a, st);
    case 32: return launch_fwd_d<T, 32>(a, st);
    case 64: return launch_fwd_d<T, 64>(a, st);
    case 128: return launch_fwd_d<T, 128>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t exact_fwd_launch(const FwdArgs& a, int dtype, cudaStream_t st) {
  switch (dtype) {
    case COROPE_DTYPE_F32: return launch_fwd_t<float>(a, st);
    case COROPE_DTYPE_F16: return launch_fwd_t<__half>(a, st);
    case COROPE_DTYPE_BF16: return launch_fwd_t<__nv_bfloat16>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

template <int D>
static size_t bwd_smem_bytes() {
  constexpr int P = D / 2;
  return sizeof(float2) * (2 * kBN * P + 2 * kBM * P) + sizeof(float) * (4 * kBM * (kBN + 1) + P);
}

template <typename T, int D>
static cudaError_t launch_bwd_d(const BwdArgs& a, cudaStream_t st) {
  constexpr int TPR = tpr_for<D>();
  const size_t smem = bwd_smem_bytes<D>();
  dim3 grid((a.S + kBM - 1) / kBM, a.H, a.B);
  cudaError_t e;
  if (a.bias) {
    auto kern = exact_bwd_kernel<T, D, TPR, true>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    kern<<<grid, kBM * TPR, smem, st>>>(a);
  } else {
    auto kern = exact_bwd_kernel<T, D, TPR, false>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    kern<<<grid, kBM * TPR, smem, st>>>(a);
  }
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_bwd_t(const BwdArgs& a, cudaStream_t st) {
  launch_pre<T>(a, st);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  switch (a.D) {
    case 4: e = launch_bwd_d<T, 4>(a, st); break;
    case 8: e = launch_bwd_d<T, 8>(a, st); break;
    case 16: e = launch_bwd_d<T, 16>(a, st); break;
    case 32: e = launch_bwd_d<T, 32>(a, st); break;
    case 64: e = launch_bwd_d<T, 64>(a, st); break;
    case 128: e = launch_bwd_d<T, 128>(a, st); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) return e;
  if (!a.dk || !a.dv) return cudaSuccess;  // query chunk: the caller keeps the fp32 sums
  return launch_post<T>(a, st);
}

template <typename T>
static cudaError_t pre_t(const BwdArgs& a, cudaStream_t st) {
  launch_pre<T>(a, st);
  return cudaGetLastError();
}
template <typename T>
static cudaError_t post_t(const BwdArgs& a, cudaStream_t st) {
  return launch_post<T>(a, st);
}

// delta = rowsum(dO * O) and lse = m + log(l) into the workspace
cudaError_t bwd_pre_launch(const BwdArgs& a, int dtype, cudaStream_t st) {
  switch (dtype) {
    case COROPE_DTYPE_F32: return pre_t<float>(a, st);
    case COROPE_DTYPE_F16: return pre_t<__half>(a, st);
    case COROPE_DTYPE_BF16: return pre_t<__nv_bfloat16>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

// fp32 dk/dv accumulators -> output dtype
cudaError_t bwd_post_launch(const BwdArgs& a, int dtype, cudaStream_t st) {
  switch (dtype) {
    case COROPE_DTYPE_F32: return post_t<float>(a, st);
    case COROPE_DTYPE_F16: return post_t<__half>(a, st);
    case COROPE_DTYPE_BF16: return post_t<__nv_bfloat16>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t exact_bwd_launch(const BwdArgs& a, int dtype, cudaStream_t st) {
  switch (dtype) {
    case COROPE_DTYPE_F32: return launch_bwd_t<float>(a, st);
    case COROPE_DTYPE_F16: return launch_bwd_t<__half>(a, st);
    case COROPE_DTYPE_BF16: return launch_bwd_t<__nv_bfloat16>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

bool exact_supports_head_dim(int D) {
  return D == 4 || D == 8 || D == 16 || D == 32 || D == 64 || D == 128;
}

}  // namespace corope
