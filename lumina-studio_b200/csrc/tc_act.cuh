// Activation rows -> tensor-pipe B fragments: the prologue of the int4
// decode GEMV (gemv_tc.cu).
//
// NB rows of K columns; item i (eight columns) is row b = i / 8P, pair
// p = (i / 8) mod P, columns 64p + 8(i mod 8) .. +7, so eight consecutive
// threads hold one pair's 64-column block and share its scale. Per block:
// q = rint(v * fp32(QMAX / amax)) clipped to +-QMAX, split q = 256 qh + ql
// into two signed bytes (high bytes are B column 2b, low bytes 2b + 1), and
// fq[p][b] = (amax / QMAX, -15 * sum q). With RMSNorm the row is first
// scaled v = (x * rinv) * w, rinv = 1 / sqrt(mean(x^2) + eps) (chat.py:63-66).
//
// A thread holds TQ_CH items in registers per pass, so the loads of a pass
// are all in flight at once; with one pass (K <= TQ_CH * 8 * threads / NB)
// the row's sum of squares comes from the same registers and costs one CTA
// barrier. The norm weights of the first pass are loaded by tq_preload
// before the kernel waits for its input.
#pragma once
#include <cstdint>

#include "common.cuh"

namespace lumina {

constexpr int TQ_QMAX = 32639;  // 256 * 127 + 127
constexpr int TQ_CH = 4;        // items per thread per pass
constexpr int TQ_MAX_ADD = 8;   // addend rows (tensor-parallel ranks)

__device__ __forceinline__ void tq_load8(float (&v)[8], const float* p, int k0, int K, bool vec) {
  if (vec && k0 + 8 <= K) {
    const float4 f0 = *reinterpret_cast<const float4*>(p + k0);
    const float4 f1 = *reinterpret_cast<const float4*>(p + k0 + 4);
    v[0] = f0.x; v[1] = f0.y; v[2] = f0.z; v[3] = f0.w;
    v[4] = f1.x; v[5] = f1.y; v[6] = f1.z; v[7] = f1.w;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = k0 + j < K ? p[k0 + j] : 0.f;
  }
}

__device__ __forceinline__ void tq_ldg8(float (&v)[8], const float* p, int k0, int K, bool vec) {
  if (vec && k0 + 8 <= K) {
    const float4 f0 = __ldg(reinterpret_cast<const float4*>(p + k0));
    const float4 f1 = __ldg(reinterpret_cast<const float4*>(p + k0 + 4));
    v[0] = f0.x; v[1] = f0.y; v[2] = f0.z; v[3] = f0.w;
    v[4] = f1.x; v[5] = f1.y; v[6] = f1.z; v[7] = f1.w;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = k0 + j < K ? __ldg(p + k0 + j) : 0.f;
  }
}

// norm weights of this thread's first-pass items (zeros elsewhere)
template <int NB>
__device__ __forceinline__ void tq_preload(float (&w)[TQ_CH][8], const float* nw, int K, int P) {
  const int n_items = NB * P * 8;
  const bool vec = (reinterpret_cast<uintptr_t>(nw) & 15) == 0;
#pragma unroll
  for (int u = 0; u < TQ_CH; ++u) {
    const int i = threadIdx.x + u * blockDim.x;
#pragma unroll
    for (int j = 0; j < 8; ++j) w[u][j] = 0.f;
    if (i < n_items) tq_ldg8(w[u], nw, (i % (P * 8)) * 8, K, vec);
  }
}

// per-row sums of squares of the CTA -> rinv (every thread); red holds
// NB x NW floats; one barrier
template <int NB, int NW>
__device__ __forceinline__ void tq_rinv(float (&ss)[NB], float (&rinv)[NB], float* red, int K, float eps) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const float s = warp_sum(ss[b]);
    if (lane == 0) red[b * NW + warp] = s;
  }
  __syncthreads();
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) tot += red[b * NW + w];
    rinv[b] = 1.0f / sqrtf(tot / (float)K + eps);
  }
}

// the rows other GPUs wrote (a tensor-parallel sum): read through L2, never
// from a stale L1 line
__device__ __forceinline__ void tq_add8(float (&v)[8], const float* p, int k0, int K, bool vec) {
  if (vec && k0 + 8 <= K) {
    const float4 f0 = __ldcg(reinterpret_cast<const float4*>(p + k0));
    const float4 f1 = __ldcg(reinterpret_cast<const float4*>(p + k0 + 4));
    v[0] += f0.x; v[1] += f0.y; v[2] += f0.z; v[3] += f0.w;
    v[4] += f1.x; v[5] += f1.y; v[6] += f1.z; v[7] += f1.w;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (k0 + j < K) v[j] += __ldcg(p + k0 + j);
  }
}

// the input rows: x, plus (n_add > 0) the rank-ordered sum of the add[]
// rows; `xout` (may be null) receives them before any normalization.
// tq_run takes it by pointer: null (every one-GPU launch) compiles it out
struct TqSum {
  const float* add[TQ_MAX_ADD] = {};
  int n_add = 0;
  float* xout = nullptr;
};

// NB rows (nb live, row stride ldx) -> xb [P][2 NB][4 lanes] uint4 and
// fq [P][NB] (sx, -lv * sum q; lv = levels - 1 of the codes); NW warps; the caller syncs the CTA before reading xb / fq
template <int NB, int NW, bool NORM>
__device__ __forceinline__ void tq_run(const float* x, int ldx, int nb, int K, int P, const float* nw, float eps,
                                       const float (&w)[TQ_CH][8], uint4* xb, int2* fq, float* red, int lv,
                                       const TqSum* sum = nullptr) {
  constexpr int NC = 2 * NB;
  const int n_items = NB * P * 8, per_pass = TQ_CH * (int)blockDim.x;
  const bool vec_x = ((ldx & 3) == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  const bool vec_w = (reinterpret_cast<uintptr_t>(nw) & 15) == 0;
  const bool one_pass = n_items <= per_pass;
  float rinv[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) rinv[b] = 1.f;
  if (NORM && !one_pass) {
    float ss[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      ss[b] = 0.f;
      if (b < nb)
        for (int k = threadIdx.x; k < K; k += blockDim.x) {
          float v = x[(size_t)b * ldx + k];
          if (sum) {
#pragma unroll
            for (int r = 0; r < TQ_MAX_ADD; ++r)
              if (r < sum->n_add) v += __ldcg(sum->add[r] + (size_t)b * ldx + k);
          }
          ss[b] = fmaf(v, v, ss[b]);
        }
    }
    tq_rinv<NB, NW>(ss, rinv, red, K, eps);
  }
  for (int base = 0; base < n_items; base += per_pass) {
    float v[TQ_CH][8];
    int row[TQ_CH];
    // every load of the pass goes out before any is used
#pragma unroll
    for (int u = 0; u < TQ_CH; ++u) {
      const int i = base + u * (int)blockDim.x + (int)threadIdx.x;
      const int b = i / (P * 8), k0 = (i % (P * 8)) * 8;
      row[u] = b;
#pragma unroll
      for (int j = 0; j < 8; ++j) v[u][j] = 0.f;
      if (i < n_items && b < nb) tq_load8(v[u], x + (size_t)b * ldx, k0, K, vec_x);
    }
    if (sum && sum->n_add > 0) {
      // x + rank 0 + rank 1 + ... (the same order on every rank)
#pragma unroll
      for (int r = 0; r < TQ_MAX_ADD; ++r) {
        if (r >= sum->n_add) break;
#pragma unroll
        for (int u = 0; u < TQ_CH; ++u) {
          const int i = base + u * (int)blockDim.x + (int)threadIdx.x;
          if (i < n_items && row[u] < nb) tq_add8(v[u], sum->add[r] + (size_t)row[u] * ldx, (i % (P * 8)) * 8, K, vec_x);
        }
      }
      if (sum->xout && blockIdx.x == 0) {
#pragma unroll
        for (int u = 0; u < TQ_CH; ++u) {
          const int i = base + u * (int)blockDim.x + (int)threadIdx.x;
          const int k0 = (i % (P * 8)) * 8;
          if (i < n_items && row[u] < nb)
#pragma unroll
            for (int j = 0; j < 8; ++j)
              if (k0 + j < K) sum->xout[(size_t)row[u] * ldx + k0 + j] = v[u][j];
        }
      }
    }
    if constexpr (NORM) {
      if (one_pass) {
        float ss[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) ss[b] = 0.f;
#pragma unroll
        for (int u = 0; u < TQ_CH; ++u) {
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < 8; ++j) s = fmaf(v[u][j], v[u][j], s);
#pragma unroll
          for (int b = 0; b < NB; ++b)
            if (row[u] == b) ss[b] += s;
        }
        tq_rinv<NB, NW>(ss, rinv, red, K, eps);
      }
#pragma unroll
      for (int u = 0; u < TQ_CH; ++u) {
        float r = 0.f;
#pragma unroll
        for (int b = 0; b < NB; ++b)
          if (row[u] == b) r = rinv[b];
        float wv[8];
        if (base == 0) {
#pragma unroll
          for (int j = 0; j < 8; ++j) wv[j] = w[u][j];
        } else {
          const int i = base + u * (int)blockDim.x + (int)threadIdx.x;
#pragma unroll
          for (int j = 0; j < 8; ++j) wv[j] = 0.f;
          if (i < n_items) tq_ldg8(wv, nw, (i % (P * 8)) * 8, K, vec_w);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) v[u][j] = (v[u][j] * r) * wv[j];
      }
    }
#pragma unroll
    for (int u = 0; u < TQ_CH; ++u) {
      if (base + u * (int)blockDim.x >= n_items) break;  // CTA-uniform
      const int i = base + u * (int)blockDim.x + (int)threadIdx.x;
      const bool item = i < n_items;
      const int b = item ? row[u] : 0, p = item ? (i >> 3) % P : 0, oc = i & 7;
      float amax = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[u][j]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
      uint32_t hw[2] = {0, 0}, lw[2] = {0, 0};
      int qs = 0;
      float sxv = 0.f;
      if (amax > 0.f) {
        const float f = __fdiv_rn((float)TQ_QMAX, amax);
        sxv = __fdiv_rn(amax, (float)TQ_QMAX);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          int q = __float2int_rn(__fmul_rn(v[u][j], f));
          q = max(-TQ_QMAX, min(TQ_QMAX, q));
          qs += q;
          const int qh = (q + 128) >> 8, ql = q - 256 * qh;
          hw[j >> 2] |= ((uint32_t)qh & 0xFFu) << (8 * (j & 3));
          lw[j >> 2] |= ((uint32_t)ql & 0xFFu) << (8 * (j & 3));
        }
      }
      qs += __shfl_xor_sync(0xffffffffu, qs, 1);
      qs += __shfl_xor_sync(0xffffffffu, qs, 2);
      qs += __shfl_xor_sync(0xffffffffu, qs, 4);
      if (!item) continue;
      // columns 8 oc .. 8 oc + 7 of the pair: k32 block oc >> 2, register
      // (oc >> 1) & 1 of lanes t = 2 (oc & 1) and the next, 4 columns each
      const int comp = ((oc >> 2) << 1) | ((oc >> 1) & 1), tt0 = 2 * (oc & 1);
      uint32_t* xw = reinterpret_cast<uint32_t*>(xb + (size_t)(p * NC + 2 * b) * 4);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        xw[(tt0 + e) * 4 + comp] = hw[e];
        xw[16 + (tt0 + e) * 4 + comp] = lw[e];
      }
      if (oc == 0) fq[(size_t)p * NB + b] = make_int2(__float_as_int(sxv), -lv * qs);
    }
  }
}

}  // namespace lumina
