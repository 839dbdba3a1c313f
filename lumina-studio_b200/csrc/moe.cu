// Virtual-MoE MLP of a decoder layer on the device: the routed branch of
// chat.py:_layer (285-299) calling qwen_next.py:moe_grouped_forward (31-78)
// with weight_mode="unit", gate_fn="sigmoid" and the router on the
// normalized row (router_feat "raw": ChatModel keeps only experts / ie /
// top_k of the header entry, chat.py:181-183).
//
// Layout. The experts are the flat matrices the reference's converter writes
// (virtual_moe.py:228-231), packed int4 in the row-major chunk layout
// (weights.cuh):
//   gate_up  (E*2Ie, D): expert e's gate rows e*2Ie + i, up rows e*2Ie + Ie + i
//   down     (E*Ie,  D): row e*Ie + i holds neuron i's D output weights; the
//                        product is down[e]^T a, so scale groups run along
//                        the OUTPUT dimension (a transposed GEMV)
// plus the router (E, D) and its bias (E), raw tensors rounded to fp16 as
// ChatModel rounds every tensor (chat.py:140).
//
// Kernels (one launch each per layer, grids fixed by the shapes so that a
// captured decode graph replays them):
//  * moe_route_kernel, one CTA per row: RMSNorm (chat.py:284, the same fp32
//    arithmetic as the GEMV prologues), router logits h . router[e] + b[e],
//    sigmoid scores with the +-40 clip (qwen_next.py:23-24), top-k by
//    descending score with ties to the lower expert index (numpy's argsort
//    of -scores, qwen_next.py:63, is an insertion sort for E <= 16 and so
//    keeps index order on ties).
//  * moe_gu_kernel, grid (expert, tile of MOE_PPC neuron pairs): rows are
//    taken in passes of MOE_ROWS; a CTA whose expert no row of the pass
//    picked skips the pass without touching its weights, so only the
//    touched experts stream from HBM. A warp owns one (gate, up) row pair
//    at a time, each lane a 16-byte chunk (32 codes) per row; the codes are
//    widened to fp32 once and dotted against every picking row held in
//    shared memory:
//      sum_k h_k * level(c_k) = s/15 * (2 * sum h_k c_k - 15 * sum h_k)
//    per 32-column chunk (one scale; level(c) = (2c - 15)/15,
//    adapters/lumina.py:135-139), then silu(g) * u with the +-40 clip
//    (qwen_next.py:71-72).
//  * moe_down_kernel, grid (64-column slice, MOE_SPLITS neuron ranges): 8
//    lanes decode 8 columns each of one down row, so a warp covers four rows
//    of a slice per load; a lane accumulates its 8 columns for up to
//    MOE_ROWS batch rows. Partial sums reduce in a fixed order -- shuffles
//    over the four row lanes, the 8 warps in shared memory, then the splits
//    in index order by the CTA that finishes a slice last (found with a
//    per-slice counter it resets for the next launch) -- which also adds the
//    residual (chat.py:299: x + d). Results therefore do not depend on CTA
//    timing.
#include "model.cuh"

namespace lumina {

namespace {

constexpr int MOE_THREADS = 256;
constexpr int MOE_WARPS = MOE_THREADS / 32;

// fp32 value of byte j (0..3) of v: the byte becomes the low mantissa bits
// of 2^23 and the exponent bias is subtracted again (exact for 0..255).
__device__ __forceinline__ float byte_to_float(uint32_t v, uint32_t j) {
  return __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7540u | j)) - 8388608.f;
}

// the 32 int4 codes of one 16-byte chunk as floats, column order
__device__ __forceinline__ void decode_chunk(const uint4& v, float (&c)[32]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t lo = w[q] & 0x0F0F0F0Fu, hi = (w[q] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      c[8 * q + 2 * j] = byte_to_float(lo, j);
      c[8 * q + 2 * j + 1] = byte_to_float(hi, j);
    }
  }
}

template <typename ST>
__device__ __forceinline__ float moe_scale(const lumina_weight& w, int row, int g) {
  const uint8_t* p = w.scales + scale_offset(w, row, g);
  if constexpr (sizeof(ST) == 2) return __half2float(*reinterpret_cast<const __half*>(p));
  else return *reinterpret_cast<const float*>(p);
}

__device__ __forceinline__ float silu_mul(float g, float u) {
  const float e = expf(-fminf(fmaxf(g, -40.f), 40.f));
  return g / (1.0f + e) * u;
}

// ---------------------------------------------------------------------------
// router
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(MOE_THREADS)
moe_route_kernel(const float* __restrict__ x, int d, const float* __restrict__ norm_w, float eps,
                 const float* __restrict__ rw, const float* __restrict__ rb, int E, int K, float* __restrict__ h,
                 int* __restrict__ sel) {
  extern __shared__ float hs[];  // d floats
  __shared__ float red[MOE_WARPS];
  __shared__ float score[MOE_MAX_E];
  const int r = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* xr = x + (size_t)r * d;
  // chat.py:63-66: x / sqrt(mean(x^2) + eps) * w, fp32
  float ss = 0.f;
  for (int k = threadIdx.x; k < d; k += MOE_THREADS) ss = fmaf(xr[k], xr[k], ss);
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < MOE_WARPS; ++i) tot += red[i];
  const float inv = 1.0f / sqrtf(tot / (float)d + eps);
  for (int k = threadIdx.x; k < d; k += MOE_THREADS) {
    const float v = (xr[k] * inv) * norm_w[k];
    hs[k] = v;
    h[(size_t)r * d + k] = v;
  }
  __syncthreads();
  // logits = h @ router^T (+ bias), sigmoid scores (qwen_next.py:57-61)
  for (int e = warp; e < E; e += MOE_WARPS) {
    const float* w = rw + (size_t)e * d;
    float acc = 0.f;
    for (int k = lane; k < d; k += 32) acc = fmaf(hs[k], w[k], acc);
    acc = warp_sum(acc);
    if (lane == 0) {
      const float lg = acc + (rb ? rb[e] : 0.f);
      score[e] = 1.0f / (1.0f + expf(-fminf(fmaxf(lg, -40.f), 40.f)));
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long taken = 0ull;
    for (int j = 0; j < K; ++j) {
      int best = -1;
      for (int e = 0; e < E; ++e)
        if (!((taken >> e) & 1ull) && (best < 0 || score[e] > score[best])) best = e;
      taken |= 1ull << best;
      sel[r * K + j] = best;
    }
  }
}

// ---------------------------------------------------------------------------
// gate/up of the picked experts + SwiGLU
// ---------------------------------------------------------------------------
// slot of expert e in row r's picks, or -1
__device__ __forceinline__ int pick_slot(const int* sel, int r, int K, int e) {
  for (int j = 0; j < K; ++j)
    if (sel[r * K + j] == e) return j;
  return -1;
}

template <typename ST>
__global__ void __launch_bounds__(MOE_THREADS)
moe_gu_kernel(const lumina_weight w, const float* __restrict__ h, int d, int n, const int* __restrict__ sel, int K,
              int Ie, float* __restrict__ act) {
  extern __shared__ __align__(16) float sm[];
  // hsw: MOE_ROWS rows of h, 4 pad floats after every 32 (conflict-free
  // 16-byte reads when lanes take consecutive chunks); hsum: per row and chunk
  const int nch = d >> 5, ldh = d + (d >> 3);
  float* hsw = sm;
  float* hsum = sm + MOE_ROWS * ldh;
  __shared__ int slot[MOE_ROWS];
  const int e = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int p0 = blockIdx.y * MOE_PPC;
  for (int r0 = 0; r0 < n; r0 += MOE_ROWS) {
    __syncthreads();  // the previous pass is done with slot / hsw
    if (threadIdx.x < MOE_ROWS) {
      const int r = r0 + threadIdx.x;
      slot[threadIdx.x] = r < n ? pick_slot(sel, r, K, e) : -1;
    }
    __syncthreads();
    int sl[MOE_ROWS];
    bool any = false;
#pragma unroll
    for (int q = 0; q < MOE_ROWS; ++q) {
      sl[q] = slot[q];
      any |= sl[q] >= 0;
    }
    if (!any) continue;
#pragma unroll
    for (int q = 0; q < MOE_ROWS; ++q) {
      if (sl[q] < 0) continue;
      const float* hr = h + (size_t)(r0 + q) * d;
      for (int k = threadIdx.x; k < d; k += MOE_THREADS) hsw[q * ldh + k + 4 * (k >> 5)] = hr[k];
    }
    __syncthreads();
    for (int t = warp; t < MOE_ROWS * nch; t += MOE_WARPS) {
      const int q = t / nch, c = t - q * nch;
      if (sl[q] < 0) continue;
      const float v = warp_sum(hsw[q * ldh + c * 36 + lane]);
      if (lane == 0) hsum[q * nch + c] = v;
    }
    __syncthreads();
    for (int pi = warp; pi < MOE_PPC; pi += MOE_WARPS) {
      const int i = p0 + pi;
      if (i >= Ie) break;
      const int rg = e * 2 * Ie + i, ru = rg + Ie;
      float ag[MOE_ROWS], au[MOE_ROWS];
#pragma unroll
      for (int q = 0; q < MOE_ROWS; ++q) ag[q] = au[q] = 0.f;
      for (int cb = 0; cb < nch; cb += 128) {
        uint4 wg[4], wu[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = cb + u * 32 + lane;
          if (c < nch) {
            wg[u] = ldg_stream(w.codes + code_offset(w, rg, c));
            wu[u] = ldg_stream(w.codes + code_offset(w, ru, c));
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = cb + u * 32 + lane;
          if (c >= nch) continue;
          const int grp = (c << 5) / w.group;
          const float sg = moe_scale<ST>(w, rg, grp), su = moe_scale<ST>(w, ru, grp);
          float cg[32], cu[32];
          decode_chunk(wg[u], cg);
          decode_chunk(wu[u], cu);
#pragma unroll
          for (int q = 0; q < MOE_ROWS; ++q) {
            if (sl[q] < 0) continue;
            const float* hv = hsw + q * ldh + c * 36;
            float dg = 0.f, du = 0.f;
#pragma unroll
            for (int t4 = 0; t4 < 8; ++t4) {
              const float4 hh = *reinterpret_cast<const float4*>(hv + 4 * t4);
              dg = fmaf(hh.x, cg[4 * t4], dg);
              dg = fmaf(hh.y, cg[4 * t4 + 1], dg);
              dg = fmaf(hh.z, cg[4 * t4 + 2], dg);
              dg = fmaf(hh.w, cg[4 * t4 + 3], dg);
              du = fmaf(hh.x, cu[4 * t4], du);
              du = fmaf(hh.y, cu[4 * t4 + 1], du);
              du = fmaf(hh.z, cu[4 * t4 + 2], du);
              du = fmaf(hh.w, cu[4 * t4 + 3], du);
            }
            const float m15 = -15.f * hsum[q * nch + c];
            ag[q] = fmaf(sg, fmaf(2.f, dg, m15), ag[q]);
            au[q] = fmaf(su, fmaf(2.f, du, m15), au[q]);
          }
        }
      }
#pragma unroll
      for (int q = 0; q < MOE_ROWS; ++q) {
        if (sl[q] < 0) continue;
        const float g = warp_sum(ag[q]) / 15.f, u = warp_sum(au[q]) / 15.f;
        if (lane == 0) act[((size_t)(r0 + q) * K + sl[q]) * Ie + i] = silu_mul(g, u);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// transposed down projection of the picked experts + residual
// ---------------------------------------------------------------------------
template <typename ST>
__global__ void __launch_bounds__(MOE_THREADS)
moe_down_kernel(const lumina_weight w, int d, int n, const int* __restrict__ sel, int E, int K, int Ie,
                const float* __restrict__ act, float* __restrict__ part, unsigned int* __restrict__ counters,
                float* __restrict__ x) {
  __shared__ float red[MOE_WARPS][MOE_ROWS][64];
  __shared__ int slot[MOE_ROWS];
  __shared__ int last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c0 = blockIdx.x * 64, split = blockIdx.y, S = gridDim.y;
  const int ib = (int)((long long)Ie * split / S), ie = (int)((long long)Ie * (split + 1) / S);
  const int rsub = lane >> 3, cl = lane & 7;
  const int grp = c0 / w.group;
  const size_t coff = (size_t)(c0 >> 1) + 4 * cl;  // this lane's 4 code bytes within a row
  for (int r0 = 0; r0 < n; r0 += MOE_ROWS) {
    float acc[MOE_ROWS][8];
#pragma unroll
    for (int q = 0; q < MOE_ROWS; ++q)
#pragma unroll
      for (int t = 0; t < 8; ++t) acc[q][t] = 0.f;
    for (int e = 0; e < E; ++e) {
      __syncthreads();
      if (threadIdx.x < MOE_ROWS) {
        const int r = r0 + threadIdx.x;
        slot[threadIdx.x] = r < n ? pick_slot(sel, r, K, e) : -1;
      }
      __syncthreads();
      int sl[MOE_ROWS];
      bool any = false;
#pragma unroll
      for (int q = 0; q < MOE_ROWS; ++q) {
        sl[q] = slot[q];
        any |= sl[q] >= 0;
      }
      if (!any) continue;
      const float* ap[MOE_ROWS];
#pragma unroll
      for (int q = 0; q < MOE_ROWS; ++q) ap[q] = act + ((size_t)(r0 + q) * K + (sl[q] < 0 ? 0 : sl[q])) * Ie;
#pragma unroll 4
      for (int i = ib + warp * 4 + rsub; i < ie; i += 4 * MOE_WARPS) {
        const int R = e * Ie + i;
        const uint32_t wv = __ldg(reinterpret_cast<const uint32_t*>(w.codes + (size_t)R * w.row_bytes + coff));
        const float s = moe_scale<ST>(w, R, grp);
        const uint32_t lo = wv & 0x0F0F0F0Fu, hi = (wv >> 4) & 0x0F0F0F0Fu;
        float lv[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          lv[2 * j] = fmaf(2.f, byte_to_float(lo, j), -15.f);
          lv[2 * j + 1] = fmaf(2.f, byte_to_float(hi, j), -15.f);
        }
#pragma unroll
        for (int q = 0; q < MOE_ROWS; ++q) {
          if (sl[q] < 0) continue;
          const float coef = __ldg(ap[q] + i) * s;
#pragma unroll
          for (int t = 0; t < 8; ++t) acc[q][t] = fmaf(coef, lv[t], acc[q][t]);
        }
      }
    }
    // lanes l, l+8, l+16, l+24 hold the same columns: fold them, then the warps
#pragma unroll
    for (int q = 0; q < MOE_ROWS; ++q)
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        float v = acc[q][t];
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        if (rsub == 0) red[warp][q][cl * 8 + t] = v;
      }
    __syncthreads();
    for (int idx = threadIdx.x; idx < MOE_ROWS * 64; idx += MOE_THREADS) {
      const int q = idx >> 6, col = idx & 63;
      if (r0 + q >= n) continue;
      float v = 0.f;
#pragma unroll
      for (int wi = 0; wi < MOE_WARPS; ++wi) v += red[wi][q][col];
      part[((size_t)split * n + r0 + q) * d + c0 + col] = v / 15.f;
    }
  }
  // the CTA that completes this slice adds the splits in index order
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(&counters[blockIdx.x], 1u) == (unsigned)(S - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int idx = threadIdx.x; idx < n * 64; idx += MOE_THREADS) {
    const int r = idx >> 6, col = c0 + (idx & 63);
    float v = 0.f;
    for (int s2 = 0; s2 < S; ++s2) v += __ldcg(part + ((size_t)s2 * n + r) * d + col);
    x[(size_t)r * d + col] += v;
  }
  if (threadIdx.x == 0) counters[blockIdx.x] = 0u;
}

size_t gu_smem_bytes(int d) { return (size_t)(MOE_ROWS * (d + d / 8) + MOE_ROWS * (d / 32)) * 4; }

}  // namespace

int moe_check(const MoeLayerArgs& a) {
  const lumina_weight* gu = a.gate_up;
  const lumina_weight* dn = a.down;
  if (!gu || !dn || !a.router_w) {
    set_error("virtual-MoE layer: missing experts.gate_up_proj, experts.down_proj or gate.weight");
    return LUMINA_E_STATE;
  }
  if (a.E < 1 || a.E > MOE_MAX_E || a.K < 1 || a.K > a.E || a.K > MOE_MAX_K || a.Ie < 1) {
    set_error("virtual-MoE layer: experts %d / top_k %d / ie %d outside 1..%d / 1..min(E, %d) / >= 1", a.E, a.K,
              a.Ie, MOE_MAX_E, MOE_MAX_K);
    return LUMINA_E_ARG;
  }
  if (gu->rows != a.E * 2 * a.Ie || dn->rows != a.E * a.Ie || gu->cols != a.d || dn->cols != a.d) {
    set_error("virtual-MoE layer: gate_up (%d, %d) / down (%d, %d) do not match E %d, ie %d, d %d", gu->rows,
              gu->cols, dn->rows, dn->cols, a.E, a.Ie, a.d);
    return LUMINA_E_ARG;
  }
  if (gu->bits != 4 || dn->bits != 4 || gu->mma || dn->mma || gu->group % 64 || dn->group % 64 ||
      gu->fp16_scales != dn->fp16_scales || a.d % 64) {
    set_error("virtual-MoE experts are built for int4 with groups of 64k in the row-major layout, d %% 64 == 0");
    return LUMINA_E_UNSUPPORTED;
  }
  if (gu_smem_bytes(a.d) > 200 * 1024) {
    set_error("virtual-MoE layer: d %d too wide for the shared-memory row stage", a.d);
    return LUMINA_E_UNSUPPORTED;
  }
  return LUMINA_OK;
}

int moe_prepare(int d) {
  const int smem = (int)gu_smem_bytes(d);
  LUMINA_CUDA_TRY(cudaFuncSetAttribute(moe_gu_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  LUMINA_CUDA_TRY(cudaFuncSetAttribute(moe_gu_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  return LUMINA_OK;
}

int launch_moe(const MoeLayerArgs& a, int n, const MoeScratch& sc, float* x, cudaStream_t s) {
  const int d = a.d;
  moe_route_kernel<<<n, MOE_THREADS, d * 4, s>>>(x, d, a.norm_w, a.eps, a.router_w, a.router_b, a.E, a.K, sc.h,
                                                 sc.sel);
  LUMINA_LAUNCH_CHECK();
  const dim3 ggu(a.E, (a.Ie + MOE_PPC - 1) / MOE_PPC);
  const size_t smem = gu_smem_bytes(d);
  if (a.gate_up->fp16_scales)
    moe_gu_kernel<__half><<<ggu, MOE_THREADS, smem, s>>>(*a.gate_up, sc.h, d, n, sc.sel, a.K, a.Ie, sc.act);
  else
    moe_gu_kernel<float><<<ggu, MOE_THREADS, smem, s>>>(*a.gate_up, sc.h, d, n, sc.sel, a.K, a.Ie, sc.act);
  LUMINA_LAUNCH_CHECK();
  const dim3 gdn(d / 64, MOE_SPLITS);
  if (a.down->fp16_scales)
    moe_down_kernel<__half><<<gdn, MOE_THREADS, 0, s>>>(*a.down, d, n, sc.sel, a.E, a.K, a.Ie, sc.act, sc.part,
                                                        sc.counters, x);
  else
    moe_down_kernel<float><<<gdn, MOE_THREADS, 0, s>>>(*a.down, d, n, sc.sel, a.E, a.K, a.Ie, sc.act, sc.part,
                                                       sc.counters, x);
  LUMINA_LAUNCH_CHECK();
  return LUMINA_OK;
}

}  // namespace lumina
