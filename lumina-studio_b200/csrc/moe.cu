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
// Kernels (one launch each per layer, grids fixed by the row count so that
// a captured decode graph replays them):
//  * moe_route_kernel, grid (row, expert): the row's RMSNorm (chat.py:284,
//    the same fp32 arithmetic as the GEMV prologues) and its router logit
//    h . router[e] + b[e] as a sigmoid score with the +-40 clip
//    (qwen_next.py:23-24). One CTA per (row, expert) keeps every load of the
//    row and the router row in flight at once; the router row is fetched
//    before the dependency wait. The three kernels chain with programmatic
//    dependent launch, so each one's CTAs are resident before its
//    predecessor ends.
//  * The expert kernels take rows in passes of up to MOE_ROWS and derive the
//    picks of a pass from the scores themselves: top-k by descending score
//    (qwen_next.py:63, np.argsort(-scores)[:, :k]) with exact ties to the
//    lower expert index (numpy's sort is not stable, so the reference orders
//    exact ties by its sort algorithm; both pick the same score values), and
//    the distinct experts the pass touches.
//  * moe_gu_kernel, grid (touched-expert slot, tile of neuron pairs): CTA x
//    works for the x-th expert the pass touches, so only touched experts
//    stream from HBM and, at decode, every CTA has work. A tile is MOE_PPC
//    pairs at decode and 8 x MOE_PPC for passes of several rows (the rows
//    are staged once per CTA). One warp per (gate, up) row pair at a time,
//    each lane a 16-byte chunk (32 codes) per row; the codes are widened to
//    fp32 once and dotted against every picking row
//    held in shared memory:
//      sum_k h_k * level(c_k) = s/15 * (2 * sum h_k c_k - 15 * sum h_k)
//    per 32-column chunk (one scale; level(c) = (2c - 15)/15,
//    adapters/lumina.py:135-139), then silu(g) * u with the +-40 clip
//    (qwen_next.py:71-72).
//  * moe_down_kernel, grid (64-column slice, neuron range): 8 lanes decode 8
//    columns each of one down row, so a warp covers four rows of a slice per
//    load; a lane accumulates its 8 columns for every row of the pass.
//    Partial sums reduce in a fixed order -- shuffles over the four row
//    lanes, the 8 warps in shared memory, then the neuron ranges in index
//    order by the CTA that finishes a slice last (found with a per-slice
//    counter it resets for the next launch) -- which also adds the residual
//    (chat.py:299: x + d). Results therefore do not depend on CTA timing.
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
constexpr int ROUTE_THREADS = 128;

__device__ __forceinline__ float block_sum_route(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();  // red is free again
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < ROUTE_THREADS / 32; ++i) t += red[i];
  return t;
}

// CTA (row r, expert e): the row's RMSNorm and its router logit for e, as
// a sigmoid score. Every CTA of a row computes the same norm factor (same
// loads, same order), so h is one value everywhere; expert 0's CTA stores it.
// The router and norm rows do not depend on the previous kernel: they are
// staged in shared memory before the dependency wait.
__global__ void __launch_bounds__(ROUTE_THREADS)
moe_route_kernel(const float* __restrict__ x, int d, const float* __restrict__ norm_w, float eps,
                 const float* __restrict__ rw, const float* __restrict__ rb, int E, float* __restrict__ h,
                 float* __restrict__ score) {
  extern __shared__ __align__(16) float4 rs[];  // [d/4] router row e, [d/4] norm weight
  __shared__ float red[ROUTE_THREADS / 32];
  const int r = blockIdx.x, e = blockIdx.y;
  const int d4 = d >> 2;
  const float4* wr = reinterpret_cast<const float4*>(rw + (size_t)e * d);
  const float4* nw = reinterpret_cast<const float4*>(norm_w);
#pragma unroll 8
  for (int k = threadIdx.x; k < d4; k += ROUTE_THREADS) {
    rs[k] = __ldg(wr + k);
    rs[d4 + k] = __ldg(nw + k);
  }
  const float bias = rb ? __ldg(rb + e) : 0.f;
  pdl_launch_dependents();
  pdl_wait();
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)r * d);
  // chat.py:63-66: x / sqrt(mean(x^2) + eps) * w, fp32
  float ss = 0.f;
#pragma unroll 8
  for (int k = threadIdx.x; k < d4; k += ROUTE_THREADS) {
    const float4 v = xr[k];
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
  }
  const float inv = 1.0f / sqrtf(block_sum_route(ss, red) / (float)d + eps);
  // logit = h . router[e] (+ bias), score = sigmoid with the +-40 clip (qwen_next.py:23-24, 57-61)
  float acc = 0.f;
#pragma unroll 8
  for (int k = threadIdx.x; k < d4; k += ROUTE_THREADS) {
    const float4 v = xr[k], w = rs[d4 + k], q = rs[k];
    float4 hv;
    hv.x = (v.x * inv) * w.x;
    hv.y = (v.y * inv) * w.y;
    hv.z = (v.z * inv) * w.z;
    hv.w = (v.w * inv) * w.w;
    acc = fmaf(hv.x, q.x, acc);
    acc = fmaf(hv.y, q.y, acc);
    acc = fmaf(hv.z, q.z, acc);
    acc = fmaf(hv.w, q.w, acc);
    if (e == 0) reinterpret_cast<float4*>(h + (size_t)r * d)[k] = hv;
  }
  const float lg = block_sum_route(acc, red) + bias;
  if (threadIdx.x == 0) score[(size_t)r * MOE_MAX_E + e] = 1.0f / (1.0f + expf(-fminf(fmaxf(lg, -40.f), 40.f)));
}

// ---------------------------------------------------------------------------
// the picks of a pass of rows, shared by the expert kernels
// ---------------------------------------------------------------------------
// top-k of a row by descending score (np.argsort(-scores)[:, :k],
// qwen_next.py:63), exact ties to the lower expert index
__device__ __forceinline__ void topk_row(const float* sc, int E, int K, int* out) {
  unsigned long long taken = 0ull;
  for (int j = 0; j < K; ++j) {
    int best = -1;
    float bv = 0.f;
    for (int e = 0; e < E; ++e) {
      const float v = sc[e];
      if (!((taken >> e) & 1ull) && (best < 0 || v > bv)) {
        best = e;
        bv = v;
      }
    }
    taken |= 1ull << best;
    out[j] = best;
  }
}

// Rows r0 .. r0+pr-1: their picks, and the distinct experts they touch in
// ascending order (thread 0 fills the shared tables).
struct PassPicks {
  int pick[MOE_ROWS][MOE_MAX_K];
  int touched[MOE_MAX_E];
  signed char slot[MOE_MAX_E][MOE_ROWS];  // slot of touched[x] among row q's picks, or -1
  int nt;
};

// Only this rank's experts [e_lo, e_lo + e_n) count as touched (all E
// without expert parallelism).
__device__ __forceinline__ void pass_picks(const float* __restrict__ score, int r0, int pr, int E, int K,
                                           int e_lo, int e_n, PassPicks& pp) {
  if (threadIdx.x == 0) {
    unsigned long long used = 0ull;
    for (int q = 0; q < pr; ++q) {
      topk_row(score + (size_t)(r0 + q) * MOE_MAX_E, E, K, pp.pick[q]);
      for (int j = 0; j < K; ++j) used |= 1ull << pp.pick[q][j];
    }
    int nt = 0;
    for (int e = e_lo; e < e_lo + e_n; ++e)
      if ((used >> e) & 1ull) {
        for (int q = 0; q < MOE_ROWS; ++q) {
          signed char j = -1;
          for (int jj = 0; q < pr && jj < K; ++jj)
            if (pp.pick[q][jj] == e) j = (signed char)jj;
          pp.slot[nt][q] = j;
        }
        pp.touched[nt++] = e;
      }
    pp.nt = nt;
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// gate/up of the picked experts + SwiGLU
// ---------------------------------------------------------------------------
// grid (touched-expert slot x, pair tile): in each pass of PR rows, CTA x
// works for the x-th distinct expert the pass touches (if any); one (gate,
// up) row pair per warp. PR = 1 (decode) keeps registers low enough for
// several CTAs per SM.
template <typename ST, int PR>
__global__ void __launch_bounds__(MOE_THREADS, PR == 1 ? 3 : 1)
moe_gu_kernel(const lumina_weight w, const float* __restrict__ h, int d, int n, const float* __restrict__ score,
              int E, int K, int Ie, int e_lo, int e_n, int ppw, float* __restrict__ act) {
  extern __shared__ __align__(16) float sm[];
  // hsw: PR rows of h, 4 pad floats after every 32 (conflict-free 16-byte
  // reads when lanes take consecutive chunks); hsum: per row and chunk
  const int nch = d >> 5, ldh = d + (d >> 3);
  float* hsw = sm;
  float* hsum = sm + PR * ldh;
  __shared__ PassPicks pp;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // this CTA's neuron pairs: ppw rounds of MOE_PPC (one per warp); several
  // rounds let a CTA stage a pass's rows once for many pairs
  const int i0 = blockIdx.y * MOE_PPC * ppw + warp;
  // everything below reads the router's outputs (scores, h)
  pdl_launch_dependents();
  pdl_wait();
  for (int r0 = 0; r0 < n; r0 += PR) {
    const int rows = min(PR, n - r0);
    __syncthreads();  // the previous pass is done with pp / hsw
    pass_picks(score, r0, rows, E, K, e_lo, e_n, pp);
    if ((int)blockIdx.x >= pp.nt) continue;
    const int e = pp.touched[blockIdx.x];
    int sl[PR];
#pragma unroll
    for (int q = 0; q < PR; ++q) sl[q] = pp.slot[blockIdx.x][q];
#pragma unroll
    for (int q = 0; q < PR; ++q) {
      if (sl[q] < 0) continue;
      const float4* hr = reinterpret_cast<const float4*>(h + (size_t)(r0 + q) * d);
#pragma unroll 4
      for (int k4 = threadIdx.x; k4 < (d >> 2); k4 += MOE_THREADS) {
        const int k = k4 << 2;  // 4 columns inside one 32-column chunk
        *reinterpret_cast<float4*>(hsw + q * ldh + k + 4 * (k >> 5)) = hr[k4];
      }
    }
    __syncthreads();
    for (int t = warp; t < rows * nch; t += MOE_WARPS) {
      const int q = t / nch, c = t - q * nch;
      if (sl[q] < 0) continue;
      const float v = warp_sum(hsw[q * ldh + c * 36 + lane]);
      if (lane == 0) hsum[q * nch + c] = v;
    }
    __syncthreads();
    for (int rr = 0; rr < ppw; ++rr) {
      const int i = i0 + rr * MOE_PPC;  // this warp's neuron pair of round rr
      if (i >= Ie) break;
      const int rg = (e - e_lo) * 2 * Ie + i, ru = rg + Ie;  // the rank's rows of expert e
      float ag[PR], au[PR];
#pragma unroll
      for (int q = 0; q < PR; ++q) ag[q] = au[q] = 0.f;
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
          const uint32_t gw[4] = {wg[u].x, wg[u].y, wg[u].z, wg[u].w};
          const uint32_t uw[4] = {wu[u].x, wu[u].y, wu[u].z, wu[u].w};
          float dg[PR], du[PR];
#pragma unroll
          for (int q = 0; q < PR; ++q) dg[q] = du[q] = 0.f;
#pragma unroll
          for (int qw = 0; qw < 4; ++qw) {
            // word qw = columns 8qw .. 8qw+7: low nibbles even, high nibbles odd
            const uint32_t glo = gw[qw] & 0x0F0F0F0Fu, ghi = (gw[qw] >> 4) & 0x0F0F0F0Fu;
            const uint32_t ulo = uw[qw] & 0x0F0F0F0Fu, uhi = (uw[qw] >> 4) & 0x0F0F0F0Fu;
            float cg[8], cu[8];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              cg[2 * j] = byte_to_float(glo, j);
              cg[2 * j + 1] = byte_to_float(ghi, j);
              cu[2 * j] = byte_to_float(ulo, j);
              cu[2 * j + 1] = byte_to_float(uhi, j);
            }
#pragma unroll
            for (int q = 0; q < PR; ++q) {
              if (sl[q] < 0) continue;
              const float* hv = hsw + q * ldh + c * 36 + 8 * qw;
              const float4 h0 = *reinterpret_cast<const float4*>(hv);
              const float4 h1 = *reinterpret_cast<const float4*>(hv + 4);
              const float hh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
              for (int t = 0; t < 8; ++t) {
                dg[q] = fmaf(hh[t], cg[t], dg[q]);
                du[q] = fmaf(hh[t], cu[t], du[q]);
              }
            }
          }
#pragma unroll
          for (int q = 0; q < PR; ++q) {
            if (sl[q] < 0) continue;
            const float m15 = -15.f * hsum[q * nch + c];
            ag[q] = fmaf(sg, fmaf(2.f, dg[q], m15), ag[q]);
            au[q] = fmaf(su, fmaf(2.f, du[q], m15), au[q]);
          }
        }
      }
#pragma unroll
      for (int q = 0; q < PR; ++q) {
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
template <typename ST, int PR>
__global__ void __launch_bounds__(MOE_THREADS, PR == 1 ? 4 : 1)
moe_down_kernel(const lumina_weight w, int d, int n, const float* __restrict__ score, int E, int K, int Ie,
                int e_lo, int e_n, const float* __restrict__ act, float* __restrict__ part,
                unsigned int* __restrict__ counters, float* __restrict__ x, float* __restrict__ out) {
  __shared__ float red[MOE_WARPS][PR][64];
  __shared__ PassPicks pp;
  __shared__ int last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c0 = blockIdx.x * 64, split = blockIdx.y, S = gridDim.y;
  const int ib = (int)((long long)Ie * split / S), ie = (int)((long long)Ie * (split + 1) / S);
  const int rsub = lane >> 3, cl = lane & 7;
  const int grp = c0 / w.group;
  const size_t coff = (size_t)(c0 >> 1) + 4 * cl;  // this lane's 4 code bytes within a row
  const int range = ie - ib;
  // everything below reads the earlier kernels' outputs (scores, act, x)
  pdl_launch_dependents();
  pdl_wait();
  for (int r0 = 0; r0 < n; r0 += PR) {
    const int rows = min(PR, n - r0);
    float acc[PR][8];
#pragma unroll
    for (int q = 0; q < PR; ++q)
#pragma unroll
      for (int t = 0; t < 8; ++t) acc[q][t] = 0.f;
    __syncthreads();  // the previous pass is done with pp / red
    pass_picks(score, r0, rows, E, K, e_lo, e_n, pp);
    // (touched expert, neuron) pairs of this CTA's range, flattened so that
    // the loads of every touched expert are in flight together
    const int total = pp.nt * range;
#pragma unroll 4
    for (int t = warp * 4 + rsub; t < total; t += 4 * MOE_WARPS) {
      const int xe = t / range, i = ib + (t - xe * range);
      const int R = (pp.touched[xe] - e_lo) * Ie + i;  // the rank's row of expert touched[xe]
      const uint32_t wv = __ldg(reinterpret_cast<const uint32_t*>(w.codes + (size_t)R * w.row_bytes + coff));
      const float s = moe_scale<ST>(w, R, grp);
      float coef[PR];
#pragma unroll
      for (int q = 0; q < PR; ++q) {
        const int j = pp.slot[xe][q];
        coef[q] = j >= 0 ? __ldg(act + ((size_t)(r0 + q) * K + j) * Ie + i) * s : 0.f;
      }
      const uint32_t lo = wv & 0x0F0F0F0Fu, hi = (wv >> 4) & 0x0F0F0F0Fu;
      float lv[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        lv[2 * j] = fmaf(2.f, byte_to_float(lo, j), -15.f);
        lv[2 * j + 1] = fmaf(2.f, byte_to_float(hi, j), -15.f);
      }
#pragma unroll
      for (int q = 0; q < PR; ++q)
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[q][c] = fmaf(coef[q], lv[c], acc[q][c]);
    }
    // lanes l, l+8, l+16, l+24 hold the same columns: fold them, then the warps
#pragma unroll
    for (int q = 0; q < PR; ++q)
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        float v = acc[q][t];
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        if (rsub == 0) red[warp][q][cl * 8 + t] = v;
      }
    __syncthreads();
    for (int idx = threadIdx.x; idx < rows * 64; idx += MOE_THREADS) {
      const int q = idx >> 6, col = idx & 63;
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
    if (out) out[(size_t)r * d + col] = v;  // this rank's share, summed over the ranks afterwards
    else x[(size_t)r * d + col] += v;
  }
  if (threadIdx.x == 0) counters[blockIdx.x] = 0u;
}

size_t gu_smem_bytes(int d, int pr) { return (size_t)(pr * (d + d / 8) + pr * (d / 32)) * 4; }

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
  if (a.e_n < 1 || a.e_lo < 0 || a.e_lo + a.e_n > a.E) {
    set_error("virtual-MoE layer: local experts [%d, %d) outside 0..%d", a.e_lo, a.e_lo + a.e_n, a.E);
    return LUMINA_E_ARG;
  }
  if (gu->rows != a.e_n * 2 * a.Ie || dn->rows != a.e_n * a.Ie || gu->cols != a.d || dn->cols != a.d) {
    set_error("virtual-MoE layer: gate_up (%d, %d) / down (%d, %d) do not match %d local experts, ie %d, d %d",
              gu->rows, gu->cols, dn->rows, dn->cols, a.e_n, a.Ie, a.d);
    return LUMINA_E_ARG;
  }
  if (gu->bits != 4 || dn->bits != 4 || gu->mma || dn->mma || gu->group % 64 || dn->group % 64 ||
      gu->fp16_scales != dn->fp16_scales || a.d % 64) {
    set_error("virtual-MoE experts are built for int4 with groups of 64k in the row-major layout, d %% 64 == 0");
    return LUMINA_E_UNSUPPORTED;
  }
  if (gu_smem_bytes(a.d, MOE_ROWS) > 200 * 1024 || a.d % 4) {
    set_error("virtual-MoE layer: d %d too wide for the shared-memory row stage", a.d);
    return LUMINA_E_UNSUPPORTED;
  }
  return LUMINA_OK;
}

int moe_prepare(int d) {
  const int s1 = (int)gu_smem_bytes(d, 1), s4 = (int)gu_smem_bytes(d, MOE_ROWS);
  LUMINA_CUDA_TRY(cudaFuncSetAttribute(moe_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, d * 8));
  LUMINA_CUDA_TRY(cudaFuncSetAttribute(moe_gu_kernel<__half, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, s1));
  LUMINA_CUDA_TRY(cudaFuncSetAttribute(moe_gu_kernel<float, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, s1));
  LUMINA_CUDA_TRY(
      cudaFuncSetAttribute(moe_gu_kernel<__half, MOE_ROWS>, cudaFuncAttributeMaxDynamicSharedMemorySize, s4));
  LUMINA_CUDA_TRY(
      cudaFuncSetAttribute(moe_gu_kernel<float, MOE_ROWS>, cudaFuncAttributeMaxDynamicSharedMemorySize, s4));
  return LUMINA_OK;
}

namespace {

template <typename ST, int PR>
int launch_experts(const MoeLayerArgs& a, int n, const MoeScratch& sc, float* x, cudaStream_t s) {
  // a pass of PR rows touches at most min(E, PR * K) experts
  // one round of MOE_PPC neuron pairs per CTA for a decode row (several
  // small CTAs per SM); 8 rounds for passes of several rows, so a CTA stages
  // the pass's rows once for 64 pairs
  const int ppw = PR == 1 ? 1 : 8;
  const dim3 ggu(std::min(a.e_n, PR * a.K), (a.Ie + MOE_PPC * ppw - 1) / (MOE_PPC * ppw));
  LUMINA_CUDA_TRY(launch_pdl(moe_gu_kernel<ST, PR>, ggu, dim3(MOE_THREADS), gu_smem_bytes(a.d, PR), s, *a.gate_up,
                             (const float*)sc.h, a.d, n, (const float*)sc.score, a.E, a.K, a.Ie, a.e_lo, a.e_n, ppw,
                             sc.act));
  const dim3 gdn(a.d / 64, moe_splits(n));
  LUMINA_CUDA_TRY(launch_pdl(moe_down_kernel<ST, PR>, gdn, dim3(MOE_THREADS), 0, s, *a.down, a.d, n,
                             (const float*)sc.score, a.E, a.K, a.Ie, a.e_lo, a.e_n, (const float*)sc.act, sc.part,
                             sc.counters, x, a.out));
  return LUMINA_OK;
}

}  // namespace

int launch_moe(const MoeLayerArgs& a, int n, const MoeScratch& sc, float* x, cudaStream_t s) {
  LUMINA_CUDA_TRY(launch_pdl(moe_route_kernel, dim3(n, a.E), dim3(ROUTE_THREADS), (size_t)a.d * 8, s,
                             (const float*)x, a.d, a.norm_w, a.eps, a.router_w, a.router_b, a.E, sc.h, sc.score));
  const bool h16 = a.gate_up->fp16_scales;
  if (n == 1) return h16 ? launch_experts<__half, 1>(a, n, sc, x, s) : launch_experts<float, 1>(a, n, sc, x, s);
  return h16 ? launch_experts<__half, MOE_ROWS>(a, n, sc, x, s) : launch_experts<float, MOE_ROWS>(a, n, sc, x, s);
}

}  // namespace lumina
