// Packed GEMV on the tensor pipe for 5..32 activation rows (decode batches,
// EAGLE tree verification), weights in the fragment layout (weights.cuh).
//
// Arithmetic: the decode GEMV's (gemv_tc.cu). Each activation row is
// quantized per 64-column pair, q = rint(x * 32639 / amax) = 256 qh + ql
// with qh and ql signed bytes, and the code bytes of a 16-row tile are the
// u8 A operand of mma.sync.m16n8k32 unchanged (low nibbles rows 0-7, high
// nibbles rows 8-15 times 16). With NB activation rows the B operand has
// 2 NB columns (qh, ql of each row): NJ = NB / 4 n8 tiles per k32 step.
// Per row, activation row and pair: T = 2 (256 Dh + Dl) - L sum q, y +=
// T * sx * s, y /= L at the end, L = 15 (adapters/lumina.py:135-139: level =
// (2c - L) / L); int3 / int2 / binary codes stored one per nibble take
// their own L = 2^bits - 1.
//
// Why not the tcgen05 projection at these sizes: that kernel dequantizes
// every weight to fp16 in shared memory, about 300 warp instructions per
// 64-column step, so at 31 rows it streams weights at 0.47 TB/s; here the
// codes feed the tensor pipe as they are and the cost per weight does not
// depend on the row count.
//
// Data flow:
//  1. act_frag_kernel: x (RMSNorm fused) -> B fragments in global memory,
//     [pair][2 NB columns][4 lanes] uint4 ({k32 block 0: b0, b1, block 1:
//     b0, b1}), then [pair][NB] (sx, -L sum q), L = 15 for int4 and
//     2^bits - 1 for narrow codes stored one per nibble.
//  2. gemv_tcb_kernel: the grid is S K-slices x CTAs per slice. A CTA
//     bulk-copies its slice of the fragments into shared memory once; each
//     of its 8 warps owns whole 32-row super-tiles over that slice and
//     streams their codes and scales (units of 4 pairs x 2 tiles) through a
//     3-stage ring filled by cp.async.bulk with mbarrier completion (the
//     first stages are requested before griddepcontrol.wait). One B
//     fragment load from shared memory feeds both tiles of the super-tile.
//  3. With S > 1 the S CTAs of a slice set form one thread-block cluster.
//     At the end of a round (one super-tile per warp) each warp leaves its
//     partial in the ring stage of its last unit, the cluster synchronizes,
//     and CTA s adds the partials of every S-th warp's super-tile over
//     distributed shared memory, in slice order (deterministic), and runs
//     the epilogue; a second cluster barrier frees the stages.
#include <cooperative_groups.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "gemv_impl.cuh"

namespace lumina {

namespace {

namespace cg = cooperative_groups;

constexpr int BW = 8;        // warps per CTA
constexpr int BTS = 3;       // ring stages per warp
constexpr int BKS = 4;       // pairs per unit
constexpr int BRT = 2;       // 16-row tiles per super-tile
constexpr int BQMAX = 32639;  // 256 * 127 + 127
constexpr int FRAG_PAIRS = 16;  // pairs per act_frag_kernel CTA

__device__ __forceinline__ void mma_a(int (&d)[4], const uint4& wq, const uint4& bq) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(wq.x & 0x0F0F0F0Fu), "r"(wq.x & 0xF0F0F0F0u), "r"(wq.y & 0x0F0F0F0Fu), "r"(wq.y & 0xF0F0F0F0u),
        "r"(bq.x), "r"(bq.y), "r"(0));
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(wq.z & 0x0F0F0F0Fu), "r"(wq.z & 0xF0F0F0F0u), "r"(wq.w & 0x0F0F0F0Fu), "r"(wq.w & 0xF0F0F0F0u),
        "r"(bq.z), "r"(bq.w));
}

// ---------------------------------------------------------------------------
// 1) activation rows -> B fragments
// ---------------------------------------------------------------------------
struct FragArgs {
  const float* x;
  int ldx;
  int nb;  // live rows (rows nb .. NB-1 get zero fragments)
  int NB;
  int lv;  // levels - 1 of the weight's codes (15 for int4)
  int K, P;
  const float* norm_w;
  float eps;
  uint4* xf;  // [P][2 NB][4]
  int2* fq;   // [P][NB]
};

// grid (NB, ceil(P / FRAG_PAIRS)), 128 threads: thread i quantizes columns
// 8 (i % 8) .. + 7 of pair p0 + i / 8 of row blockIdx.x
__global__ void __launch_bounds__(128) act_frag_kernel(FragArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x, p = blockIdx.y * FRAG_PAIRS + (threadIdx.x >> 3), oc = threadIdx.x & 7;
  const bool live = b < a.nb;
  const float* xr = a.x + (size_t)b * a.ldx;
  float rinv = 1.f;
  if (a.norm_w && live) {
    // chat.py:63-66: x / sqrt(mean(x^2) + eps) * w, the whole row
    __shared__ float red[4];
    // 16-byte loads, four independent sums: the row's loads are in flight
    // together instead of one L2 round trip per element
    float s4[4] = {0.f, 0.f, 0.f, 0.f};
    if ((a.K & 3) == 0 && (a.ldx & 3) == 0 && (reinterpret_cast<uintptr_t>(xr) & 15) == 0) {
      const float4* x4 = reinterpret_cast<const float4*>(xr);
#pragma unroll 4
      for (int k = threadIdx.x; k < (a.K >> 2); k += blockDim.x) {
        const float4 f = x4[k];
        s4[0] = fmaf(f.x, f.x, s4[0]);
        s4[1] = fmaf(f.y, f.y, s4[1]);
        s4[2] = fmaf(f.z, f.z, s4[2]);
        s4[3] = fmaf(f.w, f.w, s4[3]);
      }
    } else {
#pragma unroll 4
      for (int k = threadIdx.x; k < a.K; k += blockDim.x) s4[0] = fmaf(xr[k], xr[k], s4[0]);
    }
    float ss = (s4[0] + s4[1]) + (s4[2] + s4[3]);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    rinv = 1.0f / sqrtf((red[0] + red[1] + red[2] + red[3]) / (float)a.K + a.eps);
  }
  const int k0 = p * 64 + oc * 8;
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int k = k0 + j;
    float t = (live && p < a.P && k < a.K) ? xr[k] : 0.f;
    if (a.norm_w && live && k < a.K) t = (t * rinv) * a.norm_w[k];
    v[j] = t;
  }
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
  uint32_t hw[2] = {0, 0}, lw[2] = {0, 0};
  int qs = 0;
  float sxv = 0.f;
  if (amax > 0.f) {
    const float f = __fdiv_rn((float)BQMAX, amax);
    sxv = __fdiv_rn(amax, (float)BQMAX);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int q = __float2int_rn(__fmul_rn(v[j], f));
      q = max(-BQMAX, min(BQMAX, q));
      qs += q;
      const int qh = (q + 128) >> 8, ql = q - 256 * qh;
      hw[j >> 2] |= ((uint32_t)qh & 0xFFu) << (8 * (j & 3));
      lw[j >> 2] |= ((uint32_t)ql & 0xFFu) << (8 * (j & 3));
    }
  }
  qs += __shfl_xor_sync(0xffffffffu, qs, 1);
  qs += __shfl_xor_sync(0xffffffffu, qs, 2);
  qs += __shfl_xor_sync(0xffffffffu, qs, 4);
  if (p >= a.P) return;
  // columns 8 oc .. 8 oc + 7 of the pair: k32 block oc >> 2, register
  // (oc >> 1) & 1 of lanes t = 2 (oc & 1) and the next, 4 columns each
  const int NC = 2 * a.NB;
  const int comp = ((oc >> 2) << 1) | ((oc >> 1) & 1), tt0 = 2 * (oc & 1);
  uint32_t* xw = reinterpret_cast<uint32_t*>(a.xf + ((size_t)p * NC + 2 * b) * 4);
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    xw[(tt0 + e) * 4 + comp] = hw[e];
    xw[16 + (tt0 + e) * 4 + comp] = lw[e];
  }
  if (oc == 0) a.fq[(size_t)p * a.NB + b] = make_int2(__float_as_int(sxv), -a.lv * qs);
}

// ---------------------------------------------------------------------------
// 2) the GEMV
// ---------------------------------------------------------------------------
struct TcbArgs {
  const uint8_t* codes;
  const uint8_t* scales;
  int rows;
  int P;      // 64-column pairs per row
  int ng;     // scale groups per row
  int gsh;    // log2(group / 64)
  int T16;    // 16-row tiles (even: rows are padded to 32)
  int n_st;   // 32-row super-tiles
  const uint4* xf;
  const int2* fq;
  int nb;     // live activation rows
  float lvf;  // levels - 1 of the codes: 15 (int4), 7, 3, 1 (narrow codes one per nibble)
  float* y;
  int ldy;
  const float* resid;
  int ldr;
  int epi;      // EPI_STORE, EPI_RESID, EPI_SWIGLU, EPI_ROPE_KV
  RopeKV rk;    // EPI_ROPE_KV: RoPE + paged KV append of the fused q/k/v rows
  int qk_rows;  // EPI_STORE: rows < qk_rows of a fused q/k/v weight go to their un-permuted index
  int hd;
  int S;        // K slices = the cluster size (the S CTAs of a cluster share their super-tiles)
  int ps;       // pairs per slice (a multiple of BKS; the last slice may be shorter)
  int cps;      // CTAs per slice
  int ipw;      // super-tiles per warp
  int stage_bytes;
  int x_bytes;  // shared bytes of the fragment slice (128-byte multiple)
  int gmax;     // scale groups one unit spans at most
  int* fault;
  long long spin;
};

// RoPE pair permutation of the fused q/k/v weight: row 2p + e of a head is
// the original row p + e * hd / 2
__device__ __forceinline__ int tcb_out_row(const TcbArgs& a, int row) {
  if (row >= a.qk_rows) return row;
  const int h = row / a.hd, rr = row - h * a.hd;
  return h * a.hd + (rr >> 1) + (rr & 1) * (a.hd >> 1);
}

// RoPE + paged KV append of the fused q/k/v rows (row, row + 1) = (x1, x2)
// of activation row b: q and k rows hold rotation pairs side by side, so the
// pair rotates by the row's position (chat.py:99-100, fp32 products rounded
// separately) into q_out or the K cache; v rows go to the V cache.
__device__ __forceinline__ void tcb_rope_store(const TcbArgs& a, int row, int b, float x1, float x2) {
  const RopeKV& k = a.rk;
  const int qrows = k.nh * k.hd, krows = k.nkv * k.hd, half = k.hd / 2;
  const int tt = *k.t_prev + k.row_base + b;
  const size_t blk = k.block_table[tt / k.bs], off = tt % k.bs;
  if (row < qrows + krows) {
    const bool isq = row < qrows;
    const int rr = isq ? row : row - qrows;
    const int hh = rr / k.hd, p = (rr % k.hd) >> 1;
    const size_t ci = (size_t)k.row_pos[b] * half + p;
    const float c = k.cos_t[ci], s = k.sin_t[ci];
    const float o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    const float o2 = __fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c));
    if (isq) {
      float* q = k.q_out + (size_t)b * qrows + (size_t)hh * k.hd;
      q[p] = o1;
      q[p + half] = o2;
    } else {
      const size_t base = ((blk * k.nkv + hh) * k.bs + off) * k.hd;
      if (k.kv_fp16) {
        __half* kc = static_cast<__half*>(k.kcache) + base;
        kc[p] = __float2half_rn(o1);
        kc[p + half] = __float2half_rn(o2);
      } else {
        float* kc = static_cast<float*>(k.kcache) + base;
        kc[p] = o1;
        kc[p + half] = o2;
      }
    }
  } else {
    const float vv[2] = {x1, x2};
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int rr = row + e - qrows - krows;
      const size_t idx = ((blk * k.nkv + rr / k.hd) * k.bs + off) * k.hd + rr % k.hd;
      if (k.kv_fp16) static_cast<__half*>(k.vcache)[idx] = __float2half_rn(vv[e]);
      else static_cast<float*>(k.vcache)[idx] = vv[e];
    }
  }
}

// Epilogue of one finished value pair of this lane: rows r0 (+0, +8) of
// activation row b; v[0] = row r0 + g, v[1] = row r0 + g + 8 (already / L).
// SwiGLU and RoPE pair rows 2i, 2i+1: the odd row lives in the lane 4 above.
__device__ __forceinline__ void tcb_emit(const TcbArgs& a, int r0, int b, float v0, float v1, int lane) {
  const int g = lane >> 2;
  if (a.epi == EPI_ROPE_KV) {
    const float n0 = __shfl_down_sync(0xffffffffu, v0, 4), n1 = __shfl_down_sync(0xffffffffu, v1, 4);
    if (b >= a.nb || (g & 1)) return;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = r0 + g + 8 * h;
      if (row + 1 < a.rows) tcb_rope_store(a, row, b, h ? v1 : v0, h ? n1 : n0);
    }
    return;
  }
  if (a.epi == EPI_SWIGLU) {
    const float n0 = __shfl_down_sync(0xffffffffu, v0, 4), n1 = __shfl_down_sync(0xffffffffu, v1, 4);
    if (b >= a.nb || (g & 1)) return;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = r0 + g + 8 * h;
      if (row + 1 >= a.rows) continue;
      const float gt = h ? v1 : v0, up = h ? n1 : n0;
      const float e = expf(-fminf(fmaxf(gt, -40.f), 40.f));  // chat.py:300-302, the +-40 clip
      a.y[(size_t)b * a.ldy + (row >> 1)] = gt / (1.0f + e) * up;
    }
    return;
  }
  if (b >= a.nb) return;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = r0 + g + 8 * h;
    if (row >= a.rows) continue;
    float v = h ? v1 : v0;
    if (a.epi == EPI_RESID) v += a.resid[(size_t)b * a.ldr + row];
    a.y[(size_t)b * a.ldy + tcb_out_row(a, row)] = v;
  }
}

template <int NJ, typename ST>
__global__ void __launch_bounds__(BW * 32, 1) gemv_tcb_kernel(TcbArgs a) {
  constexpr int NB = 4 * NJ;
  constexpr int NC = 2 * NB;
  constexpr int ES = sizeof(ST);
  constexpr int SG = 16 * ES;   // scale bytes of one group of a tile
  constexpr int PLD = NB + 4;   // row stride of a partial super-tile in shared memory (floats)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;

  // this CTA's slice (its rank in the cluster of the S slices), this warp's
  // super-tiles
  const int s = (int)(blockIdx.x % a.S), ci = (int)(blockIdx.x / a.S);
  auto slice_chunks = [&](int q) {
    const int lo = q * a.ps, hi = min(a.P, lo + a.ps);
    return (hi - lo + BKS - 1) / BKS;
  };
  const int p_lo = s * a.ps, p_hi = min(a.P, p_lo + a.ps), nps = p_hi - p_lo;
  const int nchunk = slice_chunks(s);
  const int st0 = (ci * BW + warp) * a.ipw, st1 = min(a.n_st, st0 + a.ipw);
  const int n_items = max(0, st1 - st0), n_mine = n_items * nchunk;

  extern __shared__ __align__(128) uint8_t smem[];
  // [B fragments: nps x NC x 4 x 16 B][(sx, -L sum q): nps x NB x 8 B]
  // [rings: BW x BTS x stage_bytes][mbarriers: BW x BTS, then the slice's]
  uint4* xs = reinterpret_cast<uint4*>(smem);
  const int2* fqs = reinterpret_cast<const int2*>(smem + (size_t)a.ps * NC * 64);
  uint8_t* rings = smem + a.x_bytes;
  uint8_t* ring = rings + (size_t)warp * BTS * a.stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(rings + (size_t)BW * BTS * a.stage_bytes);
  uint64_t* xbar = bars + BW * BTS;
  bars += warp * BTS;

  // lane 0: unit j (super-tile st0 + j / nchunk, chunk j % nchunk) into
  // stage j % BTS: the codes and the scales of both tiles
  const uint64_t pol = l2_evict_first_policy();
  int n_issued = 0;  // lane 0: units requested so far (in order)
  auto issue = [&](int j) {
    const int st = st0 + j / nchunk, c = j - (j / nchunk) * nchunk;
    const int p0 = p_lo + c * BKS, np = min(BKS, p_hi - p0);
    const int G0 = p0 >> a.gsh, G1 = ((p0 + np - 1) >> a.gsh) + 1;
    uint8_t* stg = ring + (size_t)(j % BTS) * a.stage_bytes;
    const uint32_t cb = (uint32_t)np * 512u, sb = (uint32_t)(G1 - G0) * SG;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_expect_tx(&bars[j % BTS], BRT * (cb + sb));
#pragma unroll
    for (int r = 0; r < BRT; ++r) {
      const int tile = st * BRT + r;
      bulk_g2s_hint(stg + r * BKS * 512, a.codes + ((size_t)tile * a.P + p0) * 512, cb, &bars[j % BTS], pol);
      bulk_g2s_hint(stg + BRT * BKS * 512 + r * a.gmax * SG, a.scales + ((size_t)tile * a.ng + G0) * SG, sb,
                    &bars[j % BTS], pol);
    }
    n_issued = j + 1;
  };

  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < BTS; ++i) mbar_init(&bars[i], 1);
    if (warp == 0) mbar_init(xbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // weights never depend on the previous kernel: the first stages go out
  // before the dependency wait
  if (lane == 0)
    for (int j = 0; j < min(BTS, n_mine); ++j) issue(j);
  pdl_launch_dependents();
  pdl_wait();
  // the slice's activation fragments (written by act_frag_kernel)
  if (threadIdx.x == 0) {
    const uint32_t xb = (uint32_t)nps * NC * 64, fb = (uint32_t)nps * NB * 8;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_expect_tx(xbar, xb + fb);
    bulk_g2s(xs, a.xf + (size_t)p_lo * NC * 4, xb, xbar);
    bulk_g2s(smem + (size_t)a.ps * NC * 64, a.fq + (size_t)p_lo * NB, fb, xbar);
  }
  bool bad = !__all_sync(0xffffffffu, mbar_wait_bounded(xbar, 0, a.spin));

  float acc[BRT][NJ][2];
#pragma unroll
  for (int r = 0; r < BRT; ++r)
#pragma unroll
    for (int jj = 0; jj < NJ; ++jj) acc[r][jj][0] = acc[r][jj][1] = 0.f;
  int waited = 0;  // units whose stage has landed
  // Every warp runs ipw rounds, one super-tile each: with S > 1 a round
  // ends with two cluster barriers (collective), so a warp without an item
  // in a round still takes part in them.
  for (int k = 0; k < a.ipw; ++k) {
    const bool have = k < n_items;
    const int j_last = k * nchunk + nchunk - 1;
    for (int c = 0; have && c < nchunk; ++c) {
      const int j = k * nchunk + c;
      if (!bad) {
        if (__all_sync(0xffffffffu, mbar_wait_bounded(&bars[j % BTS], (uint32_t)((j / BTS) & 1), a.spin)))
          ++waited;
        else
          bad = true;
      }
      if (bad) continue;
      const int p0 = p_lo + c * BKS, np = min(BKS, p_hi - p0);
      const int G0 = p0 >> a.gsh;
      const uint8_t* stg = ring + (size_t)(j % BTS) * a.stage_bytes;
      auto pair = [&](int i) {
        const int pl = p0 + i - p_lo;  // pair within the slice
        uint4 bq[NJ];
        int2 fv[NJ];
#pragma unroll
        for (int jj = 0; jj < NJ; ++jj) {
          bq[jj] = xs[((size_t)pl * NC + 8 * jj + g) * 4 + t];
          fv[jj] = fqs[(size_t)pl * NB + 4 * jj + t];
        }
        const int gi = ((p0 + i) >> a.gsh) - G0;
#pragma unroll
        for (int r = 0; r < BRT; ++r) {
          const uint4 wq = reinterpret_cast<const uint4*>(stg + r * BKS * 512 + i * 512)[lane];
          float s0, s1;
          const uint8_t* sp = stg + BRT * BKS * 512 + r * a.gmax * SG + gi * SG + g * 2 * ES;
          if constexpr (ES == 2) {
            const __half2 hh = *reinterpret_cast<const __half2*>(sp);
            s0 = __low2float(hh);
            s1 = __high2float(hh);
          } else {
            const float2 ff = *reinterpret_cast<const float2*>(sp);
            s0 = ff.x;
            s1 = ff.y;
          }
          s1 *= 0.0625f;  // rows g + 8 carry codes * 16
#pragma unroll
          for (int jj = 0; jj < NJ; ++jj) {
            int cc[4];
            mma_a(cc, wq, bq[jj]);
            const float fx = __int_as_float(fv[jj].x);
            const int T0 = cc[0] * 512 + cc[1] * 2 + fv[jj].y;
            const int T1 = cc[2] * 512 + cc[3] * 2 + fv[jj].y * 16;
            acc[r][jj][0] = fmaf((float)T0, fx * s0, acc[r][jj][0]);
            acc[r][jj][1] = fmaf((float)T1, fx * s1, acc[r][jj][1]);
          }
        }
      };
      if (np == BKS) {
#pragma unroll
        for (int i = 0; i < BKS; ++i) pair(i);
      } else {
        for (int i = 0; i < np; ++i) pair(i);
      }
      __syncwarp();  // every lane is done with stage j % BTS
      // with S > 1 the stage of the item's last unit holds its partial
      // until the round's combine is over: its refill waits for that
      if (lane == 0 && j + BTS < n_mine && (a.S == 1 || j != j_last)) issue(j + BTS);
    }

    if (a.S == 1) {
      if (have) {
#pragma unroll
        for (int r = 0; r < BRT; ++r)
#pragma unroll
          for (int jj = 0; jj < NJ; ++jj)
            tcb_emit(a, ((st0 + k) * BRT + r) * 16, 4 * jj + t, acc[r][jj][0] / a.lvf, acc[r][jj][1] / a.lvf,
                     lane);
      }
    } else {
      // the partial super-tile -> the stage of the item's last unit
      if (have) {
        float* pst = reinterpret_cast<float*>(ring + (size_t)(j_last % BTS) * a.stage_bytes);
#pragma unroll
        for (int r = 0; r < BRT; ++r)
#pragma unroll
          for (int jj = 0; jj < NJ; ++jj)
#pragma unroll
            for (int h = 0; h < 2; ++h) pst[(r * 16 + g + 8 * h) * PLD + 4 * jj + t] = acc[r][jj][h];
      }
      cg::cluster_group cluster = cg::this_cluster();
      cluster.sync();  // every slice's partials of this round are in place
      // CTA s combines the super-tiles of warps s, s + S, ...: the S
      // partials in slice order (deterministic), then the epilogue; a
      // thread takes rows 2i, 2i+1 of one activation row
      const int nw = (BW - s + a.S - 1) / a.S;
      for (int e = threadIdx.x; e < nw * 16 * NB; e += blockDim.x) {
        const int wl = e / (16 * NB), rem = e - wl * 16 * NB, b = rem >> 4, i = rem & 15;
        const int w = s + wl * a.S, st = (ci * BW + w) * a.ipw + k;
        if (st >= a.n_st || b >= a.nb) continue;
        float v0 = 0.f, v1 = 0.f;
#pragma unroll 8
        for (int q = 0; q < a.S; ++q) {
          const int sq = ((k + 1) * slice_chunks(q) - 1) % BTS;
          const float* src = reinterpret_cast<const float*>(rings + ((size_t)w * BTS + sq) * a.stage_bytes);
          const float* rp = cluster.map_shared_rank(src, q) + (2 * i) * PLD + b;
          v0 += rp[0];
          v1 += rp[PLD];
        }
        const int row = st * 32 + 2 * i;
        v0 /= a.lvf;
        v1 /= a.lvf;
        if (a.epi == EPI_SWIGLU) {
          if (row + 1 < a.rows) {
            const float e2 = expf(-fminf(fmaxf(v0, -40.f), 40.f));  // chat.py:300-302, the +-40 clip
            a.y[(size_t)b * a.ldy + (row >> 1)] = v0 / (1.0f + e2) * v1;
          }
        } else if (a.epi == EPI_ROPE_KV) {
          if (row + 1 < a.rows) tcb_rope_store(a, row, b, v0, v1);
        } else {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int rr = row + h;
            if (rr >= a.rows) continue;
            float v = h ? v1 : v0;
            if (a.epi == EPI_RESID) v += a.resid[(size_t)b * a.ldr + rr];
            a.y[(size_t)b * a.ldy + tcb_out_row(a, rr)] = v;
          }
        }
      }
      cluster.sync();  // every CTA is done reading this round's partials
      if (have && !bad && lane == 0 && j_last + BTS < n_mine) issue(j_last + BTS);
    }
#pragma unroll
    for (int r = 0; r < BRT; ++r)
#pragma unroll
      for (int jj = 0; jj < NJ; ++jj) acc[r][jj][0] = acc[r][jj][1] = 0.f;
  }
  if (bad) {
    // record it, and let the copies still in flight land before the CTA's
    // shared memory is released (unit j completes phase j / BTS of stage
    // j % BTS; these waits take the full limit)
    if (lane == 0) {
      atomicOr(a.fault, 16);
      for (int j = waited; j < n_issued; ++j) mbar_wait_bounded(&bars[j % BTS], (uint32_t)((j / BTS) & 1));
      if (warp == 0) mbar_wait_bounded(xbar, 0);
    }
    __syncwarp();
  }
}

template <int NJ, typename ST>
int launch_tcb(const TcbArgs& a, size_t smem, int grid, cudaStream_t s) {
  auto kern = gemv_tcb_kernel<NJ, ST>;
  int rc = set_smem_limit((const void*)kern, smem, "gemv_tcb");
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(BW * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = a.S;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  {
    // a cluster of S CTAs of this size must fit the GPU (checked once per
    // device and configuration)
    static std::mutex mu;
    static std::map<std::tuple<const void*, int, int, size_t>, int> fits;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    auto key = std::make_tuple((const void*)kern, dev, a.S, smem);
    auto it = fits.find(key);
    if (it == fits.end()) {
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
      }
      it = fits.emplace(key, n).first;
    }
    if (it->second < 1) return LUMINA_E_UNSUPPORTED;
  }
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) {
    set_error("gemv_tcb launch: %s", cudaGetErrorString(e));
    return LUMINA_E_CUDA;
  }
  return LUMINA_OK;
}

template <int NJ>
int tcb_st(const TcbArgs& a, bool fp16, size_t smem, int grid, cudaStream_t s) {
  return fp16 ? launch_tcb<NJ, __half>(a, smem, grid, s) : launch_tcb<NJ, float>(a, smem, grid, s);
}

size_t round128(size_t v) { return (v + 127) / 128 * 128; }

}  // namespace

static int tcb_nb(int M) { return M <= 8 ? 8 : M <= 16 ? 16 : 32; }

size_t gemv_tcb_frag_bytes(int M, int cols) {
  const size_t P = (size_t)(cols + 63) / 64;
  return P * tcb_nb(M) * 136;
}

int gemv_tcb_launch(const lumina_weight* w, const float* x, int ldx, int M, const float* norm_w, float eps,
                    void* frag, size_t frag_bytes, float* y, int ldy, int epi, const float* resid, int ldr,
                    int qk_rows, int hd, cudaStream_t s, const RopeKV* rk) {
  if (!w->mma || (w->group % 64) || M < 1 || M > 32) return LUMINA_E_UNSUPPORTED;
  const int gp = w->group / 64;
  if ((gp & (gp - 1)) || gp > 4) return LUMINA_E_UNSUPPORTED;
  if (epi != EPI_STORE && epi != EPI_RESID && epi != EPI_SWIGLU && (epi != EPI_ROPE_KV || !rk))
    return LUMINA_E_UNSUPPORTED;
  if ((epi == EPI_SWIGLU || epi == EPI_ROPE_KV) && (w->rows & 1)) {
    set_error("gemv_tcb: a paired epilogue needs an even row count");
    return LUMINA_E_ARG;
  }
  const int NB = tcb_nb(M), P = w->n_chunks / 2;
  if (!frag || frag_bytes < (size_t)P * NB * 136 || (reinterpret_cast<uintptr_t>(frag) & 15))
    return LUMINA_E_UNSUPPORTED;
  int* fault = fault_flag_ptr();
  if (!fault) {
    set_error("gemv_tcb: fault flag unavailable");
    return LUMINA_E_CUDA;
  }
  TcbArgs a{};
  a.codes = w->codes;
  a.scales = w->scales;
  a.rows = w->rows;
  a.P = P;
  a.ng = w->n_groups;
  a.gsh = gp == 1 ? 0 : gp == 2 ? 1 : 2;
  a.T16 = w->rows_pad / 16;
  a.n_st = a.T16 / BRT;
  a.xf = static_cast<const uint4*>(frag);
  a.fq = reinterpret_cast<const int2*>(static_cast<const uint8_t*>(frag) + (size_t)P * NB * 128);
  a.nb = M;
  a.lvf = (float)((1 << w->bits) - 1);
  a.y = y;
  a.ldy = ldy;
  a.resid = resid;
  a.ldr = ldr;
  a.epi = epi;
  a.qk_rows = epi == EPI_STORE ? qk_rows : 0;
  if (rk) a.rk = *rk;
  a.hd = hd > 0 ? hd : 1;
  a.fault = fault;
  a.spin = wait_spin_limit();
  const int es = w->fp16_scales ? 2 : 4;
  a.gmax = std::max(1, BKS >> a.gsh);
  // a stage also holds a warp's partial super-tile (32 rows x (NB + 4) floats)
  a.stage_bytes = (int)std::max(round128((size_t)BRT * BKS * 512 + (size_t)BRT * a.gmax * 16 * es),
                                round128((size_t)32 * (NB + 4) * 4));
  const size_t ring_bytes = (size_t)BW * BTS * a.stage_bytes, bar_bytes = (size_t)(BW * BTS + 1) * 8;
  const size_t budget = 227 * 1024 - 1024;
  const size_t per_pair = (size_t)NB * 136;
  const long pmax = ((long)budget - (long)ring_bytes - (long)bar_bytes - 128) / (long)per_pair / BKS * BKS;
  if (pmax < BKS) return LUMINA_E_UNSUPPORTED;
  // K slices: the largest slice (fewest partials) whose grid fills at
  // least 80% of the SMs with busy warps, else the best-filled one; a slice
  // needs its fragments in shared memory, and the S slices form one
  // cluster (at most 8 CTAs)
  const int sms = sm_count();
  const long warps = (long)sms * BW;
  int best_ps = 0, best_S = 0, best_ipw = 0, best_cps = 0;
  double best_fill = -1.0;
  const int ps_start = (int)std::min<long>(pmax, (P + BKS - 1) / BKS * BKS);
  for (int ps = ps_start; ps >= BKS; ps -= BKS) {
    const int S = (P + ps - 1) / ps;
    if (S > 8) break;
    const long items = (long)a.n_st * S;
    int ipw = (int)std::max(1L, (items + warps - 1) / warps), cps = 0;
    for (;; ++ipw) {
      cps = (a.n_st + BW * ipw - 1) / (BW * ipw);
      if ((long)S * cps <= sms || cps == 1) break;
    }
    const double fill = (double)items / ((double)ipw * S * cps * BW) * std::min(1.0, (double)S * cps / sms);
    if (fill > best_fill) {
      best_fill = fill;
      best_ps = ps;
      best_S = S;
      best_ipw = ipw;
      best_cps = cps;
    }
    if (fill >= 0.8) break;
  }
  if (best_ps == 0) return LUMINA_E_UNSUPPORTED;
  const int S = best_S, ps = best_ps;
  a.S = S;
  a.ps = ps;
  a.ipw = best_ipw;
  a.cps = best_cps;
  a.x_bytes = (int)round128((size_t)ps * per_pair);
  const size_t smem = (size_t)a.x_bytes + ring_bytes + bar_bytes;
  if (smem > budget) return LUMINA_E_UNSUPPORTED;

  // 1) the fragments
  FragArgs f{};
  f.x = x;
  f.ldx = ldx;
  f.nb = M;
  f.NB = NB;
  f.lv = (1 << w->bits) - 1;
  f.K = w->cols;
  f.P = P;
  f.norm_w = norm_w;
  f.eps = eps;
  f.xf = static_cast<uint4*>(frag);
  f.fq = reinterpret_cast<int2*>(static_cast<uint8_t*>(frag) + (size_t)P * NB * 128);
  cudaError_t e = launch_pdl(act_frag_kernel, dim3(NB, (P + FRAG_PAIRS - 1) / FRAG_PAIRS), dim3(128), 0, s, f);
  if (e != cudaSuccess) {
    set_error("act_frag launch: %s", cudaGetErrorString(e));
    return LUMINA_E_CUDA;
  }
  // 2) the GEMV
  const int grid = S * a.cps;
  switch (NB) {
    case 8: return tcb_st<2>(a, w->fp16_scales, smem, grid, s);
    case 16: return tcb_st<4>(a, w->fp16_scales, smem, grid, s);
    default: return tcb_st<8>(a, w->fp16_scales, smem, grid, s);
  }
}

// per-device activation-fragment scratch for the library's own entry points
int tcb_frag_scratch(int device, size_t bytes, void** out) {
  static std::mutex mu;
  static void* buf[64] = {};
  static size_t cap[64] = {};
  if (device < 0 || device >= 64) {
    set_error("gemv_tcb: bad device %d", device);
    return LUMINA_E_ARG;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (cap[device] < bytes) {
    if (buf[device]) {
      cudaDeviceSynchronize();  // queued work may still read the smaller buffer
      cudaFree(buf[device]);
      buf[device] = nullptr;
      cap[device] = 0;
    }
    const size_t want = std::max(bytes, (size_t)1 << 20);
    if (cudaMalloc(&buf[device], want) != cudaSuccess) {
      cudaGetLastError();
      set_error("gemv_tcb: cudaMalloc of %zu bytes failed", want);
      return LUMINA_E_OOM;
    }
    cap[device] = want;
  }
  *out = buf[device];
  return LUMINA_OK;
}

}  // namespace lumina
