// int4 dequant GEMV with the integer dot products on the tensor pipe.
//
// Same arithmetic as the CUDA-core path (gemv_impl.cuh): activations are
// quantized to int16 per 32-column block, D = sum q_k c_k is computed exactly
// per block, and y = sum_blocks (2D - 15 sum q) * sx * scale / 15. Here the
// per-block dot runs as two mma.sync.m16n8k32 int8 products: the int16
// activation q splits exactly into q = 256 * qh + ql (qh signed byte, ql
// unsigned byte), so D = 256 * (codes . qh) + (codes . ql) with codes as
// unsigned bytes (0..15) in the A operand and the activation bytes in B.
// The CUDA-core dp2a path issues ~1.3 instructions per weight and measured
// issue-bound; this path issues ~0.05.
//
// Weight layout (int4, group size a multiple of 64), rows padded to 32:
//   codes  [tile of 16 rows][pair of 32-column blocks][lane][16 bytes]
//          lane (g = lane/4, t = lane%4), block b of the pair, word w in {0,1}:
//          byte i = code(row g, col 32b + 16w + 4t + i)
//                 | code(row g + 8, same col) << 4
//          so `& 0x0F0F0F0F` and `>> 4 & 0x0F0F0F0F` are the A fragment
//          registers of rows g and g + 8 (mma.m16n8k32 .u8 A layout).
//   scales [tile][group][g in 0..7][2]: (row g, row g + 8) side by side.
// A CTA of 16 warps owns a group of 32 rows (two tiles) and splits K across
// 8 warps per tile; partial sums meet in shared memory in a fixed order
// (deterministic) and one thread per output applies the epilogue.
#include "gemv_impl.cuh"

namespace lumina {

constexpr int MW = 16;        // warps per CTA
constexpr int MT = 2;         // 16-row tiles per row group (32 rows)
constexpr int MKS = MW / MT;  // K slices per tile
constexpr int MU = 8;         // block pairs per pipeline step (per lane 8 x 16 bytes)

struct MmaArgs {
  const uint8_t* codes;
  const uint8_t* scales;
  int rows, cols, np, ng, group, fp16;
  const float* x;
  int ldx;
  const float* norm_w;
  float eps;
  float* y;
  int ldy;
  const float* resid;
  int ldr;
  RopeKV rk;
  int nb;    // live batch rows of this launch (<= NB)
  int n_rg;  // 32-row groups
};

__device__ __forceinline__ void mma_u8s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  d[0] = d[1] = d[2] = d[3] = 0;
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_u8u8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  d[0] = d[1] = d[2] = d[3] = 0;
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename ST>
struct ScalePair;
template <>
struct ScalePair<__half> {
  using T = uint32_t;  // half2 (row g, row g + 8)
  __device__ static T load(const uint8_t* p) { return __ldg(reinterpret_cast<const unsigned*>(p)); }
  __device__ static float lo(T v) { return __low2float(*reinterpret_cast<const __half2*>(&v)); }
  __device__ static float hi(T v) { return __high2float(*reinterpret_cast<const __half2*>(&v)); }
};
template <>
struct ScalePair<float> {
  using T = float2;
  __device__ static T load(const uint8_t* p) { return __ldg(reinterpret_cast<const float2*>(p)); }
  __device__ static float lo(T v) { return v.x; }
  __device__ static float hi(T v) { return v.y; }
};

template <int NB, typename ST>
struct MmaStep {
  uint4 c[MU];
  typename ScalePair<ST>::T s[MU];
};

template <int NB, typename ST, int EPI, bool NORM>
__global__ void __launch_bounds__(MW * 32, 1)
gemv_mma_kernel(MmaArgs a) {
  using SP = ScalePair<ST>;
  constexpr int ES = sizeof(ST);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int tl = warp / MKS, ks = warp % MKS;
  const int np = a.np, nbp = 2 * np;
  const int p0 = ks * np / MKS, p1 = (ks + 1) * np / MKS;
  const int nsteps = max(1, (p1 - p0 + MU - 1) / MU);

  extern __shared__ __align__(128) uint8_t smem[];
  uint4* xb = reinterpret_cast<uint4*>(smem);                      // [nbp][NB][4 t]
  float* sxs = reinterpret_cast<float*>(xb + (size_t)nbp * NB * 4);  // [nbp][NB]
  int* xss = reinterpret_cast<int*>(sxs + (size_t)nbp * NB);        // [nbp][NB]
  float* red = reinterpret_cast<float*>(xss + (size_t)nbp * NB);    // [MT][MKS][16][NB]
  __shared__ float ssum[MW];
  __shared__ int ep_blk[NB], ep_off[NB], ep_pos[NB];

  // step i of this warp across row groups: (rg = blockIdx.x + (i / nsteps) *
  // gridDim.x, st = i % nsteps)
  auto load = [&](int i, MmaStep<NB, ST>& b) {
    const int rg = blockIdx.x + (i / nsteps) * gridDim.x, st = i % nsteps;
    const int T = rg * MT + tl;
#pragma unroll
    for (int u = 0; u < MU; ++u) {
      const int p = p0 + st * MU + u;
      const bool v = p < p1 && rg < a.n_rg;
      const int pc = v ? p : p0;
      const int G = (pc * 64) / a.group;
      b.c[u] = v ? ldg_stream(a.codes + (((size_t)T * np + pc) * 32 + lane) * 16) : make_uint4(0, 0, 0, 0);
      if (v) b.s[u] = SP::load(a.scales + (((size_t)T * a.ng + G) * 8 + g) * 2 * ES);
    }
  };

  // 1) the first step's codes and scales go out before the wait on the
  //    previous kernel (weights never depend on it)
  const int my_rg = blockIdx.x < a.n_rg ? (a.n_rg - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  const int total = my_rg * nsteps;
  MmaStep<NB, ST> A, B;
  if (total > 0) load(0, A);
  pdl_launch_dependents();
  pdl_wait();

  // 2) activations -> int16 per 32-column block -> B fragments in shared
  //    memory; two threads per block (16 columns each)
  if constexpr (EPI == EPI_ROPE_KV) {
    if (threadIdx.x < NB && threadIdx.x < a.nb) {
      const int tt = *a.rk.t_prev + a.rk.row_base + threadIdx.x;
      ep_blk[threadIdx.x] = a.rk.block_table[tt / a.rk.bs];
      ep_off[threadIdx.x] = tt % a.rk.bs;
      ep_pos[threadIdx.x] = a.rk.row_pos[threadIdx.x];
    }
  }
  const bool vec_ok = ((a.ldx & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0);
  const int half = threadIdx.x & 1;
  for (int bb = 0; bb < NB; ++bb) {
    const bool live = bb < a.nb;
    const float* xr = a.x + (size_t)bb * a.ldx;
    for (int blk0 = 0; blk0 < nbp; blk0 += blockDim.x / 2) {
      const int blk = blk0 + (threadIdx.x >> 1);
      const bool mine = blk < nbp;
      const int k0 = blk * 32 + 16 * half;
      float v[16], wn[16];
      if (live && mine && vec_ok && k0 + 16 <= a.cols) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 f = *reinterpret_cast<const float4*>(xr + k0 + 4 * q);
          v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
          if constexpr (NORM) {
            const float4 u = __ldg(reinterpret_cast<const float4*>(a.norm_w + k0 + 4 * q));
            wn[4 * q] = u.x; wn[4 * q + 1] = u.y; wn[4 * q + 2] = u.z; wn[4 * q + 3] = u.w;
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const bool in = live && mine && k0 + j < a.cols;
          v[j] = in ? xr[k0 + j] : 0.f;
          if constexpr (NORM) wn[j] = in ? a.norm_w[k0 + j] : 0.f;
        }
      }
      float rinv = 1.f;
      if constexpr (NORM) {
        // chat.py:63-66: x / sqrt(mean(x^2) + eps) * w (fp32); the whole row
        // is in this pass (dispatch requires nbp <= blockDim.x / 2)
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) ss = fmaf(v[j], v[j], ss);
        ss = warp_sum(ss);
        if (lane == 0) ssum[warp] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int i = 0; i < MW; ++i) tot += ssum[i];
        rinv = 1.0f / sqrtf(tot / (float)a.cols + a.eps);
        __syncthreads();
      }
      float amax = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if constexpr (NORM) v[j] = (v[j] * rinv) * wn[j];
        amax = fmaxf(amax, fabsf(v[j]));
      }
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      uint32_t hw[4] = {0, 0, 0, 0}, lw[4] = {0, 0, 0, 0};  // per t: 4 bytes of qh / ql
      int qs = 0;
      float sxv = 0.f;
      if (amax > 0.f) {
        const float f = __fdiv_rn(32767.f, amax);
        sxv = __fdiv_rn(amax, 32767.f);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          int q = __float2int_rn(__fmul_rn(v[j], f));
          q = max(-32767, min(32767, q));
          qs += q;
          hw[j >> 2] |= ((uint32_t)(q >> 8) & 0xFFu) << (8 * (j & 3));
          lw[j >> 2] |= ((uint32_t)q & 0xFFu) << (8 * (j & 3));
        }
      }
      qs += __shfl_xor_sync(0xffffffffu, qs, 1);
      if (!mine) continue;
      // columns 16*half + 4t .. +3 of the block feed lane t's b{half}
      uint32_t* xw = reinterpret_cast<uint32_t*>(xb + ((size_t)blk * NB + bb) * 4);
#pragma unroll
      for (int tt = 0; tt < 4; ++tt) {
        xw[tt * 4 + half] = hw[tt];      // {qh b0, qh b1, ql b0, ql b1}
        xw[tt * 4 + 2 + half] = lw[tt];
      }
      if (half == 0) {
        sxs[(size_t)blk * NB + bb] = sxv;
        xss[(size_t)blk * NB + bb] = 15 * qs;
      }
    }
  }
  __syncthreads();

  // 3) pipelined sweep over (row group, step); partial sums meet per group
  float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};  // rows (g, g+8) x cols (2t, 2t+1)
  auto compute = [&](const MmaStep<NB, ST>& b, int st) {
#pragma unroll
    for (int u = 0; u < MU; ++u) {
      const int p = p0 + st * MU + u;
      if (p >= p1) continue;  // warp-uniform
      const uint32_t w[4] = {b.c[u].x, b.c[u].y, b.c[u].z, b.c[u].w};
      const float s0 = SP::lo(b.s[u]), s1 = SP::hi(b.s[u]);
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        const int blk = 2 * p + hb;
        const uint32_t af[4] = {w[2 * hb] & 0x0F0F0F0Fu, (w[2 * hb] >> 4) & 0x0F0F0F0Fu,
                                w[2 * hb + 1] & 0x0F0F0F0Fu, (w[2 * hb + 1] >> 4) & 0x0F0F0F0Fu};
        uint4 bq = make_uint4(0, 0, 0, 0);
        if (g < NB) bq = xb[((size_t)blk * NB + g) * 4 + t];
        int dh[4], dl[4];
        mma_u8s8(dh, af, bq.x, bq.y);
        mma_u8u8(dl, af, bq.z, bq.w);
#pragma unroll
        for (int ci = 0; ci < 2; ++ci) {
          const int col = 2 * t + ci;
          if (col < NB) {
            const int xs = xss[(size_t)blk * NB + col];
            const float fx = sxs[(size_t)blk * NB + col];
            const int D0 = 256 * dh[ci] + dl[ci], D1 = 256 * dh[2 + ci] + dl[2 + ci];
            acc[0][ci] = fmaf((float)(2 * D0 - xs), fx * s0, acc[0][ci]);
            acc[1][ci] = fmaf((float)(2 * D1 - xs), fx * s1, acc[1][ci]);
          }
        }
      }
    }
  };

  auto finish = [&](int rg) {
    // partials of this warp -> shared, then one thread per output
#pragma unroll
    for (int ri = 0; ri < 2; ++ri)
#pragma unroll
      for (int ci = 0; ci < 2; ++ci) {
        const int col = 2 * t + ci;
        if (col < NB) red[(((size_t)tl * MKS + ks) * 16 + g + 8 * ri) * NB + col] = acc[ri][ci];
        acc[ri][ci] = 0.f;
      }
    __syncthreads();
    const int row_base = rg * MT * 16;
    auto total_of = [&](int lr, int col) {  // lr: row within the 32-row group
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < MKS; ++k) s += red[(((size_t)(lr >> 4) * MKS + k) * 16 + (lr & 15)) * NB + col];
      return s / 15.f;
    };
    if constexpr (EPI == EPI_STORE || EPI == EPI_RESID) {
      for (int i = threadIdx.x; i < MT * 16 * NB; i += blockDim.x) {
        const int lr = i / NB, col = i % NB, row = row_base + lr;
        if (row < a.rows && col < a.nb) {
          float v = total_of(lr, col);
          if constexpr (EPI == EPI_RESID) v = a.resid[(size_t)col * a.ldr + row] + v;
          a.y[(size_t)col * a.ldy + row] = v;
        }
      }
    } else if constexpr (EPI == EPI_SWIGLU) {
      // rows 2i = gate_i, 2i+1 = up_i (chat.py:300-302, the +-40 clip)
      for (int i = threadIdx.x; i < MT * 8 * NB; i += blockDim.x) {
        const int q = i / NB, col = i % NB, row = row_base + 2 * q;
        if (row + 1 < a.rows && col < a.nb) {
          const float gv = total_of(2 * q, col), uv = total_of(2 * q + 1, col);
          const float e = expf(-fminf(fmaxf(gv, -40.f), 40.f));
          a.y[(size_t)col * a.ldy + (row >> 1)] = gv / (1.0f + e) * uv;
        }
      }
    } else {
      const RopeKV& k = a.rk;
      const int qrows = k.nh * k.hd, krows = k.nkv * k.hd, hh = k.hd / 2;
      for (int i = threadIdx.x; i < MT * 8 * NB; i += blockDim.x) {
        const int q = i / NB, col = i % NB, row = row_base + 2 * q;
        if (row + 1 >= a.rows || col >= a.nb) continue;
        const float x1 = total_of(2 * q, col), x2 = total_of(2 * q + 1, col);
        const size_t blk = ep_blk[col], off = ep_off[col];
        if (row < qrows + krows) {
          const bool isq = row < qrows;
          const int rr = isq ? row : row - qrows;
          const int h = rr / k.hd, pp = (rr % k.hd) >> 1;
          const int pos = ep_pos[col];
          const float c = k.cos_t[(size_t)pos * hh + pp], s = k.sin_t[(size_t)pos * hh + pp];
          // rotate-half RoPE, fp32 products rounded separately (chat.py:99-100)
          const float o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
          const float o2 = __fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c));
          if (isq) {
            float* qo = k.q_out + (size_t)col * qrows + (size_t)h * k.hd;
            qo[pp] = o1;
            qo[pp + hh] = o2;
          } else {
            const size_t base = ((blk * k.nkv + h) * k.bs + off) * k.hd;
            if (k.kv_fp16) {
              static_cast<__half*>(k.kcache)[base + pp] = __float2half_rn(o1);
              static_cast<__half*>(k.kcache)[base + pp + hh] = __float2half_rn(o2);
            } else {
              static_cast<float*>(k.kcache)[base + pp] = o1;
              static_cast<float*>(k.kcache)[base + pp + hh] = o2;
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
    }
    __syncthreads();
  };

  for (int i = 0; i < total; i += 2) {
    if (i + 1 < total) load(i + 1, B);
    compute(A, i % nsteps);
    if (i % nsteps == nsteps - 1) finish(blockIdx.x + (i / nsteps) * gridDim.x);
    if (i + 1 >= total) break;
    if (i + 2 < total) load(i + 2, A);
    compute(B, (i + 1) % nsteps);
    if ((i + 1) % nsteps == nsteps - 1) finish(blockIdx.x + ((i + 1) / nsteps) * gridDim.x);
  }
}

template <int NB, typename ST, int EPI, bool NORM>
static int launch_mma(const MmaArgs& a, cudaStream_t s) {
  auto kern = gemv_mma_kernel<NB, ST, EPI, NORM>;
  const int nbp = 2 * a.np;
  if (NORM && nbp > MW * 16) return LUMINA_E_UNSUPPORTED;  // one-pass row norm
  const size_t smem = (size_t)nbp * NB * (64 + 8) + (size_t)MT * MKS * 16 * NB * 4;
  if (smem > 227 * 1024 - 2048) return LUMINA_E_UNSUPPORTED;
  const int rc = set_smem_limit((const void*)kern, smem, "gemv_mma");
  if (rc) return rc;
  const int grid = std::max(1, std::min(sm_count(), a.n_rg));
  const cudaError_t e = launch_pdl(kern, dim3(grid), dim3(MW * 32), smem, s, a);
  if (e != cudaSuccess) {
    set_error("gemv_mma launch: %s", cudaGetErrorString(e));
    return LUMINA_E_CUDA;
  }
  return LUMINA_OK;
}

template <int NB, typename ST>
static int mma_epi(const MmaArgs& a, int epi, bool norm, cudaStream_t s) {
  switch (epi) {
    case EPI_STORE: return norm ? launch_mma<NB, ST, EPI_STORE, true>(a, s) : launch_mma<NB, ST, EPI_STORE, false>(a, s);
    case EPI_RESID: return norm ? LUMINA_E_UNSUPPORTED : launch_mma<NB, ST, EPI_RESID, false>(a, s);
    case EPI_SWIGLU: return norm ? launch_mma<NB, ST, EPI_SWIGLU, true>(a, s) : LUMINA_E_UNSUPPORTED;
    default: return norm ? launch_mma<NB, ST, EPI_ROPE_KV, true>(a, s) : LUMINA_E_UNSUPPORTED;
  }
}

// batch in tiles of 8 (the MMA's N); each tile quantizes its own rows
int gemv_mma_launch(const lumina_weight* w, const float* x, int ldx, int batch, const float* norm_w, float eps,
                    float* y, int ldy, int epi, const float* resid, int ldr, cudaStream_t s, const RopeKV* rk) {
  if (!w->mma || w->bits != 4) return LUMINA_E_UNSUPPORTED;
  if ((epi == EPI_SWIGLU || epi == EPI_ROPE_KV) && (w->rows & 1)) {
    set_error("gemv: paired epilogue needs an even row count");
    return LUMINA_E_ARG;
  }
  for (int done = 0; done < batch;) {
    const int left = batch - done;
    const int nb = left >= 8 ? 8 : (left >= 4 ? 4 : (left >= 2 ? 2 : 1));
    MmaArgs a{};
    a.codes = w->codes;
    a.scales = w->scales;
    a.rows = w->rows;
    a.cols = w->cols;
    a.np = w->n_chunks / 2;  // MMA layout: n_chunks counts 32-column blocks, padded to pairs
    a.ng = w->n_groups;
    a.group = w->group;
    a.fp16 = w->fp16_scales;
    a.x = x + (size_t)done * ldx;
    a.ldx = ldx;
    a.norm_w = norm_w;
    a.eps = eps;
    a.y = y + (size_t)done * ldy;
    a.ldy = ldy;
    a.resid = resid ? resid + (size_t)done * ldr : nullptr;
    a.ldr = ldr;
    if (rk) {
      a.rk = *rk;
      a.rk.row_pos = rk->row_pos + done;
      a.rk.q_out = rk->q_out + (size_t)done * rk->nh * rk->hd;
      a.rk.row_base = rk->row_base + done;
    }
    a.nb = std::min(nb, left);
    a.n_rg = w->rows_pad / (MT * 16);
    int rc;
    const bool norm = norm_w != nullptr;
    if (w->fp16_scales) {
      rc = nb == 8 ? mma_epi<8, __half>(a, epi, norm, s) : nb == 4 ? mma_epi<4, __half>(a, epi, norm, s)
         : nb == 2 ? mma_epi<2, __half>(a, epi, norm, s) : mma_epi<1, __half>(a, epi, norm, s);
    } else {
      rc = nb == 8 ? mma_epi<8, float>(a, epi, norm, s) : nb == 4 ? mma_epi<4, float>(a, epi, norm, s)
         : nb == 2 ? mma_epi<2, float>(a, epi, norm, s) : mma_epi<1, float>(a, epi, norm, s);
    }
    if (rc) return rc;
    done += nb;
  }
  return LUMINA_OK;
}

}  // namespace lumina
