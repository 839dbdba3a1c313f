// Fused dequant GEMV over packed Lumina codes (the decode hot path).
//
// y[b, n] = sum_k x[b, k] * scale[n, k/g] * level(code[n, k]),
// level(c) = -1 + 2c/L, L = 2^bits - 1 (adapters/lumina.py:135-139;
// binary: c in {0,1} -> -1/+1, lumina.py:141-148).
//
// Arithmetic. Activations are quantized once per GEMV to int16 per 32-column
// block (the reference's own fused path repacks activations once per matmul,
// fused.py:91-102, with 8 bits; 16 bits keeps the activation error near 5e-5
// relative). For a block with activation scale sx, int16 values q and codes c:
//   sum_k x_k * level(c_k) = sx / L * (2 * sum q_k c_k - L * sum q_k)
// The integer dot sum q_k c_k is exact (dp2a: two int16 x two code bytes per
// instruction); codes are widened to bytes with one AND per four codes. Each
// block is scaled once in fp32; the row total is divided by L at the end.
//
// Mapping. One warp owns R rows at a time and sweeps K with its 32 lanes: lane
// l reads chunk (it*32 + l) of each of the R rows (16 contiguous bytes per row
// per lane, so a warp reads 512 contiguous bytes of a row), U chunks are in
// flight per row. The grid is persistent (grid-stride over row groups), sized
// from the occupancy of the instantiation. Partial sums are reduced with warp
// shuffles; lane k writes output k.
#include <mutex>
#include <vector>

#include "weights.cuh"

namespace lumina {

__device__ __forceinline__ int dp2a_lo(uint32_t a, uint32_t b, int c) {
  return __dp2a_lo((int)a, (int)b, c);
}
__device__ __forceinline__ int dp2a_hi(uint32_t a, uint32_t b, int c) {
  return __dp2a_hi((int)a, (int)b, c);
}

// Integer dot of one 32-column block: w = BITS words of codes, x = 16 words
// of permuted int16 activations.
template <int BITS>
__device__ __forceinline__ int block_dot(const uint32_t* w, const uint32_t* x, int d);

template <>
__device__ __forceinline__ int block_dot<4>(const uint32_t* w, const uint32_t* x, int d) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t lo = w[i] & 0x0F0F0F0Fu;         // columns 0,2,4,6 of the word
    const uint32_t hi = (w[i] >> 4) & 0x0F0F0F0Fu;  // columns 1,3,5,7
    d = dp2a_lo(x[4 * i + 0], lo, d);
    d = dp2a_hi(x[4 * i + 1], lo, d);
    d = dp2a_lo(x[4 * i + 2], hi, d);
    d = dp2a_hi(x[4 * i + 3], hi, d);
  }
  return d;
}

template <>
__device__ __forceinline__ int block_dot<2>(const uint32_t* w, const uint32_t* x, int d) {
#pragma unroll
  for (int i = 0; i < 2; ++i) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const uint32_t v = (w[i] >> (2 * t)) & 0x03030303u;  // columns t, 4+t, 8+t, 12+t
      d = dp2a_lo(x[8 * i + 2 * t], v, d);
      d = dp2a_hi(x[8 * i + 2 * t + 1], v, d);
    }
  }
  return d;
}

template <>
__device__ __forceinline__ int block_dot<3>(const uint32_t* w, const uint32_t* x, int d) {
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint32_t h = w[2] >> (4 * i);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const uint32_t v = ((w[i] >> (2 * t)) & 0x03030303u) | (((h >> t) & 0x01010101u) << 2);
      d = dp2a_lo(x[8 * i + 2 * t], v, d);
      d = dp2a_hi(x[8 * i + 2 * t + 1], v, d);
    }
  }
  return d;
}

template <>
__device__ __forceinline__ int block_dot<1>(const uint32_t* w, const uint32_t* x, int d) {
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const uint32_t v = (w[0] >> t) & 0x01010101u;  // columns t, 8+t, 16+t, 24+t
    d = dp2a_lo(x[2 * t], v, d);
    d = dp2a_hi(x[2 * t + 1], v, d);
  }
  return d;
}

template <typename ST>
__device__ __forceinline__ float load_scale(const void* p, size_t i) {
  if constexpr (sizeof(ST) == 2) {
    return __half2float(__ldg(reinterpret_cast<const __half*>(p) + i));
  } else {
    return __ldg(reinterpret_cast<const float*>(p) + i);
  }
}

constexpr int GEMV_WARPS = 8;

template <int BITS, int R, int U, int NB, typename ST, int EPI>
__global__ void __launch_bounds__(GEMV_WARPS * 32)
gemv_kernel(GemvArgs a) {
  using Lt = Layout<BITS>;
  constexpr int CW = Lt::CHUNK_WORDS;
  constexpr int CB = Lt::CB;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int n_tasks = (a.rows + R - 1) / R;
  const int stride = gridDim.x * GEMV_WARPS;
  bool waited = false;
  pdl_launch_dependents();

  for (int task = blockIdx.x * GEMV_WARPS + warp; task < n_tasks; task += stride) {
    const int row0 = task * R;
    float acc[R][NB];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[r][b] = 0.f;

    for (int cbase = 0; cbase < a.n_chunks; cbase += 32 * U) {
      uint32_t wv[U][R][CW];
      // 1) issue every code load of this sweep step (weights never depend on
      //    the previous kernel, so they go out before the PDL wait)
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = cbase + u * 32 + lane;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int row = min(row0 + r, a.rows - 1);
          const uint8_t* p = a.codes + (size_t)row * a.row_bytes + (size_t)c * Lt::CHUNK_BYTES;
#pragma unroll
          for (int q = 0; q < CW / 4; ++q) {
            uint4 v = make_uint4(0, 0, 0, 0);
            if (c < a.n_chunks) v = ldg_stream(p + 16 * q);
            wv[u][r][4 * q + 0] = v.x;
            wv[u][r][4 * q + 1] = v.y;
            wv[u][r][4 * q + 2] = v.z;
            wv[u][r][4 * q + 3] = v.w;
          }
        }
      }
      if (!waited) {
        pdl_wait();
        waited = true;
      }
      // 2) consume chunk by chunk
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = cbase + u * 32 + lane;
        if (c >= a.n_chunks) continue;
#pragma unroll
        for (int cb = 0; cb < CB; ++cb) {
          const int blk = c * CB + cb;
          const int g = (blk * 32) / a.group;
          float sc[R];
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const int row = min(row0 + r, a.rows - 1);
            sc[r] = load_scale<ST>(a.scales, (size_t)row * a.n_groups + g);
          }
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            const size_t xb = (size_t)b * a.nblk_pad + blk;
            uint32_t xr[16];
            const uint4* xp = reinterpret_cast<const uint4*>(a.xq + xb * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 v = ldg_cached(xp + q);
              xr[4 * q + 0] = v.x;
              xr[4 * q + 1] = v.y;
              xr[4 * q + 2] = v.z;
              xr[4 * q + 3] = v.w;
            }
            const int xs = __ldg(a.xsum + xb);
            const float fx = __ldg(a.sx + xb);
#pragma unroll
            for (int r = 0; r < R; ++r) {
              const int d = block_dot<BITS>(&wv[u][r][cb * BITS], xr, 0);
              const int t = 2 * d - xs;
              acc[r][b] = fmaf((float)t, fx * sc[r], acc[r][b]);
            }
          }
        }
      }
    }
    if (!waited) {
      pdl_wait();
      waited = true;
    }
    // 3) reduce and write: lane k owns output k of the R x NB tile
    float mine = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const float v = warp_sum(acc[r][b]) / (float)Lt::L;
        if (lane == r * NB + b) mine = v;
        acc[r][b] = v;
      }
    if constexpr (EPI == EPI_SWIGLU) {
      // rows are interleaved gate/up pairs: row 2i = gate_i, 2i+1 = up_i
      // (chat.py:300-302: silu(g) * u with the +-40 clip)
#pragma unroll
      for (int j = 0; j < R / 2; ++j)
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const int o = (row0 >> 1) + j;
          if (lane == j * NB + b && row0 + 2 * j + 1 < a.rows) {
            const float gv = acc[2 * j][b], uv = acc[2 * j + 1][b];
            const float e = expf(-fminf(fmaxf(gv, -40.f), 40.f));
            a.y[(size_t)b * a.ldy + o] = gv / (1.0f + e) * uv;
          }
        }
    } else {
      if (lane < R * NB) {
        const int r = lane / NB, b = lane % NB;
        const int row = row0 + r;
        if (row < a.rows) {
          float v = mine;
          if constexpr (EPI == EPI_RESID) v = a.resid[(size_t)b * a.ldr + row] + v;
          a.y[(size_t)b * a.ldy + row] = v;
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// activation quantization
// ---------------------------------------------------------------------------

// Slot of column j of a 32-column block in the permuted order.
template <int PERM>
__device__ __forceinline__ int perm_slot(int j) {
  if constexpr (PERM == 8) {
    const int g = j >> 3, i = j & 7;
    return g * 8 + ((i & 1) ? 4 + (i >> 1) : (i >> 1));
  } else if constexpr (PERM == 16) {
    const int g = j >> 4, i = j & 15;
    return g * 16 + (i & 3) * 4 + (i >> 2);
  } else {
    return (j & 7) * 4 + (j >> 3);
  }
}

template <int PERM, bool NORM>
__global__ void __launch_bounds__(256)
act_quant_kernel(const float* __restrict__ x, int ldx, int K, const float* __restrict__ norm_w,
                 float eps, int L, int16_t* __restrict__ xq, float* __restrict__ sx,
                 int* __restrict__ xsum, int nblk_pad) {
  const int b = blockIdx.x;
  const float* xr = x + (size_t)b * ldx;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __shared__ float red[8];
  pdl_launch_dependents();
  pdl_wait();
  float inv = 1.f;
  if constexpr (NORM) {
    // chat.py:63-66: x / sqrt(mean(x^2) + eps) * w, fp32
    float ss = 0.f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) ss = fmaf(xr[k], xr[k], ss);
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (warp == 0) {
      float v = lane < 8 ? red[lane] : 0.f;
      v = warp_sum(v);
      if (lane == 0) red[0] = v;
    }
    __syncthreads();
    inv = sqrtf(red[0] / (float)K + eps);
  }
  for (int blk = warp; blk < nblk_pad; blk += 8) {
    const int k = blk * 32 + lane;
    float v = 0.f;
    if (k < K) {
      v = xr[k];
      if constexpr (NORM) v = (v / inv) * norm_w[k];
    }
    const float amax = warp_max(fabsf(v));
    int q = 0;
    float s = 0.f;
    if (amax > 0.f) {
      const float f = __fdiv_rn(32767.f, amax);
      q = __float2int_rn(__fmul_rn(v, f));
      q = max(-32767, min(32767, q));
      s = __fdiv_rn(amax, 32767.f);
    }
    const int qs = warp_sum_int(q);
    const size_t base = (size_t)b * nblk_pad + blk;
    xq[base * 32 + perm_slot<PERM>(lane)] = (int16_t)q;
    if (lane == 0) {
      sx[base] = s;
      xsum[base] = L * qs;
    }
  }
}

int act_quant(const float* x, int ldx, int batch, int K, const float* norm_w, float eps, int bits,
              const ActQ& q, cudaStream_t s) {
  const int L = (1 << bits) - 1;
  const int perm = perm_kind(bits);
  dim3 grid(batch), block(256);
  cudaError_t e;
#define AQ(P, N)                                                                          \
  e = launch_pdl(act_quant_kernel<P, N>, grid, block, 0, s, x, ldx, K, norm_w, eps, L, q.xq, \
                 q.sx, q.xsum, q.nblk_pad)
  if (norm_w) {
    if (perm == 8) AQ(8, true); else if (perm == 16) AQ(16, true); else AQ(32, true);
  } else {
    if (perm == 8) AQ(8, false); else if (perm == 16) AQ(16, false); else AQ(32, false);
  }
#undef AQ
  if (e != cudaSuccess) {
    set_error("act_quant launch: %s", cudaGetErrorString(e));
    return LUMINA_E_CUDA;
  }
  return LUMINA_OK;
}

// ---------------------------------------------------------------------------
// launch dispatch
// ---------------------------------------------------------------------------

template <int BITS, int R, int U, int NB, typename ST, int EPI>
static int launch_one(const GemvArgs& a, cudaStream_t s) {
  auto kern = gemv_kernel<BITS, R, U, NB, ST, EPI>;
  static int per_sm = -1;
  if (per_sm < 0) {
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, kern, GEMV_WARPS * 32, 0) != cudaSuccess || v < 1)
      v = 1;
    per_sm = v;
  }
  const int n_tasks = (a.rows + R - 1) / R;
  int grid = (n_tasks + GEMV_WARPS - 1) / GEMV_WARPS;
  grid = std::min(grid, per_sm * sm_count());
  grid = std::max(grid, 1);
  cudaError_t e = launch_pdl(kern, dim3(grid), dim3(GEMV_WARPS * 32), 0, s, a);
  if (e != cudaSuccess) {
    set_error("gemv launch: %s", cudaGetErrorString(e));
    return LUMINA_E_CUDA;
  }
  return LUMINA_OK;
}

template <int BITS, int R, int U, typename ST, int EPI>
static int dispatch_nb(const GemvArgs& a, int nb, cudaStream_t s) {
  switch (nb) {
    case 1: return launch_one<BITS, R, U, 1, ST, EPI>(a, s);
    case 2: return launch_one<BITS, R, U, 2, ST, EPI>(a, s);
    case 4: return launch_one<BITS, R, U, 4, ST, EPI>(a, s);
    case 8: return launch_one<BITS, R, 1, 8, ST, EPI>(a, s);
  }
  set_error("gemv: unsupported batch tile %d", nb);
  return LUMINA_E_UNSUPPORTED;
}

template <int BITS, typename ST, int EPI>
static int dispatch_shape(const GemvArgs& a, int nb, cudaStream_t s) {
  // R rows per warp, U chunks in flight per row: R*U chunk loads outstanding
  // per lane. Fewer, taller tasks when there are many rows; more, shorter
  // tasks when rows are few so every SM gets warps.
  constexpr int RB = (BITS == 3) ? 2 : 4;
  const long tasks4 = (a.rows + 3) / 4;
  if (tasks4 >= 148L * 16 || EPI == EPI_SWIGLU)
    return dispatch_nb<BITS, RB, (BITS == 3 ? 2 : 2), ST, EPI>(a, nb, s);
  return dispatch_nb<BITS, 2, (BITS == 3 ? 2 : 4), ST, EPI>(a, nb, s);
}

template <int BITS>
static int dispatch_bits(const GemvArgs& a, int nb, int fp16, int epi, cudaStream_t s) {
  if (fp16) {
    if (epi == EPI_STORE) return dispatch_shape<BITS, __half, EPI_STORE>(a, nb, s);
    if (epi == EPI_RESID) return dispatch_shape<BITS, __half, EPI_RESID>(a, nb, s);
    return dispatch_shape<BITS, __half, EPI_SWIGLU>(a, nb, s);
  }
  if (epi == EPI_STORE) return dispatch_shape<BITS, float, EPI_STORE>(a, nb, s);
  if (epi == EPI_RESID) return dispatch_shape<BITS, float, EPI_RESID>(a, nb, s);
  return dispatch_shape<BITS, float, EPI_SWIGLU>(a, nb, s);
}

int gemv_launch(const lumina_weight* w, const ActQ& q, int batch, float* y, int ldy, int epi,
                const float* resid, int ldr, cudaStream_t s) {
  if (epi == EPI_SWIGLU && (w->rows & 1)) {
    set_error("gemv: swiglu epilogue needs an even (gate/up interleaved) row count");
    return LUMINA_E_ARG;
  }
  int done = 0;
  while (done < batch) {
    const int left = batch - done;
    const int nb = left >= 8 ? 8 : (left >= 4 ? 4 : (left >= 2 ? 2 : 1));
    GemvArgs a;
    a.codes = w->codes;
    a.scales = w->scales;
    a.rows = w->rows;
    a.row_bytes = w->row_bytes;
    a.n_chunks = w->n_chunks;
    a.n_groups = w->n_groups;
    a.group = w->group;
    a.xq = q.xq + (size_t)done * q.nblk_pad * 32;
    a.sx = q.sx + (size_t)done * q.nblk_pad;
    a.xsum = q.xsum + (size_t)done * q.nblk_pad;
    a.nblk_pad = q.nblk_pad;
    a.y = y + (size_t)done * ldy;
    a.ldy = ldy;
    a.resid = resid ? resid + (size_t)done * ldr : nullptr;
    a.ldr = ldr;
    int rc;
    switch (w->bits) {
      case 4: rc = dispatch_bits<4>(a, nb, w->fp16_scales, epi, s); break;
      case 3: rc = dispatch_bits<3>(a, nb, w->fp16_scales, epi, s); break;
      case 2: rc = dispatch_bits<2>(a, nb, w->fp16_scales, epi, s); break;
      case 1: rc = dispatch_bits<1>(a, nb, w->fp16_scales, epi, s); break;
      default: set_error("gemv: bad bits %d", w->bits); return LUMINA_E_ARG;
    }
    if (rc) return rc;
    done += nb;
  }
  return LUMINA_OK;
}

}  // namespace lumina
