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
// Two kernels share that arithmetic:
//  * gemv_fused_kernel (decode, batch <= 4): one CTA of 16 warps per SM.
//    Each warp owns a contiguous run of R-row groups and streams their
//    (row group, slice) tiles -- codes and scales -- from HBM into its own
//    ring of S shared-memory stages with cp.async.bulk (the bulk-copy
//    engine), completion tracked by mbarriers. The first S tiles are
//    requested before griddepcontrol.wait, i.e. while the previous kernel of
//    the layer is still finishing (weights never depend on it). The CTA then
//    RMS-normalizes (optional) and quantizes the activation rows into shared
//    memory and consumes tiles as they land.
//  * gemv_kernel (any batch): activations pre-quantized in global memory by
//    act_quant_kernel; one warp per R rows, lanes across K with 16-byte
//    streaming loads. Used for prefill chunks.
// Epilogues: store, residual add (in place), SwiGLU over interleaved
// gate/up rows, and RoPE + paged KV append over the fused q/k/v rows.
#include <mutex>
#include <vector>

#include "gemv_impl.cuh"

namespace lumina {

extern template int gemv_bits<1>(const GemvArgs&, int, int, int, cudaStream_t);
extern template int gemv_bits<2>(const GemvArgs&, int, int, int, cudaStream_t);
extern template int gemv_bits<3>(const GemvArgs&, int, int, int, cudaStream_t);
extern template int gemv_bits<4>(const GemvArgs&, int, int, int, cudaStream_t);
extern template int gemv_fused_bits<1>(FusedArgs&, const lumina_weight*, int, int, bool, cudaStream_t);
extern template int gemv_fused_bits<2>(FusedArgs&, const lumina_weight*, int, int, bool, cudaStream_t);
extern template int gemv_fused_bits<3>(FusedArgs&, const lumina_weight*, int, int, bool, cudaStream_t);
extern template int gemv_fused_bits<4>(FusedArgs&, const lumina_weight*, int, int, bool, cudaStream_t);

// ---------------------------------------------------------------------------
// activation quantization into global memory (prefill path)
// ---------------------------------------------------------------------------
// One warp per 32-column block, 8 blocks per CTA, grid (blocks / 8, batch).
// With NORM each CTA first reduces the whole row's sum of squares.
template <int PERM, bool NORM>
__global__ void __launch_bounds__(256)
act_quant_kernel(const float* __restrict__ x, int ldx, int K, const float* __restrict__ norm_w,
                 float eps, int L, int16_t* __restrict__ xq, float* __restrict__ sx,
                 int* __restrict__ xsum, int nblk_pad) {
  const int b = blockIdx.y;
  const float* xr = x + (size_t)b * ldx;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int blk = blockIdx.x * 8 + warp;
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
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    inv = 1.0f / sqrtf(tot / (float)K + eps);
  }
  if (blk >= nblk_pad) return;
  const int k = blk * 32 + lane;
  float v = 0.f;
  if (k < K) {
    v = xr[k];
    if constexpr (NORM) v = (v * inv) * norm_w[k];  // same arithmetic as the fused GEMV prologue
  }
  int q, qs;
  float s;
  quant_block(v, q, s, qs);
  const size_t base = (size_t)b * nblk_pad + blk;
  xq[base * 32 + perm_slot<PERM>(lane)] = (int16_t)q;
  if (lane == 0) {
    sx[base] = s;
    xsum[base] = L * qs;
  }
}

int act_quant(const float* x, int ldx, int batch, int K, const float* norm_w, float eps, int bits,
              const ActQ& q, cudaStream_t s) {
  const int L = (1 << bits) - 1;
  const int perm = perm_kind(bits);
  dim3 grid((q.nblk_pad + 7) / 8, batch), block(256);
  cudaError_t e;
#define AQ(P, N)                                                                                 \
  e = launch_pdl(act_quant_kernel<P, N>, grid, block, 0, s, x, ldx, K, norm_w, eps, L, q.xq, q.sx, \
                 q.xsum, q.nblk_pad)
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

static GemvArgs make_args(const lumina_weight* w, float* y, int ldy, const float* resid, int ldr,
                          const RopeKV* rk) {
  GemvArgs a{};
  a.w = *w;
  a.y = y;
  a.ldy = ldy;
  a.resid = resid;
  a.ldr = ldr;
  if (rk) a.rk = *rk;
  return a;
}

int gemv_launch(const lumina_weight* w, const ActQ& q, int batch, float* y, int ldy, int epi, const float* resid,
                int ldr, cudaStream_t s, const RopeKV* rk) {
  if ((epi == EPI_SWIGLU || epi == EPI_ROPE_KV) && (w->rows & 1)) {
    set_error("gemv: paired epilogue needs an even row count");
    return LUMINA_E_ARG;
  }
  int done = 0;
  while (done < batch) {
    const int left = batch - done;
    const int nb = left >= 8 ? 8 : (left >= 4 ? 4 : (left >= 2 ? 2 : 1));
    GemvArgs a = make_args(w, y + (size_t)done * ldy, ldy, resid ? resid + (size_t)done * ldr : nullptr, ldr, rk);
    a.xq = q.xq + (size_t)done * q.nblk_pad * 32;
    a.sx = q.sx + (size_t)done * q.nblk_pad;
    a.xsum = q.xsum + (size_t)done * q.nblk_pad;
    a.nblk_pad = q.nblk_pad;
    if (rk) {
      a.rk.row_pos = rk->row_pos + done;
      a.rk.q_out = rk->q_out + (size_t)done * rk->nh * rk->hd;
      a.rk.row_base = rk->row_base + done;
    }
    int rc;
    switch (w->bits) {
      case 4: rc = gemv_bits<4>(a, nb, w->fp16_scales, epi, s); break;
      case 3: rc = gemv_bits<3>(a, nb, w->fp16_scales, epi, s); break;
      case 2: rc = gemv_bits<2>(a, nb, w->fp16_scales, epi, s); break;
      case 1: rc = gemv_bits<1>(a, nb, w->fp16_scales, epi, s); break;
      default: set_error("gemv: bad bits %d", w->bits); return LUMINA_E_ARG;
    }
    if (rc) return rc;
    done += nb;
  }
  return LUMINA_OK;
}

int gemv_fused_launch(const lumina_weight* w, const float* x, int ldx, int batch, const float* norm_w, float eps,
                      float* y, int ldy, int epi, const float* resid, int ldr, cudaStream_t s, const RopeKV* rk) {
  if (batch != 1 && batch != 2 && batch != 4) return LUMINA_E_UNSUPPORTED;
  if ((epi == EPI_SWIGLU || epi == EPI_ROPE_KV) && (w->rows & 1)) {
    set_error("gemv: paired epilogue needs an even row count");
    return LUMINA_E_ARG;
  }
  int* fault = fault_flag_ptr();
  if (!fault) {
    set_error("gemv_fused: fault flag unavailable");
    return LUMINA_E_CUDA;
  }
  FusedArgs fa{};
  fa.g = make_args(w, y, ldy, resid, ldr, rk);
  fa.x = x;
  fa.ldx = ldx;
  fa.norm_w = norm_w;
  fa.eps = eps;
  fa.K = w->cols;
  fa.fault = fault;
  fa.spin = wait_spin_limit();
  const bool norm = norm_w != nullptr;
  switch (w->bits) {
    case 4: return gemv_fused_bits<4>(fa, w, batch, epi, norm, s);
    case 3: return gemv_fused_bits<3>(fa, w, batch, epi, norm, s);
    case 2: return gemv_fused_bits<2>(fa, w, batch, epi, norm, s);
    case 1: return gemv_fused_bits<1>(fa, w, batch, epi, norm, s);
  }
  return LUMINA_E_UNSUPPORTED;
}

}  // namespace lumina
