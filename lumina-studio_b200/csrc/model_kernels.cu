// Decode-step kernels around the packed GEMV: embedding gather, RoPE + paged
// KV append, split-KV attention and its combine, fp16 dense GEMV (LM head and
// raw projections), argmax, KV row gather / read-back.
#include <cfloat>

#include "model.cuh"

namespace lumina {

#define RET_LAUNCH(e)                                                  \
  do {                                                                 \
    cudaError_t _e = (e);                                              \
    if (_e != cudaSuccess) {                                           \
      set_error("launch failed: %s (%s:%d)", cudaGetErrorString(_e), __FILE__, __LINE__); \
      return LUMINA_E_CUDA;                                            \
    }                                                                  \
  } while (0)

// ---------------------------------------------------------------------------
// embedding: x[i] = float(embed[tokens[i]])  (chat.py:326,400,541 — the fp16
// model copy, chat.py:140, cast to fp32)
// ---------------------------------------------------------------------------
__global__ void embed_kernel(const __half* __restrict__ emb, int d, const int* __restrict__ tokens,
                             const DevParams* __restrict__ P, float* __restrict__ x, int vocab,
                             unsigned long long* __restrict__ argmax_key) {
  pdl_launch_dependents();
  pdl_wait();
  const int i = blockIdx.y;
  if (argmax_key && i == 0 && blockIdx.x == 0 && threadIdx.x == 0) *argmax_key = 0ull;
  if (i >= P->n) return;
  int t = tokens[i];
  t = t < 0 ? 0 : (t >= vocab ? vocab - 1 : t);  // ids are range-checked on the host
  const __half* row = emb + (size_t)t * d;
  for (int k = (blockIdx.x * blockDim.x + threadIdx.x) * 2; k < d; k += gridDim.x * blockDim.x * 2) {
    const float2 v = __half22float2(*reinterpret_cast<const __half2*>(row + k));
    x[(size_t)i * d + k] = v.x;
    x[(size_t)i * d + k + 1] = v.y;
  }
}

// ---------------------------------------------------------------------------
// RoPE (rotate-half, chat.py:88-103) on q and k, then K/V rows into the paged
// cache at positions t_prev + i. cos/sin come from tables indexed by the row
// position (rope_freqs / rope_angles_at, chat.py:69-85).
// qkv: (n, (nh + 2 nkv) * hd) fp32. q_out: (n, nh * hd) rotated queries.
// ---------------------------------------------------------------------------
template <typename KT>
__global__ void rope_append_kernel(const float* __restrict__ qkv, int nh, int nkv, int hd,
                                   const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                   int half, const int* __restrict__ row_pos, const DevParams* __restrict__ P,
                                   const int* __restrict__ block_table, int bs, KT* __restrict__ kcache,
                                   KT* __restrict__ vcache, float* __restrict__ q_out) {
  pdl_launch_dependents();
  pdl_wait();
  const int i = blockIdx.x;  // row
  if (i >= P->n) return;
  const int width = (nh + 2 * nkv) * hd;
  const float* src = qkv + (size_t)i * width;
  const int pos = row_pos[i];
  const float* c = cos_t + (size_t)pos * half;
  const float* s = sin_t + (size_t)pos * half;
  const int t = P->t_prev + i;
  const int blk = block_table[t / bs], off = t % bs;
  const int P2 = hd / 2;
  // queries
  for (int e = threadIdx.x; e < nh * P2; e += blockDim.x) {
    const int h = e / P2, j = e % P2;
    const float x1 = src[h * hd + j], x2 = src[h * hd + P2 + j];
    q_out[(size_t)i * nh * hd + h * hd + j] = __fsub_rn(__fmul_rn(x1, c[j]), __fmul_rn(x2, s[j]));
    q_out[(size_t)i * nh * hd + h * hd + P2 + j] = __fadd_rn(__fmul_rn(x1, s[j]), __fmul_rn(x2, c[j]));
  }
  // keys (rotated) and values
  const size_t bstride = (size_t)nkv * bs * hd;
  for (int e = threadIdx.x; e < nkv * P2; e += blockDim.x) {
    const int h = e / P2, j = e % P2;
    const float x1 = src[(nh + h) * hd + j], x2 = src[(nh + h) * hd + P2 + j];
    KT* kr = kcache + (size_t)blk * bstride + ((size_t)h * bs + off) * hd;
    kr[j] = to_kv<KT>(__fsub_rn(__fmul_rn(x1, c[j]), __fmul_rn(x2, s[j])));
    kr[P2 + j] = to_kv<KT>(__fadd_rn(__fmul_rn(x1, s[j]), __fmul_rn(x2, c[j])));
  }
  for (int e = threadIdx.x; e < nkv * hd; e += blockDim.x) {
    const int h = e / hd, j = e % hd;
    KT* vr = vcache + (size_t)blk * bstride + ((size_t)h * bs + off) * hd;
    vr[j] = to_kv<KT>(src[(nh + nkv + h) * hd + j]);
  }
}

// ---------------------------------------------------------------------------
// fp16-weight GEMV, fp32 x / accumulate: the LM head (chat.py:388, fp16 head
// from chat.py:140) and projections a file keeps raw. Warp per 2 rows, lanes
// along K with 16-byte loads.
// ---------------------------------------------------------------------------
// orderable key of (value, index): larger value wins, then the smaller index
__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
  const unsigned u = __float_as_uint(v);
  const unsigned ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)i);
}

template <int NB, int EPI>
__global__ void __launch_bounds__(256)
dense_gemv_kernel(const __half* __restrict__ W, int N, int K, const float* __restrict__ x, int ldx,
                  float* __restrict__ y, int ldy, const float* __restrict__ resid, int ldr,
                  unsigned long long* __restrict__ amax, L2Prefetch pf) {
  unsigned long long best = 0ull;
  constexpr int R = 2;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n_tasks = (N + R - 1) / R;
  const int n8 = K / 8;
  pdl_launch_dependents();
  if (lane == 0) l2_prefetch_share(pf, blockIdx.x * 8 + warp, gridDim.x * 8);
  bool waited = false;
  for (int task = blockIdx.x * 8 + warp; task < n_tasks; task += gridDim.x * 8) {
    const int row0 = task * R;
    float acc[R][NB];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[r][b] = 0.f;
    for (int c0 = 0; c0 < n8; c0 += 64) {
      uint4 wv[2][R];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int c = c0 + u * 32 + lane;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int row = min(row0 + r, N - 1);
          wv[u][r] = c < n8 ? ldg_stream(W + (size_t)row * K + (size_t)c * 8) : make_uint4(0, 0, 0, 0);
        }
      }
      if (!waited) {
        pdl_wait();
        waited = true;
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c >= n8) continue;
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const float4* xp = reinterpret_cast<const float4*>(x + (size_t)b * ldx + (size_t)c * 8);
          const float4 xa = __ldg(xp), xb = __ldg(xp + 1);
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const __half2* hp = reinterpret_cast<const __half2*>(&wv[u][r]);
            const float2 w0 = __half22float2(hp[0]), w1 = __half22float2(hp[1]);
            const float2 w2 = __half22float2(hp[2]), w3 = __half22float2(hp[3]);
            float a = acc[r][b];
            a = fmaf(xa.x, w0.x, a); a = fmaf(xa.y, w0.y, a);
            a = fmaf(xa.z, w1.x, a); a = fmaf(xa.w, w1.y, a);
            a = fmaf(xb.x, w2.x, a); a = fmaf(xb.y, w2.y, a);
            a = fmaf(xb.z, w3.x, a); a = fmaf(xb.w, w3.y, a);
            acc[r][b] = a;
          }
        }
      }
    }
    if (!waited) {
      pdl_wait();
      waited = true;
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const float v = warp_sum(acc[r][b]);
        const int row = row0 + r;
        if (amax && b == 0 && row < N) best = max(best, argmax_key(v, row));
        if (lane == r * NB + b && row < N) {
          if constexpr (EPI == EPI_RESID) y[(size_t)b * ldy + row] = resid[(size_t)b * ldr + row] + v;
          else y[(size_t)b * ldy + row] = v;
        }
      }
  }
  if (amax && lane == 0 && best) atomicMax(amax, best);
}

// Build a fused weight: out row r <- row src_row[r] of source src_sel[r]
// (all sources share kind / group / width / scale type / layout). Row-major
// layouts copy whole chunks; the fragment layout rebuilds each byte from the
// two source rows (g, g + 8) that share it.
__device__ __forceinline__ int gather_code(const lumina_weight& w, int r, int k) {
  if (!w.mma)  // row-major int4: 32 columns per 16-byte chunk, even column in the low nibble
    return (w.codes[code_offset(w, r, k >> 5) + ((k & 31) >> 1)] >> (4 * (k & 1))) & 0xF;
  int nib = 0;
  const size_t o = mma_code_byte(w, r, k, &nib);
  return (w.codes[o] >> (4 * nib)) & 0xF;
}

__global__ void gather_rows_kernel(lumina_weight out, lumina_weight s0, lumina_weight s1, lumina_weight s2,
                                   const int* __restrict__ sel, const int* __restrict__ srow) {
  const int es = out.fp16_scales ? 2 : 4;
  auto src_of = [&](int r) -> const lumina_weight& { return sel[r] == 0 ? s0 : (sel[r] == 1 ? s1 : s2); };
  if (!out.mma) {
    const int chb = chunk_bytes(out.bits);
    const size_t total = (size_t)out.rows * (out.n_chunks + out.n_groups);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
      const int r = (int)(i / (out.n_chunks + out.n_groups));
      const int k = (int)(i % (out.n_chunks + out.n_groups));
      const lumina_weight& src = src_of(r);
      const int sr = srow[r];
      if (k < out.n_chunks) {
        const uint8_t* a = src.codes + code_offset(src, sr, k);
        uint8_t* b = out.codes + code_offset(out, r, k);
        for (int q = 0; q < chb; q += 16) *reinterpret_cast<uint4*>(b + q) = *reinterpret_cast<const uint4*>(a + q);
      } else {
        const int g = k - out.n_chunks;
        const uint8_t* a = src.scales + scale_offset(src, sr, g);
        uint8_t* b = out.scales + scale_offset(out, r, g);
        for (int q = 0; q < es; ++q) b[q] = a[q];
      }
    }
    return;
  }
  // fragment layout: one thread per output code byte (rows g and g + 8)
  const int cols = out.n_chunks * 32;
  const size_t nbytes = (size_t)out.rows_pad * cols / 2;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nbytes; i += (size_t)gridDim.x * blockDim.x) {
    // invert mma_code_byte: i = (((T * np + p) * 32 + lane) * 16 + j * 4 + cc3)
    const int cc3 = (int)(i & 3), j = (int)((i >> 2) & 3), lane = (int)((i >> 4) & 31);
    const size_t tp = i >> 9;
    const int np = out.n_chunks / 2;
    const int p = (int)(tp % np), T = (int)(tp / np);
    const int g = lane >> 2, t = lane & 3;
    const int col = (2 * p + (j >> 1)) * 32 + (j & 1) * 16 + 4 * t + cc3;
    uint8_t v = 0;
    for (int h = 0; h < 2; ++h) {
      const int r = T * 16 + g + 8 * h;
      if (r < out.rows && col < out.cols) v |= (uint8_t)(gather_code(src_of(r), srow[r], col) << (4 * h));
    }
    out.codes[i] = v;
  }
  const size_t nsc = (size_t)out.rows * out.n_groups;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nsc; i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / out.n_groups), g = (int)(i % out.n_groups);
    const lumina_weight& src = src_of(r);
    const uint8_t* a = src.scales + (src.mma ? mma_scale_offset(src, srow[r], g) : scale_offset(src, srow[r], g));
    uint8_t* b = out.scales + mma_scale_offset(out, r, g);
    for (int q = 0; q < es; ++q) b[q] = a[q];
  }
}

int launch_gather_rows(const lumina_weight& out, const lumina_weight& s0, const lumina_weight& s1,
                       const lumina_weight& s2, const int* sel, const int* srow, cudaStream_t s) {
  gather_rows_kernel<<<4 * sm_count(), 256, 0, s>>>(out, s0, s1, s2, sel, srow);
  RET_LAUNCH(cudaGetLastError());
  return LUMINA_OK;
}

// SwiGLU on separate gate/up outputs (chat.py:300-302).
__global__ void swiglu_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ o,
                              int n, int ffn, int ld) {
  pdl_launch_dependents();
  pdl_wait();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (size_t)n * ffn;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / ffn, c = i % ffn;
    const float gv = g[r * ld + c], uv = u[r * ld + c];
    o[r * ffn + c] = gv / (1.0f + expf(-fminf(fmaxf(gv, -40.f), 40.f))) * uv;
  }
}

// Argmax of one logits row, first maximum wins (np.argmax, chat.py:339).
__global__ void argmax_kernel(const float* __restrict__ v, int n, int* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float x = v[i];
    if (x > best || bi == 0x7fffffff) {  // strided scan: the first maximum is kept
      best = x;
      bi = i;
    }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) {
      best = ob;
      bi = oi;
    }
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) {
    sb[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sb[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    if (lane == 0) *out = bi == 0x7fffffff ? 0 : bi;
  }
}

// Rows [start, start+n) of one layer to fp32 (n, n_heads, hd), GQA-expanded.
template <typename KT>
__global__ void kv_read_kernel(const KT* __restrict__ kc, const KT* __restrict__ vc, const int* __restrict__ bt,
                               int bs, int nh, int nkv, int hd, int start, int n, float* __restrict__ ko,
                               float* __restrict__ vo) {
  const size_t total = (size_t)n * nh * hd;
  const size_t bstride = (size_t)nkv * bs * hd;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / ((size_t)nh * hd));
    const int h = (int)((i / hd) % nh), e = (int)(i % hd);
    const int t = start + r;
    const size_t src = (size_t)bt[t / bs] * bstride + ((size_t)(h / (nh / nkv)) * bs + t % bs) * hd + e;
    ko[i] = from_kv(kc[src]);
    vo[i] = from_kv(vc[src]);
  }
}

// EAGLE commit gather (eagle.py:343-350): row base+i <- row base+src[i].
// Reads every source row into `tmp` first, then writes, so overlapping moves
// are safe. tmp: (n, 2, nkv, hd) per layer, launched per layer.
template <typename KT>
__global__ void kv_gather_kernel(KT* __restrict__ kc, KT* __restrict__ vc, const int* __restrict__ bt, int bs,
                                 int nkv, int hd, int base, const int* __restrict__ src, int n,
                                 KT* __restrict__ tmp, int phase) {
  const size_t per = (size_t)nkv * hd;
  const size_t bstride = (size_t)nkv * bs * hd;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (size_t)n * per;
       i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / per);
    const int h = (int)((i % per) / hd), e = (int)(i % hd);
    const int t = phase == 0 ? base + src[r] : base + r;
    const size_t off = (size_t)bt[t / bs] * bstride + ((size_t)h * bs + t % bs) * hd + e;
    if (phase == 0) {
      tmp[(size_t)r * 2 * per + (i % per)] = kc[off];
      tmp[(size_t)r * 2 * per + per + (i % per)] = vc[off];
    } else {
      kc[off] = tmp[(size_t)r * 2 * per + (i % per)];
      vc[off] = tmp[(size_t)r * 2 * per + per + (i % per)];
    }
  }
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------


int launch_embed(const __half* emb, int d, int vocab, const int* tokens, const DevParams* P, float* x, int max_n,
                 unsigned long long* argmax_key, cudaStream_t s) {
  const int gx = std::max(1, (d / 2 + 255) / 256);
  RET_LAUNCH(launch_pdl(embed_kernel, dim3(gx, std::max(1, max_n)), dim3(256), 0, s, emb, d, tokens, P, x, vocab,
                        argmax_key));
  return LUMINA_OK;
}

int launch_rope_append(bool fp16, const float* qkv, int nh, int nkv, int hd, const float* cos_t, const float* sin_t,
                       const int* row_pos, const DevParams* P, const int* bt, int bs, void* kc, void* vc,
                       float* q_out, int max_n, cudaStream_t s) {
  const int half = hd / 2;
  if (fp16)
    RET_LAUNCH(launch_pdl(rope_append_kernel<__half>, dim3(max_n), dim3(256), 0, s, qkv, nh, nkv, hd, cos_t, sin_t,
                          half, row_pos, P, bt, bs, (__half*)kc, (__half*)vc, q_out));
  else
    RET_LAUNCH(launch_pdl(rope_append_kernel<float>, dim3(max_n), dim3(256), 0, s, qkv, nh, nkv, hd, cos_t, sin_t,
                          half, row_pos, P, bt, bs, (float*)kc, (float*)vc, q_out));
  return LUMINA_OK;
}

int launch_dense_gemv(const __half* W, int N, int K, const float* x, int ldx, int batch, float* y, int ldy,
                      const float* resid, int ldr, cudaStream_t s, unsigned long long* amax, const L2Prefetch* pf) {
  const L2Prefetch none;
  if (K % 8) {
    set_error("dense gemv: K=%d must be a multiple of 8", K);
    return LUMINA_E_UNSUPPORTED;
  }
  int done = 0;
  while (done < batch) {
    const int left = batch - done;
    const int nb = left >= 4 ? 4 : (left >= 2 ? 2 : 1);
    const int tasks = (N + 1) / 2;
    const int grid = std::max(1, std::min((tasks + 7) / 8, 4 * sm_count()));
    const float* xp = x + (size_t)done * ldx;
    float* yp = y + (size_t)done * ldy;
    const float* rp = resid ? resid + (size_t)done * ldr : nullptr;
#define DG(NB_, E_) \
  RET_LAUNCH(launch_pdl(dense_gemv_kernel<NB_, E_>, dim3(grid), dim3(256), 0, s, W, N, K, xp, ldx, yp, ldy, rp, ldr, \
                        done == 0 ? amax : nullptr, (done == 0 && pf) ? *pf : none))
    if (resid) {
      if (nb == 4) DG(4, EPI_RESID); else if (nb == 2) DG(2, EPI_RESID); else DG(1, EPI_RESID);
    } else {
      if (nb == 4) DG(4, EPI_STORE); else if (nb == 2) DG(2, EPI_STORE); else DG(1, EPI_STORE);
    }
#undef DG
    done += nb;
  }
  return LUMINA_OK;
}

int launch_swiglu(const float* g, const float* u, float* o, int n, int ffn, int ld, cudaStream_t s) {
  const int grid = std::max(1, std::min((int)(((size_t)n * ffn + 255) / 256), 4 * sm_count()));
  RET_LAUNCH(launch_pdl(swiglu_kernel, dim3(grid), dim3(256), 0, s, g, u, o, n, ffn, ld));
  return LUMINA_OK;
}

int launch_argmax(const float* v, int n, int* out, cudaStream_t s) {
  RET_LAUNCH(launch_pdl(argmax_kernel, dim3(1), dim3(1024), 0, s, v, n, out));
  return LUMINA_OK;
}

int launch_kv_read(bool fp16, const void* kc, const void* vc, const int* bt, int bs, int nh, int nkv, int hd,
                   int start, int n, float* ko, float* vo, cudaStream_t s) {
  const int grid = std::max(1, std::min((int)(((size_t)n * nh * hd + 255) / 256), 4 * sm_count()));
  if (fp16)
    kv_read_kernel<__half><<<grid, 256, 0, s>>>((const __half*)kc, (const __half*)vc, bt, bs, nh, nkv, hd, start, n,
                                                ko, vo);
  else
    kv_read_kernel<float><<<grid, 256, 0, s>>>((const float*)kc, (const float*)vc, bt, bs, nh, nkv, hd, start, n, ko,
                                               vo);
  RET_LAUNCH(cudaGetLastError());
  return LUMINA_OK;
}

int launch_kv_gather(bool fp16, void* kc, void* vc, const int* bt, int bs, int nkv, int hd, int base, const int* src,
                     int n, void* tmp, cudaStream_t s) {
  const int grid = std::max(1, std::min((int)(((size_t)n * nkv * hd + 255) / 256), 4 * sm_count()));
  for (int phase = 0; phase < 2; ++phase) {
    if (fp16)
      kv_gather_kernel<__half><<<grid, 256, 0, s>>>((__half*)kc, (__half*)vc, bt, bs, nkv, hd, base, src, n,
                                                    (__half*)tmp, phase);
    else
      kv_gather_kernel<float><<<grid, 256, 0, s>>>((float*)kc, (float*)vc, bt, bs, nkv, hd, base, src, n,
                                                   (float*)tmp, phase);
    RET_LAUNCH(cudaGetLastError());
  }
  return LUMINA_OK;
}

}  // namespace lumina
