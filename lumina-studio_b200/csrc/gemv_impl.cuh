// Kernel templates of the packed GEMV, instantiated per bit width in
// gemv_b1.cu .. gemv_b4.cu (see gemv.cu for the design notes).
#pragma once
#include <atomic>

#include "weights.cuh"

namespace lumina {


__device__ __forceinline__ int dp2a_lo(uint32_t a, uint32_t b, int c) { return __dp2a_lo((int)a, (int)b, c); }
__device__ __forceinline__ int dp2a_hi(uint32_t a, uint32_t b, int c) { return __dp2a_hi((int)a, (int)b, c); }

// Integer dot of one 32-column block: w = BITS words of codes, x = 16 words
// of permuted int16 activations.
template <int BITS>
__device__ __forceinline__ int block_dot(const uint32_t* w, const uint32_t* x, int d);

template <>
__device__ __forceinline__ int block_dot<4>(const uint32_t* w, const uint32_t* x, int d) {
  int e = 0;  // two accumulators halve the dependent dp2a chain
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t lo = w[i] & 0x0F0F0F0Fu;         // columns 0,2,4,6 of the word
    const uint32_t hi = (w[i] >> 4) & 0x0F0F0F0Fu;  // columns 1,3,5,7
    d = dp2a_lo(x[4 * i + 0], lo, d);
    e = dp2a_hi(x[4 * i + 1], lo, e);
    d = dp2a_lo(x[4 * i + 2], hi, d);
    e = dp2a_hi(x[4 * i + 3], hi, e);
  }
  return d + e;
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
__device__ __forceinline__ float ld_scale(const uint8_t* p) {
  if constexpr (sizeof(ST) == 2) return __half2float(*reinterpret_cast<const __half*>(p));
  else return *reinterpret_cast<const float*>(p);
}

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

template <int BITS>
constexpr int perm_of() { return BITS == 4 ? 8 : (BITS == 1 ? 32 : 16); }

// int16 quantization of one 32-column block held one value per lane.
__device__ __forceinline__ void quant_block(float v, int& q, float& s, int& qs) {
  const float amax = warp_max(fabsf(v));
  q = 0;
  s = 0.f;
  if (amax > 0.f) {
    const float f = __fdiv_rn(32767.f, amax);
    q = __float2int_rn(__fmul_rn(v, f));
    q = max(-32767, min(32767, q));
    s = __fdiv_rn(amax, 32767.f);
  }
  qs = warp_sum_int(q);
}

// ---------------------------------------------------------------------------
// epilogue shared by both kernels: lane-parallel writes of an R x NB tile
// ---------------------------------------------------------------------------
// Values an epilogue can have fetched before the row group's last tile:
// the residual element or the cos/sin pair of this lane's output, and the
// KV page slot and RoPE position of each batch row.
struct EpiPre {
  bool have;           // res / c / s were prefetched for this lane
  float res, c, s;
  const int* kv_blk;   // per batch row (shared memory) or null
  const int* kv_off;
  const int* pos;
};

template <int R, int NB, int EPI>
__device__ __forceinline__ void epilogue(const GemvArgs& a, int row0, float (&acc)[R][NB], int lane,
                                         const EpiPre& pre) {
  const int rows = a.w.rows;
  if constexpr (EPI == EPI_SWIGLU) {
    // rows are interleaved gate/up pairs: row 2i = gate_i, 2i+1 = up_i
    // (chat.py:300-302: silu(g) * u with the +-40 clip)
#pragma unroll
    for (int j = 0; j < R / 2; ++j)
#pragma unroll
      for (int b = 0; b < NB; ++b)
        if (lane == j * NB + b && row0 + 2 * j + 1 < rows) {
          const float gv = acc[2 * j][b], uv = acc[2 * j + 1][b];
          const float e = expf(-fminf(fmaxf(gv, -40.f), 40.f));
          a.y[(size_t)b * a.ldy + (row0 >> 1) + j] = gv / (1.0f + e) * uv;
        }
  } else if constexpr (EPI == EPI_ROPE_KV) {
    // fused q/k/v rows: [q heads (pairs adjacent)][k heads (pairs adjacent)][v]
    const RopeKV& k = a.rk;
    const int qrows = k.nh * k.hd, krows = k.nkv * k.hd, half = k.hd / 2;
#pragma unroll
    for (int j = 0; j < R / 2; ++j)
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (lane != j * NB + b) continue;
        const int row = row0 + 2 * j;
        if (row + 1 >= rows) continue;
        size_t blk, off;
        if (pre.kv_blk) {
          blk = pre.kv_blk[b];
          off = pre.kv_off[b];
        } else {
          const int t = *k.t_prev + k.row_base + b;
          blk = k.block_table[t / k.bs];
          off = t % k.bs;
        }
        if (row < qrows + krows) {
          const bool isq = row < qrows;
          const int rr = isq ? row : row - qrows;
          const int h = rr / k.hd, p = (rr % k.hd) >> 1;
          float c, s;
          if (pre.have) {
            c = pre.c;
            s = pre.s;
          } else {
            const int pos = pre.pos ? pre.pos[b] : k.row_pos[b];
            c = k.cos_t[(size_t)pos * half + p];
            s = k.sin_t[(size_t)pos * half + p];
          }
          const float x1 = acc[2 * j][b], x2 = acc[2 * j + 1][b];
          // rotate-half RoPE, fp32 products rounded separately (chat.py:99-100)
          const float o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
          const float o2 = __fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c));
          if (isq) {
            float* q = k.q_out + (size_t)b * qrows + (size_t)h * k.hd;
            q[p] = o1;
            q[p + half] = o2;
          } else {
            const size_t base = ((blk * k.nkv + h) * k.bs + off) * k.hd;
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
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int rr = row + e - qrows - krows;
            const int h = rr / k.hd, dd = rr % k.hd;
            const size_t idx = ((blk * k.nkv + h) * k.bs + off) * k.hd + dd;
            if (k.kv_fp16) static_cast<__half*>(k.vcache)[idx] = __float2half_rn(acc[2 * j + e][b]);
            else static_cast<float*>(k.vcache)[idx] = acc[2 * j + e][b];
          }
        }
      }
  } else {
    float mine = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int b = 0; b < NB; ++b)
        if (lane == r * NB + b) mine = acc[r][b];
    if (lane < R * NB) {
      const int r = lane / NB, b = lane % NB;
      const int row = row0 + r;
      if (row < rows) {
        float v = mine;
        if constexpr (EPI == EPI_RESID) v = (pre.have ? pre.res : a.resid[(size_t)b * a.ldr + row]) + v;
        a.y[(size_t)b * a.ldy + row] = v;
      }
    }
  }
}

template <int R, int NB, int L>
__device__ __forceinline__ void reduce_tile(float (&acc)[R][NB]) {
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[r][b] = warp_sum(acc[r][b]) / (float)L;
}

// ---------------------------------------------------------------------------
// gemv_kernel: pre-quantized activations in global memory (prefill path)
// ---------------------------------------------------------------------------
constexpr int GEMV_WARPS = 8;

template <int BITS, int R, int U, int NB, typename ST, int EPI>
__global__ void __launch_bounds__(GEMV_WARPS * 32)
gemv_kernel(GemvArgs a) {
  using Lt = Layout<BITS>;
  constexpr int CW = Lt::CHUNK_WORDS;
  constexpr int CB = Lt::CB;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const lumina_weight& w = a.w;
  const int n_tasks = (w.rows + R - 1) / R;
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

    for (int cbase = 0; cbase < w.n_chunks; cbase += 32 * U) {
      uint32_t wv[U][R][CW];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = cbase + u * 32 + lane;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int row = min(row0 + r, w.rows_pad - 1);
          const uint8_t* p = w.codes + code_offset(w, row, min(c, w.n_chunks - 1));
#pragma unroll
          for (int q = 0; q < CW / 4; ++q) {
            uint4 v = make_uint4(0, 0, 0, 0);
            if (c < w.n_chunks) v = ldg_stream(p + 16 * q);
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
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = cbase + u * 32 + lane;
        if (c >= w.n_chunks) continue;
#pragma unroll
        for (int cb = 0; cb < CB; ++cb) {
          const int blk = c * CB + cb;
          const int g = (blk * 32) / w.group;
          float sc[R];
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const int row = min(row0 + r, w.rows_pad - 1);
            sc[r] = ld_scale<ST>(w.scales + scale_offset(w, row, g));
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
              acc[r][b] = fmaf((float)(2 * d - xs), fx * sc[r], acc[r][b]);
            }
          }
        }
      }
    }
    if (!waited) {
      pdl_wait();
      waited = true;
    }
    reduce_tile<R, NB, Lt::L>(acc);
    const EpiPre none{false, 0.f, 0.f, 0.f, nullptr, nullptr, nullptr};
    epilogue<R, NB, EPI>(a, row0, acc, lane, none);
  }
}

// ---------------------------------------------------------------------------
// gemv_fused_kernel: decode path
// ---------------------------------------------------------------------------
// One CTA of FW = 16 warps per SM. A warp owns tasks of R rows (grid-stride) and
// sweeps K in steps of 32*U chunks (lane l takes chunk step*32*U + u*32 + l
// of each row). Code words stream through a per-warp ring of S shared-memory
// stages filled with cp.async (16 bytes per lane, each lane owns its slots):
// S-1 steps are in flight while one is consumed, about 128 KB per SM, which
// is what HBM needs in flight to run near its copy bandwidth on this part.
// The warp's first S-1 steps are requested before griddepcontrol.wait
// (weights never depend on the previous kernel). The scale rows of a task (R
// rows, one contiguous span) are bulk-copied into a per-warp shared buffer
// one task ahead, completion tracked by an mbarrier. The CTA quantizes (and
// RMS-normalizes) the activation rows into shared memory after the wait.
constexpr int FW = 16;
constexpr long MBAR_SPIN_LIMIT = 1L << 24;  // bounded wait (~seconds), then a fault flag

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// false once `limit` polls found the phase still pending (limit 0: at once)
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  long long limit = MBAR_SPIN_LIMIT) {
  for (long long i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
// a whole warp waits for a phase: lane 0 polls and the others wait at the
// shuffle (32 lanes polling one mbarrier word serialize in the shared-memory
// pipe and take issue slots from the warps that have work)
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, long long limit, int lane) {
  int ok = 1;
  if (lane == 0) ok = mbar_wait_bounded(bar, parity, limit) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}
// global -> shared bulk copy (bytes % 16 == 0, both addresses 16-byte aligned)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// the same with an L2 eviction-priority policy (createpolicy) for the source lines
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// lines read once: first to leave L2 (keeps room for the lines prefetched
// for the next kernel)
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool pred) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %2, 0;\n @p cp.async.cg.shared.global [%0], [%1], 16;\n}\n" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"((int)pred)
      : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

struct FusedArgs {
  GemvArgs g;
  const float* x;
  int ldx;
  const float* norm_w;
  float eps;
  int K;
  int n_tasks;     // rows_pad / R
  int x_bytes;     // shared bytes of the quantized activations
  int sbuf_bytes;  // one scale buffer (R * spr)
  int ring_bytes;  // one warp's code ring (S stages)
  int* fault;
  long long spin;  // polls before a wait on a scale copy gives up (wait_spin_limit())
};

template <int BITS, int R, int U, int S, int NB, typename ST, int EPI, bool NORM>
struct FusedCtx {
  using Lt = Layout<BITS>;
  static constexpr int CB = Lt::CB, CHB = Lt::CHUNK_BYTES, CV = Lt::CHUNK_WORDS / 4;  // uint4 per chunk
  static constexpr int STAGE_U4 = U * R * CV * 32;  // uint4 slots of one stage
  const FusedArgs& fa;
  const lumina_weight& w;
  int lane, gw, W, n_it, nch, total;
  const uint4* xs_u;
  const float* sx_s;
  const int* xsum_s;
  uint8_t* sbuf;
  uint64_t* bars;
  uint4* ring;

  __device__ __forceinline__ int task_of(int k) const { return gw + k * W; }

  // this lane's code words of step `st` into stage st % S (one commit group,
  // empty past the last step so group counting stays uniform)
  __device__ __forceinline__ void issue(int st) const {
    if (st < total) {
      const int k = st / n_it, it = st % n_it;
      const int row0 = task_of(k) * R;
      uint4* stage = ring + (size_t)(st % S) * STAGE_U4;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = (it * U + u) * 32 + lane;
        const int cc = c < nch ? c : nch - 1;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const uint8_t* p = w.codes + (size_t)(row0 + r) * w.row_bytes + (size_t)cc * CHB;
#pragma unroll
          for (int q = 0; q < CV; ++q)
            cp_async16(stage + ((u * R + r) * CV + q) * 32 + lane, p + 16 * q, c < nch);
        }
      }
    }
    cp_async_commit();
  }

  // lane 0: scale rows of the warp's k-th task into buffer k & 1
  __device__ __forceinline__ void issue_scales(int k) const {
    const int row0 = task_of(k) * R;
    uint8_t* dst = sbuf + (size_t)(k & 1) * fa.sbuf_bytes;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_expect_tx(&bars[k & 1], (uint32_t)(R * w.spr));
    bulk_g2s(dst, w.scales + (size_t)row0 * w.spr, (uint32_t)(R * w.spr), &bars[k & 1]);
  }

  __device__ __forceinline__ void consume(int st, float (&acc)[R][NB]) const {
    const int k = st / n_it, it = st % n_it;
    const uint8_t* sc_base = sbuf + (size_t)(k & 1) * fa.sbuf_bytes;
    const uint4* stage = ring + (size_t)(st % S) * STAGE_U4;
    constexpr int es = sizeof(ST);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = (it * U + u) * 32 + lane;
      if (c >= nch) continue;
      uint32_t wv[R][4 * CV];
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int q = 0; q < CV; ++q) {
          const uint4 v = stage[((u * R + r) * CV + q) * 32 + lane];
          wv[r][4 * q + 0] = v.x;
          wv[r][4 * q + 1] = v.y;
          wv[r][4 * q + 2] = v.z;
          wv[r][4 * q + 3] = v.w;
        }
#pragma unroll
      for (int cb = 0; cb < CB; ++cb) {
        const int g = ((c * CB + cb) * 32) / w.group;
        float sc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) sc[r] = ld_scale<ST>(sc_base + (size_t)r * w.spr + (size_t)g * es);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          uint32_t xr[16];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 v = xs_u[(size_t)((b * CB + cb) * 4 + q) * nch + c];
            xr[4 * q + 0] = v.x;
            xr[4 * q + 1] = v.y;
            xr[4 * q + 2] = v.z;
            xr[4 * q + 3] = v.w;
          }
          const int xs = xsum_s[(b * CB + cb) * nch + c];
          const float fx = sx_s[(b * CB + cb) * nch + c];
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const int d = block_dot<BITS>(&wv[r][cb * BITS], xr, 0);
            acc[r][b] = fmaf((float)(2 * d - xs), fx * sc[r], acc[r][b]);
          }
        }
      }
    }
  }
};

template <int BITS, int R, int U, int S, int NB, typename ST, int EPI, bool NORM>
__global__ void __launch_bounds__(FW * 32, 1)
gemv_fused_kernel(FusedArgs fa) {
  using Ctx = FusedCtx<BITS, R, U, S, NB, ST, EPI, NORM>;
  using Lt = Layout<BITS>;
  constexpr int CB = Lt::CB, CV = Ctx::CV;
  constexpr int PERM = perm_of<BITS>();
  const GemvArgs& a = fa.g;
  const lumina_weight& w = a.w;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nch = w.n_chunks;
  const int nblk_pad = nch * CB;

  extern __shared__ __align__(128) uint8_t smem[];
  // [x int16 units: NB x CB x 4 x nch x 16B][sx: NB x CB x nch][xsum: same]
  // [code rings: FW x ring_bytes][scale buffers: FW x 2 x sbuf_bytes][mbarriers: FW x 2]
  uint4* xs_u = reinterpret_cast<uint4*>(smem);
  float* sx_s = reinterpret_cast<float*>(smem + (size_t)NB * nblk_pad * 64);
  int* xsum_s = reinterpret_cast<int*>(sx_s + NB * nblk_pad);
  uint8_t* rings = smem + fa.x_bytes;
  uint8_t* sbufs = rings + (size_t)FW * fa.ring_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sbufs + (size_t)FW * 2 * fa.sbuf_bytes) + warp * 2;
  __shared__ float red[FW];
  __shared__ int ep_blk[4], ep_off[4], ep_pos[4];

  Ctx cx{fa, w, lane, (int)(blockIdx.x * FW + warp), (int)(gridDim.x * FW), 0, nch, 0, xs_u, sx_s, xsum_s,
         sbufs + (size_t)warp * 2 * fa.sbuf_bytes, bars,
         reinterpret_cast<uint4*>(rings + (size_t)warp * fa.ring_bytes)};
  cx.n_it = (nch + 32 * U - 1) / (32 * U);
  const int my_tasks = cx.gw < fa.n_tasks ? (fa.n_tasks - cx.gw + cx.W - 1) / cx.W : 0;
  const int total = my_tasks * cx.n_it;
  cx.total = total;

  if (lane == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();

  // 1) the first S-1 steps' code words and the first task's scales go out
  //    before the wait on the previous kernel
#pragma unroll
  for (int i = 0; i < S - 1; ++i) cx.issue(i);
  if (total > 0 && lane == 0) cx.issue_scales(0);
  pdl_launch_dependents();
  pdl_wait();

  // 2) quantize (and normalize) the activation rows into shared memory: one
  //    thread per 32-column block, x and the norm weights loaded in one burst
  if constexpr (EPI == EPI_ROPE_KV) {
    if (threadIdx.x < NB) {
      const int t = *a.rk.t_prev + a.rk.row_base + threadIdx.x;
      ep_blk[threadIdx.x] = a.rk.block_table[t / a.rk.bs];
      ep_off[threadIdx.x] = t % a.rk.bs;
      ep_pos[threadIdx.x] = a.rk.row_pos[threadIdx.x];
    }
  }
  // two adjacent threads per 32-column block, 16 values each
  const bool vec_ok = ((fa.ldx & 3) == 0) && ((reinterpret_cast<uintptr_t>(fa.x) & 15) == 0);
  const int half_id = threadIdx.x & 1;
  for (int b = 0; b < NB; ++b) {
    const float* xr = fa.x + (size_t)b * fa.ldx;
    for (int blk0 = 0; blk0 < nblk_pad; blk0 += blockDim.x / 2) {
      const int blk = blk0 + (threadIdx.x >> 1);
      const bool mine = blk < nblk_pad;
      float v[16], wn[16];
      const int k0 = blk * 32 + 16 * half_id;
      if (mine && vec_ok && k0 + 16 <= fa.K) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 t = *reinterpret_cast<const float4*>(xr + k0 + 4 * q);
          v[4 * q] = t.x; v[4 * q + 1] = t.y; v[4 * q + 2] = t.z; v[4 * q + 3] = t.w;
          if constexpr (NORM) {
            const float4 u = __ldg(reinterpret_cast<const float4*>(fa.norm_w + k0 + 4 * q));
            wn[4 * q] = u.x; wn[4 * q + 1] = u.y; wn[4 * q + 2] = u.z; wn[4 * q + 3] = u.w;
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const bool in = mine && k0 + j < fa.K;
          v[j] = in ? xr[k0 + j] : 0.f;
          if constexpr (NORM) wn[j] = in ? fa.norm_w[k0 + j] : 0.f;
        }
      }
      float rinv = 1.f;
      if constexpr (NORM) {
        // chat.py:63-66: x / sqrt(mean(x^2) + eps) * w (fp32); the whole row
        // is in this pass (dispatch requires 2 * nblk_pad <= blockDim.x)
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) ss = fmaf(v[j], v[j], ss);
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int i = 0; i < FW; ++i) tot += red[i];
        rinv = 1.0f / sqrtf(tot / (float)fa.K + fa.eps);
        __syncthreads();
      }
      float amax = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if constexpr (NORM) v[j] = (v[j] * rinv) * wn[j];
        amax = fmaxf(amax, fabsf(v[j]));
      }
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));  // the block's two halves
      uint32_t packed[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) packed[j] = 0u;
      int qs = 0;
      float sxv = 0.f;
      if (amax > 0.f) {
        const float f = __fdiv_rn(32767.f, amax);
        sxv = __fdiv_rn(amax, 32767.f);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if ((j >> 4) != half_id) continue;
          int q = __float2int_rn(__fmul_rn(v[j & 15], f));
          q = max(-32767, min(32767, q));
          qs += q;
          const int slot = perm_slot<PERM>(j);
          packed[slot >> 1] |= ((uint32_t)q & 0xFFFFu) << (16 * (slot & 1));
        }
      }
      // merge the two halves' packed words and sums (disjoint bits)
#pragma unroll
      for (int j = 0; j < 16; ++j) packed[j] |= __shfl_xor_sync(0xffffffffu, packed[j], 1);
      qs += __shfl_xor_sync(0xffffffffu, qs, 1);
      if (!mine) continue;
      const int c = blk / CB, cb = blk % CB;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int uu = 2 * half_id + u;
        xs_u[(size_t)((b * CB + cb) * 4 + uu) * nch + c] =
            make_uint4(packed[4 * uu], packed[4 * uu + 1], packed[4 * uu + 2], packed[4 * uu + 3]);
      }
      if (half_id == 0) {
        sx_s[(b * CB + cb) * nch + c] = sxv;
        xsum_s[(b * CB + cb) * nch + c] = Lt::L * qs;
      }
    }
  }
  __syncthreads();

  // 3) pipelined sweep: loads of step s+1 in flight while step s is consumed
  float acc[R][NB];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[r][b] = 0.f;
  EpiPre pre{false, 0.f, 0.f, 0.f, nullptr, nullptr, nullptr};
  if constexpr (EPI == EPI_ROPE_KV) {
    pre.kv_blk = ep_blk;
    pre.kv_off = ep_off;
    pre.pos = ep_pos;
  }
  int failed = -1;  // the task whose scale copy a wait gave up on
  for (int st = 0; st < total; ++st) {
    const int k = st / cx.n_it, it = st % cx.n_it;
    cx.issue(st + S - 1);  // refill the stage consumed last step
    if (it == 0) {
      if (lane == 0 && k + 1 < my_tasks) cx.issue_scales(k + 1);
      if (!mbar_wait_warp(&bars[k & 1], (uint32_t)((k >> 1) & 1), fa.spin, lane)) {
        failed = k;
        break;
      }
      const int row0 = cx.task_of(k) * R;
      pre.have = false;
      if constexpr (EPI == EPI_RESID) {
        if (lane < R * NB && row0 + lane / NB < w.rows) {
          pre.res = a.resid[(size_t)(lane % NB) * a.ldr + row0 + lane / NB];
          pre.have = true;
        }
      } else if constexpr (EPI == EPI_ROPE_KV) {
        const int qk = (a.rk.nh + a.rk.nkv) * a.rk.hd;
        const int row = row0 + 2 * (lane / NB);
        if (lane < (R / 2) * NB && row < qk) {
          const int rr = row < a.rk.nh * a.rk.hd ? row : row - a.rk.nh * a.rk.hd;
          const int p = (rr % a.rk.hd) >> 1, half = a.rk.hd / 2;
          const int pos = ep_pos[lane % NB];
          pre.c = a.rk.cos_t[(size_t)pos * half + p];
          pre.s = a.rk.sin_t[(size_t)pos * half + p];
          pre.have = true;
        }
      }
    }
    cp_async_wait<S - 1>();  // this lane's copies of step st have landed
    cx.consume(st, acc);
    if (it == cx.n_it - 1) {
      reduce_tile<R, NB, Lt::L>(acc);
      epilogue<R, NB, EPI>(a, cx.task_of(k) * R, acc, lane, pre);
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[r][b] = 0.f;
      __syncwarp();  // every lane is done with this task's scale buffer
    }
  }
  cp_async_wait<0>();
  if (failed >= 0) {
    // a scale copy did not land in time: record it, and let this warp's
    // scale copies still in flight (tasks `failed` and, if it was issued,
    // `failed` + 1, each on its own buffer and phase) land, waiting with the
    // full limit, before the CTA's shared memory is released
    if (lane == 0) {
      atomicOr(fa.fault, 1);
      for (int k = failed; k < failed + 2 && k < my_tasks; ++k)
        mbar_wait_bounded(&bars[k & 1], (uint32_t)((k >> 1) & 1));
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// launch dispatch
// ---------------------------------------------------------------------------
template <int BITS, int R, int U, int NB, typename ST, int EPI>
inline int launch_one(const GemvArgs& a, cudaStream_t s) {
  auto kern = gemv_kernel<BITS, R, U, NB, ST, EPI>;
  // resident CTAs per SM, per device (atomics: racing host threads store
  // the same value)
  static std::atomic<int> per_sm_dev[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  std::atomic<int>& slot = per_sm_dev[dev >= 0 && dev < 64 ? dev : 0];
  int per_sm = slot.load(std::memory_order_relaxed);
  if (per_sm < 1) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, GEMV_WARPS * 32, 0) != cudaSuccess ||
        per_sm < 1) {
      cudaGetLastError();
      per_sm = 1;
    }
    slot.store(per_sm, std::memory_order_relaxed);
  }
  const int n_tasks = (a.w.rows + R - 1) / R;
  int grid = (n_tasks + GEMV_WARPS - 1) / GEMV_WARPS;
  grid = std::max(1, std::min(grid, per_sm * sm_count()));
  cudaError_t e = launch_pdl(kern, dim3(grid), dim3(GEMV_WARPS * 32), 0, s, a);
  if (e != cudaSuccess) {
    set_error("gemv launch: %s", cudaGetErrorString(e));
    return LUMINA_E_CUDA;
  }
  return LUMINA_OK;
}

template <int BITS, typename ST, int EPI>
inline int dispatch_nb(const GemvArgs& a, int nb, cudaStream_t s) {
  constexpr int RR = (BITS == 3) ? 2 : 4;  // whole tiles, even for the paired epilogues
  switch (nb) {
    case 1: return launch_one<BITS, RR, 2, 1, ST, EPI>(a, s);
    case 2: return launch_one<BITS, RR, 2, 2, ST, EPI>(a, s);
    case 4: return launch_one<BITS, RR, 2, 4, ST, EPI>(a, s);
    case 8: return launch_one<BITS, RR, 1, 8, ST, EPI>(a, s);
  }
  set_error("gemv: unsupported batch tile %d", nb);
  return LUMINA_E_UNSUPPORTED;
}

template <int BITS>
inline int dispatch_bits(const GemvArgs& a, int nb, int fp16, int epi, cudaStream_t s) {
#define DB(ST)                                                                   \
  switch (epi) {                                                                 \
    case EPI_STORE: return dispatch_nb<BITS, ST, EPI_STORE>(a, nb, s);           \
    case EPI_RESID: return dispatch_nb<BITS, ST, EPI_RESID>(a, nb, s);           \
    case EPI_SWIGLU: return dispatch_nb<BITS, ST, EPI_SWIGLU>(a, nb, s);         \
    default: return dispatch_nb<BITS, ST, EPI_ROPE_KV>(a, nb, s);                \
  }
  if (fp16) {
    DB(__half)
  } else {
    DB(float)
  }
#undef DB
}

template <int BITS, int R, int U, int S, int NB, typename ST, int EPI, bool NORM>
inline int launch_fused(const FusedArgs& fa, size_t smem, cudaStream_t s) {
  auto kern = gemv_fused_kernel<BITS, R, U, S, NB, ST, EPI, NORM>;
  const int rc = set_smem_limit((const void*)kern, smem, "gemv_fused");
  if (rc) return rc;
  const int grid = std::max(1, std::min(sm_count(), (fa.n_tasks + FW - 1) / FW));
  const cudaError_t e = launch_pdl(kern, dim3(grid), dim3(FW * 32), smem, s, fa);
  if (e != cudaSuccess) {
    set_error("gemv_fused launch: %s", cudaGetErrorString(e));
    return LUMINA_E_CUDA;
  }
  return LUMINA_OK;
}

// R rows per task (even for the paired epilogues), U chunks per lane per
// step, S = 3 ring stages (two in flight per warp): a stage is U*R*32 chunks,
// 4 KB for int4 at U=4, R=2. Returns LUMINA_E_UNSUPPORTED when the shared
// memory does not fit.
template <int BITS, int R, int U, int NB, typename ST, int EPI, bool NORM>
inline int fused_try(FusedArgs& fa, const lumina_weight* w, cudaStream_t s) {
  constexpr int S = 3;
  const int nblk_pad = w->n_chunks * Layout<BITS>::CB;
  if (NORM && 2 * nblk_pad > FW * 32) return LUMINA_E_UNSUPPORTED;  // one-pass row norm
  fa.sbuf_bytes = (R * w->spr + 127) / 128 * 128;
  fa.x_bytes = (NB * nblk_pad * (64 + 8) + 127) / 128 * 128;
  fa.ring_bytes = S * U * R * Layout<BITS>::CHUNK_BYTES * 32;
  fa.n_tasks = w->rows_pad / R;
  const size_t smem =
      (size_t)fa.x_bytes + (size_t)FW * fa.ring_bytes + (size_t)FW * 2 * fa.sbuf_bytes + FW * 2 * 8;
  if (smem > 227 * 1024 - 1024) return LUMINA_E_UNSUPPORTED;
  return launch_fused<BITS, R, U, S, NB, ST, EPI, NORM>(fa, smem, s);
}

template <int BITS, int NB, typename ST, int EPI, bool NORM>
inline int fused_rs(FusedArgs& fa, const lumina_weight* w, cudaStream_t s) {
  constexpr bool paired = EPI == EPI_SWIGLU || EPI == EPI_ROPE_KV;
  constexpr int R = paired ? 2 : (NB >= 4 ? 1 : 2);
  if constexpr (BITS == 3) {
    return fused_try<BITS, R, 1, NB, ST, EPI, NORM>(fa, w, s);
  } else if constexpr (NB == 1) {
    const int rc = fused_try<BITS, R, 4, NB, ST, EPI, NORM>(fa, w, s);
    if (rc != LUMINA_E_UNSUPPORTED) return rc;
    return fused_try<BITS, R, 2, NB, ST, EPI, NORM>(fa, w, s);
  } else {
    return fused_try<BITS, R, 2, NB, ST, EPI, NORM>(fa, w, s);
  }
}

template <int BITS, typename ST, int EPI, bool NORM>
inline int fused_nb(FusedArgs& fa, const lumina_weight* w, int nb, cudaStream_t s) {
  switch (nb) {
    case 1: return fused_rs<BITS, 1, ST, EPI, NORM>(fa, w, s);
    case 2: return fused_rs<BITS, 2, ST, EPI, NORM>(fa, w, s);
    case 4: return fused_rs<BITS, 4, ST, EPI, NORM>(fa, w, s);
  }
  return LUMINA_E_UNSUPPORTED;
}

template <int BITS, typename ST>
inline int fused_epi(FusedArgs& fa, const lumina_weight* w, int nb, int epi, bool norm, cudaStream_t s) {
  // the combinations the decoder uses: normalized inputs feed q/k/v and
  // gate/up, raw inputs feed o and down (and the plain GEMV entry)
  switch (epi) {
    case EPI_STORE:
      return norm ? fused_nb<BITS, ST, EPI_STORE, true>(fa, w, nb, s) : fused_nb<BITS, ST, EPI_STORE, false>(fa, w, nb, s);
    case EPI_RESID:
      return norm ? LUMINA_E_UNSUPPORTED : fused_nb<BITS, ST, EPI_RESID, false>(fa, w, nb, s);
    case EPI_SWIGLU:
      return norm ? fused_nb<BITS, ST, EPI_SWIGLU, true>(fa, w, nb, s) : LUMINA_E_UNSUPPORTED;
    default:
      return norm ? fused_nb<BITS, ST, EPI_ROPE_KV, true>(fa, w, nb, s) : LUMINA_E_UNSUPPORTED;
  }
}


// per-bit entry points (defined in gemv_bN.cu)
template <int BITS>
int gemv_bits(const GemvArgs& a, int nb, int fp16, int epi, cudaStream_t s) {
  return dispatch_bits<BITS>(a, nb, fp16, epi, s);
}

template <int BITS>
int gemv_fused_bits(FusedArgs& fa, const lumina_weight* w, int nb, int epi, bool norm, cudaStream_t s) {
  return w->fp16_scales ? fused_epi<BITS, __half>(fa, w, nb, epi, norm, s) : fused_epi<BITS, float>(fa, w, nb, epi, norm, s);
}

}  // namespace lumina
