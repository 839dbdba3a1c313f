// One decode step (batch 1) as a single persistent kernel.
//
// Why: a decode step of the multi-kernel path is 163 launches, and every
// GEMV launch pays a fixed cost of about 2 us (its first weight bytes arrive
// a DRAM latency after its CTAs become resident, and they become resident
// only when the previous kernel's CTAs leave the SM). Weights never depend on
// activations, so here each warp's shared-memory ring is fed continuously
// across all 128 GEMVs of the step while the activations flow through the
// phases behind it.
//
// Layout: one 512-thread CTA per SM (cooperative launch: all CTAs are
// resident, which the dataflow waits below rely on). Each warp consumes one
// stream of units through its ring of shared-memory stages (filled by lane 0
// with cp.async.bulk, completion on an mbarrier per stage); per layer:
//   qkv GEMV units (RMSNorm prologue; RoPE + paged KV append epilogue)
//   attention units: MK_AK consecutive keys of one head (their K and V rows
//     are contiguous within a KV page, so a unit is at most four copies);
//     they stream in while the qkv GEMV runs, since only the new row depends
//     on it (that row is re-read after the wait and patched in)
//   o GEMV units (residual), gate/up (RMSNorm; SwiGLU), down (residual)
// then the fp16 LM head with the argmax fused and, for greedy chains, the
// commit of the next token (as greedy_commit_kernel). The GEMV units are the
// arithmetic of gemv_tc.cu (64-column int16 activation blocks split into two
// signed bytes, mma.sync u8 x s8, whole 16-row tiles per CTA, in-CTA
// deterministic combine). Attention keeps an online softmax per warp over its
// units (lanes along the head dimension); the warp that completes a head's
// key count merges the warps' partial states in key order.
//
// Synchronization is dataflow, not barriers: a producer publishes each
// finished tile / head with a release increment of a counter; a consumer
// waits (acquire loads, bounded) until the counter reaches the count it
// needs. The dependency order is acyclic and every CTA runs the phases in
// order, so with all CTAs resident every wait ends. A wait that gives up sets
// the fault word and an abort flag that ends every other wait; each warp then
// lets its copies in flight land before the CTA exits.
#include "gemv_impl.cuh"
#include "model.cuh"
#include "tc_act.cuh"

namespace lumina {

namespace {

constexpr int MK_TW = 16;           // warps per CTA
constexpr int MK_TS = 3;            // ring stages per warp
constexpr int MK_KS = 7;            // 64-column pairs per GEMV unit
constexpr int MK_AK = 7;            // keys per attention unit
constexpr int MK_ROWB = 256;        // K/V row bytes (head_dim x element size)
constexpr int MK_STAGE = 3840;      // max(7 x 512 B codes + 7 x 32 B scales, 7 keys x 2 x 256 B), 128-aligned
constexpr long MK_SPIN = 1L << 22;  // bounded dataflow waits (with nanosleep)

struct MkWeight {
  const uint8_t* codes;
  const uint8_t* scales;
};
struct MkLayer {
  MkWeight w[4];  // qkv, o, gate/up, down
  const float* in_norm;
  const float* post_norm;
};

// sync words: [0] abort, [1] embed CTAs, [2] head CTAs,
// [4 + 4l + k] CTAs done with GEMV k of layer l, [4 + 4L + l] heads done,
// [4 + 5L + l*nh + h] key splits done of head h
struct MkArgs {
  const MkLayer* layers;
  int n_layer, d, nh, nkv, hd, ffn;
  float eps, sdiv;
  int rows[4], cols[4], T16[4], P[4], ng[4], UT[4], per[4], G[4];
  float* x;
  float* q_buf;
  float* attn;
  float* ffn_buf;
  void* kpool;
  void* vpool;
  size_t layer_elems;
  int kv_fp16;
  const int* bt;
  int bs;
  const float* cos_t;
  const float* sin_t;
  DevParams* Pd;
  int* rowpos;
  int* tokens;
  const __half* embed;
  int embed_rows;
  const __half* head;
  int vocab;
  float* logits;
  unsigned long long* amax_key;
  int greedy;
  int* chain_tokens;
  int* chain_count;
  int max_splits;
  float* part_o;   // [nh][cmax][hd] attention partial outputs (per warp range)
  float* part_ml;  // [nh][cmax][2] their (max, sum)
  int cmax;        // attention units per head at the longest context
  unsigned int* sync;
  int* fault;
  int Pmax;
  int off_fq, off_cnt, off_part, off_ring, off_bars;
};

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// thread 0 of the CTA: wait until *c >= target; false on abort / give-up
__device__ bool mk_wait(const MkArgs& a, const unsigned* c, unsigned target) {
  for (long i = 0; i < MK_SPIN; ++i) {
    if (ld_acquire(c) >= target) return true;
    if (ld_acquire(a.sync) != 0u) return false;
    __nanosleep(200);
  }
  atomicOr(a.fault, 4);
  atomicExch(a.sync, 1u);
  return false;
}

// whole CTA: wait on a counter, true when the CTA may go on
__device__ bool cta_wait(const MkArgs& a, const unsigned* c, unsigned target, int* flag) {
  __syncthreads();
  if (threadIdx.x == 0) *flag = mk_wait(a, c, target) ? 1 : 0;
  __syncthreads();
  return *flag != 0;
}

__device__ __forceinline__ void mma_first(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  const int z = 0;
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(z));
}
__device__ __forceinline__ void mma_acc(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <typename KT>
__global__ void __launch_bounds__(MK_TW * 32, 1) decode_mk_kernel(MkArgs a) {
  constexpr int ES = sizeof(KT), HD = MK_ROWB / ES, DPL = HD / 32;  // head dims per lane
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int L = a.n_layer;
  const unsigned b = blockIdx.x, G = gridDim.x;
  extern __shared__ __align__(128) uint8_t smem[];
  uint4* xb = reinterpret_cast<uint4*>(smem);  // [Pmax][2 columns][4 lanes] x 16 B
  int2* fq = reinterpret_cast<int2*>(smem + a.off_fq);
  int* cnt_s = reinterpret_cast<int*>(smem + a.off_cnt);
  float* part_s = reinterpret_cast<float*>(smem + a.off_part);
  uint8_t* ring = smem + a.off_ring + (size_t)warp * MK_TS * MK_STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.off_bars) + warp * MK_TS;
  __shared__ float red[MK_TW];
  __shared__ int ep_blk, ep_off, ep_pos, go_flag, last_flag;

  const int T = a.Pd->t_tot, t_prev = a.Pd->t_prev;
  unsigned* done = a.sync + 4;
  unsigned* heads_done = a.sync + 4 + 4 * L;
  unsigned* att_cnt = a.sync + 4 + 5 * L;

  // this warp's unit runs: GEMV k (the same in every layer) and attention
  int wu0[4], wu1[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    wu0[k] = wu1[k] = 0;
    if ((int)b < a.G[k]) {
      const int ct0 = ((int)b * a.T16[k]) / a.G[k], ct1 = (((int)b + 1) * a.T16[k]) / a.G[k];
      const int cu0 = ct0 * a.UT[k], nU = (ct1 - ct0) * a.UT[k];
      wu0[k] = cu0 + ((warp * nU) >> 4);
      wu1[k] = cu0 + (((warp + 1) * nU) >> 4);
    }
  }
  // attention: units of MK_AK keys; a head's C units are cut into S key
  // splits, and task (head h, split s) = h * S + s runs on CTA b = task mod G,
  // its units shared by the CTA's warps in contiguous runs
  const int C = (T + MK_AK - 1) / MK_AK;
  const int S = max(1, min((int)G / a.nh, C));
  const int NT = a.nh * S;
  auto task_units = [&](int tau, int& h, int& u0, int& u1) {  // this warp's run of task tau
    h = tau / S;
    const int sp = tau - h * S, c0 = (sp * C) / S, n = ((sp + 1) * C) / S - c0;
    u0 = c0 + ((warp * n) >> 4);
    u1 = c0 + (((warp + 1) * n) >> 4);
  };
  int n_att = 0;
  for (int tau = (int)b; tau < NT; tau += (int)G) {
    int h, u0, u1;
    task_units(tau, h, u0, u1);
    n_att += u1 - u0;
  }
  auto run_len = [&](int ph) {  // stream phases: 0 qkv, 1 attention, 2 o, 3 gate/up, 4 down
    return ph == 1 ? n_att : (ph == 0 ? wu1[0] - wu0[0] : wu1[ph - 1] - wu0[ph - 1]);
  };

  // ---- the unit stream: issue cursor (lane 0) ------------------------------
  int is_l = 0, is_ph = 0, is_j = 0;
  unsigned issued = 0;
  auto issue_next = [&]() {  // lane 0 only
    while (is_l < L && is_j >= run_len(is_ph)) {
      is_j = 0;
      if (++is_ph == 5) {
        is_ph = 0;
        ++is_l;
      }
    }
    if (is_l >= L) return;
    const int slot = issued % MK_TS;
    uint8_t* st = ring + (size_t)slot * MK_STAGE;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (is_ph == 1) {
      // keys k0 .. k0+n-1 of head h: K rows then V rows, one or two page segments
      int h = 0, c = 0;
      for (int tau = (int)b, j = is_j; tau < NT; tau += (int)G) {
        int u0, u1;
        task_units(tau, h, u0, u1);
        if (j < u1 - u0) {
          c = u0 + j;
          break;
        }
        j -= u1 - u0;
      }
      const int k0 = c * MK_AK, n = min(MK_AK, T - k0);
      const int kvh = h / (a.nh / a.nkv);
      const uint8_t* kb = reinterpret_cast<const uint8_t*>(a.kpool) + (size_t)is_l * a.layer_elems * ES;
      const uint8_t* vb = reinterpret_cast<const uint8_t*>(a.vpool) + (size_t)is_l * a.layer_elems * ES;
      mbar_expect_tx(&bars[slot], (uint32_t)n * 2u * MK_ROWB);
      int done_rows = 0;
      while (done_rows < n) {
        const int key = k0 + done_rows, off = key % a.bs;
        const int seg = min(n - done_rows, a.bs - off);
        const size_t src = (((size_t)a.bt[key / a.bs] * a.nkv + kvh) * a.bs + off) * MK_ROWB;
        bulk_g2s(st + done_rows * MK_ROWB, kb + src, (uint32_t)seg * MK_ROWB, &bars[slot]);
        bulk_g2s(st + (MK_AK + done_rows) * MK_ROWB, vb + src, (uint32_t)seg * MK_ROWB, &bars[slot]);
        done_rows += seg;
      }
    } else {
      const int k = is_ph == 0 ? 0 : is_ph - 1, u = wu0[k] + is_j;
      const int tile = u / a.UT[k], p0 = (u - tile * a.UT[k]) * MK_KS, np = min(a.P[k] - p0, MK_KS);
      const MkWeight& w = a.layers[is_l].w[k];
      const uint32_t cb = (uint32_t)np * 512u, sb = (uint32_t)np * 32u;
      mbar_expect_tx(&bars[slot], cb + sb);
      bulk_g2s(st, w.codes + ((size_t)tile * a.P[k] + p0) * 512, cb, &bars[slot]);
      bulk_g2s(st + MK_KS * 512, w.scales + ((size_t)tile * a.ng[k] + p0) * 32, sb, &bars[slot]);
    }
    ++issued;
    ++is_j;
  };
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < MK_TS; ++i) mbar_init(&bars[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int i = 0; i < MK_TS; ++i) issue_next();
  }
  __syncwarp();
  unsigned consumed = 0;
  bool ok = true;  // CTA-uniform: cleared only by a failed CTA-wide wait
  bool warp_ok = true;
  // next ring slot of this warp; false (with the abort raised) if it never lands
  auto take = [&](const uint8_t*& st) -> bool {
    const unsigned slot = consumed % MK_TS;
    const bool landed = mbar_wait_bounded(&bars[slot], (consumed / MK_TS) & 1u);
    if (!__all_sync(0xffffffffu, landed)) {
      if (lane == 0) {
        atomicOr(a.fault, 2);
        atomicExch(a.sync, 1u);
      }
      return false;
    }
    st = ring + (size_t)slot * MK_STAGE;
    return true;
  };
  auto release = [&]() {  // done with the slot: refill it with the next unit
    __syncwarp();
    ++consumed;
    if (lane == 0) issue_next();
  };

  // ---- embed: x = E[token] (chat.py:321), argmax key reset ----------------
  {
    if (b == 0 && tid == 0) *a.amax_key = 0ull;
    int tok = a.tokens[0];
    tok = tok < 0 ? 0 : (tok >= a.embed_rows ? a.embed_rows - 1 : tok);
    const __half* row = a.embed + (size_t)tok * a.d;
    for (int k = ((int)b * blockDim.x + tid) * 2; k < a.d; k += G * blockDim.x * 2) {
      const float2 v = __half22float2(*reinterpret_cast<const __half2*>(row + k));
      a.x[k] = v.x;
      a.x[k + 1] = v.y;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) red_release(a.sync + 1, 1u);
  }

  // the new row's page, offset and RoPE position (the same in every layer)
  if (tid == 0) {
    ep_blk = a.bt[t_prev / a.bs];
    ep_off = t_prev % a.bs;
    ep_pos = a.rowpos[0];
  }
  for (int l = 0; l < L && ok; ++l) {
    const MkLayer& Ly = a.layers[l];
    for (int ph = 0; ph < 5 && ok; ++ph) {
      if (ph == 1) {
        // ---- attention tasks of this CTA (chat.py:264-281, one new row) ----
        if ((int)b >= NT) continue;
        // every qkv CTA is done (one waiting thread per CTA)
        if (!cta_wait(a, done + 4 * l, (unsigned)a.G[0], &go_flag)) {
          ok = false;
          break;
        }
        for (int tau = (int)b; tau < NT; tau += (int)G) {
          int h, u0, u1;
          task_units(tau, h, u0, u1);
          float m = -INFINITY, lsum = 0.f, o[DPL], qv[DPL];
#pragma unroll
          for (int i = 0; i < DPL; ++i) {
            o[i] = 0.f;
            qv[i] = a.q_buf[(size_t)h * HD + lane * DPL + i];
          }
          for (int c = u0; c < u1 && warp_ok; ++c) {
            const int k0 = c * MK_AK, n = min(MK_AK, T - k0);
            const uint8_t* st;
            if (!take(st)) {
              warp_ok = false;
              break;
            }
            // the new row (t_prev) was written by the qkv epilogue after the
            // stage was requested: patch it in from global memory
            if (t_prev >= k0 && t_prev < k0 + n) {
              const int jn = t_prev - k0;
              const size_t src = (((size_t)a.bt[t_prev / a.bs] * a.nkv + h / (a.nh / a.nkv)) * a.bs + t_prev % a.bs) *
                                 MK_ROWB;
              const uint8_t* kb = reinterpret_cast<const uint8_t*>(a.kpool) + (size_t)l * a.layer_elems * ES;
              const uint8_t* vb = reinterpret_cast<const uint8_t*>(a.vpool) + (size_t)l * a.layer_elems * ES;
              const uint2 kn = __ldcg(reinterpret_cast<const uint2*>(kb + src) + lane);
              const uint2 vn = __ldcg(reinterpret_cast<const uint2*>(vb + src) + lane);
              reinterpret_cast<uint2*>(const_cast<uint8_t*>(st) + jn * MK_ROWB)[lane] = kn;
              reinterpret_cast<uint2*>(const_cast<uint8_t*>(st) + (MK_AK + jn) * MK_ROWB)[lane] = vn;
              __syncwarp();
            }
            float sc[MK_AK];
            float mc = -INFINITY;
#pragma unroll
            for (int jj = 0; jj < MK_AK; ++jj) {
              sc[jj] = -INFINITY;
              if (jj < n) {
                const uint2 kw = reinterpret_cast<const uint2*>(st + jj * MK_ROWB)[lane];
                float d;
                if constexpr (ES == 2) {
                  const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&kw.x));
                  const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&kw.y));
                  d = qv[0] * f0.x;
                  d = fmaf(qv[1], f0.y, d);
                  d = fmaf(qv[2], f1.x, d);
                  d = fmaf(qv[3], f1.y, d);
                } else {
                  d = qv[0] * __uint_as_float(kw.x);
                  d = fmaf(qv[1], __uint_as_float(kw.y), d);
                }
                d = warp_sum(d);
                sc[jj] = __fdiv_rn(d, a.sdiv);
                mc = fmaxf(mc, sc[jj]);
              }
            }
            const float m_new = fmaxf(m, mc);
            const float alpha = m == -INFINITY ? 0.f : expf(m - m_new);
            lsum *= alpha;
#pragma unroll
            for (int i = 0; i < DPL; ++i) o[i] *= alpha;
#pragma unroll
            for (int jj = 0; jj < MK_AK; ++jj) {
              if (jj < n) {
                const float p = expf(sc[jj] - m_new);
                lsum += p;
                const uint2 vw = reinterpret_cast<const uint2*>(st + (MK_AK + jj) * MK_ROWB)[lane];
                if constexpr (ES == 2) {
                  const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&vw.x));
                  const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&vw.y));
                  o[0] = fmaf(p, f0.x, o[0]);
                  o[1] = fmaf(p, f0.y, o[1]);
                  o[2] = fmaf(p, f1.x, o[2]);
                  o[3] = fmaf(p, f1.y, o[3]);
                } else {
                  o[0] = fmaf(p, __uint_as_float(vw.x), o[0]);
                  o[1] = fmaf(p, __uint_as_float(vw.y), o[1]);
                }
              }
            }
            m = m_new;
            release();
          }
          // warp partials -> shared memory (the B-fragment area, idle between
          // the qkv and o GEMVs); warp 0 merges them in warp order
          float* pa = reinterpret_cast<float*>(smem) + warp * (HD + 2);
#pragma unroll
          for (int i = 0; i < DPL; ++i) pa[lane * DPL + i] = o[i];
          if (lane == 0) {
            pa[HD] = m;
            pa[HD + 1] = lsum;
          }
          __syncthreads();
          if (warp == 0) {
            const float* pb = reinterpret_cast<const float*>(smem);
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < MK_TW; ++w) M = fmaxf(M, pb[w * (HD + 2) + HD]);
            float Ls = 0.f, acc[DPL];
#pragma unroll
            for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
#pragma unroll
            for (int w = 0; w < MK_TW; ++w) {
              const float* q = pb + w * (HD + 2);
              const float wgt = expf(q[HD] - M);  // 0 for a warp without keys
              Ls = fmaf(wgt, q[HD + 1], Ls);
#pragma unroll
              for (int i = 0; i < DPL; ++i) acc[i] = fmaf(wgt, q[lane * DPL + i], acc[i]);
            }
            bool last = true;
            if (S > 1) {
              // split partial -> global; the last split of the head merges all S
              const int sp = tau - h * S;
              const size_t pi = (size_t)h * S + sp;
#pragma unroll
              for (int i = 0; i < DPL; ++i) a.part_o[pi * HD + lane * DPL + i] = acc[i];
              if (lane == 0) {
                a.part_ml[pi * 2] = M;
                a.part_ml[pi * 2 + 1] = Ls;
              }
              __threadfence();
              __syncwarp();
              unsigned old = 0;
              if (lane == 0) old = atomicAdd(att_cnt + (size_t)l * a.nh + h, 1u);
              old = __shfl_sync(0xffffffffu, old, 0);
              last = old + 1u == (unsigned)S;
              if (last) {
                __threadfence();
                const size_t p0 = (size_t)h * S;
                M = -INFINITY;
                for (int q = 0; q < S; ++q) M = fmaxf(M, __ldcg(&a.part_ml[(p0 + q) * 2]));
                Ls = 0.f;
#pragma unroll
                for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
#pragma unroll 4
                for (int q = 0; q < S; ++q) {
                  const float wgt = expf(__ldcg(&a.part_ml[(p0 + q) * 2]) - M);
                  Ls = fmaf(wgt, __ldcg(&a.part_ml[(p0 + q) * 2 + 1]), Ls);
#pragma unroll
                  for (int i = 0; i < DPL; ++i)
                    acc[i] = fmaf(wgt, __ldcg(&a.part_o[(p0 + q) * HD + lane * DPL + i]), acc[i]);
                }
              }
            }
            if (last) {
#pragma unroll
              for (int i = 0; i < DPL; ++i) a.attn[(size_t)h * HD + lane * DPL + i] = acc[i] / Ls;
              __threadfence();
              __syncwarp();
              if (lane == 0) red_release(heads_done + l, 1u);
            }
          }
          if (tau + (int)G < NT) __syncthreads();  // the next task reuses the partial area
        }
        continue;
      }

      // ---- GEMV k of layer l ------------------------------------------------
      const int k = ph == 0 ? 0 : ph - 1;
      const int P = a.P[k];
      const bool active = (int)b < a.G[k];
      if (!active) continue;
      const unsigned* need;
      unsigned target;
      if (k == 0) {
        need = l == 0 ? a.sync + 1 : done + 4 * (l - 1) + 3;
        target = l == 0 ? G : (unsigned)a.G[3];
      } else if (k == 1) {
        need = heads_done + l;
        target = (unsigned)a.nh;
      } else {
        need = done + 4 * l + (k - 1);
        target = (unsigned)a.G[k - 1];
      }
      const float* xin = k == 0 || k == 2 ? a.x : (k == 1 ? a.attn : a.ffn_buf);
      const float* nw = k == 0 ? Ly.in_norm : (k == 2 ? Ly.post_norm : nullptr);
      const int K = a.cols[k];
      float wpre[TQ_CH][8];  // norm weights, loaded while the input is awaited
      if (nw) tq_preload<1>(wpre, nw, K, P);
      if (!cta_wait(a, need, target, &go_flag)) {
        ok = false;
        break;
      }
      const int ct0 = ((int)b * a.T16[k]) / a.G[k];
      for (int i = tid; i < a.per[k]; i += blockDim.x) cnt_s[i] = 0;
      // activation row (RMSNorm for qkv and gate/up, chat.py:63-66) -> B fragments
      if (nw) tq_run<1, MK_TW, true>(xin, K, 1, K, P, nw, a.eps, wpre, xb, fq, red);
      else tq_run<1, MK_TW, false>(xin, K, 1, K, P, nw, a.eps, wpre, xb, fq, red);
      __syncthreads();

      // this warp's units of the GEMV
      const int UT = a.UT[k];
      const int n_mine = warp_ok ? wu1[k] - wu0[k] : 0;
      const uint4* xbl = xb + (g & 1) * 4 + t;  // B column g (0 high, 1 low bytes); others read a valid one
      float acc0 = 0.f, acc1 = 0.f;
      int tile = 0, ku = 0;
      if (n_mine > 0) {
        tile = wu0[k] / UT;
        ku = wu0[k] - tile * UT;
      }
      for (int j = 0; j < n_mine; ++j) {
        const int p0 = ku * MK_KS, np = min(P - p0, MK_KS);
        const uint8_t* st;
        if (!take(st)) {
          warp_ok = false;
          break;
        }
        const uint4* cw = reinterpret_cast<const uint4*>(st) + lane;
        const uint8_t* sl = st + MK_KS * 512 + g * 4;
        const uint4* bp = xbl + (size_t)p0 * 8;
        const int2* fp = fq + p0;
        auto pair = [&](int i) {
          const uint4 wq = cw[i * 32];
          const uint4 bq = bp[i * 8];
          const int2 fv = fp[i];
          const __half2 hs = *reinterpret_cast<const __half2*>(sl + i * 32);
          const float s0 = __low2float(hs), s1 = __high2float(hs);
          int c[4];
          mma_first(c, wq.x & 0x0F0F0F0Fu, wq.x & 0xF0F0F0F0u, wq.y & 0x0F0F0F0Fu, wq.y & 0xF0F0F0F0u, bq.x, bq.y);
          mma_acc(c, wq.z & 0x0F0F0F0Fu, wq.z & 0xF0F0F0F0u, wq.w & 0x0F0F0F0Fu, wq.w & 0xF0F0F0F0u, bq.z, bq.w);
          const float fx = __int_as_float(fv.x);
          const int T0 = c[0] * 512 + c[1] * 2 + fv.y;
          const int T1 = c[2] * 512 + c[3] * 2 + fv.y * 16;
          acc0 = fmaf((float)T0, fx * s0, acc0);
          acc1 = fmaf((float)T1, fx * (s1 * 0.0625f), acc1);
        };
        if (np == MK_KS) {
#pragma unroll
          for (int i = 0; i < MK_KS; ++i) pair(i);
        } else {
          for (int i = 0; i < np; ++i) pair(i);
        }
        release();

        const bool tile_end = j + 1 == n_mine || ku + 1 == UT;
        if (++ku == UT) ku = 0;
        if (!tile_end) continue;
        const int tu0 = tile * UT, tu1 = tu0 + UT;
        float v0 = acc0, v1 = acc1;
        bool have = true;
        if (wu0[k] > tu0 || wu1[k] < tu1) {
          float* ps = part_s + ((size_t)(warp * 2 + (wu0[k] >= tu0 ? 0 : 1)) * 16 + g);
          if (t == 0) {
            ps[0] = acc0;
            ps[8] = acc1;
          }
          __threadfence_block();
          __syncwarp();
          const int mine = min(wu1[k], tu1) - max(wu0[k], tu0);
          int old = 0;
          if (lane == 0) old = atomicAdd(&cnt_s[tile - ct0], mine);
          old = __shfl_sync(0xffffffffu, old, 0);
          have = old + mine == UT;
          if (have) {
            __threadfence_block();
            v0 = v1 = 0.f;
            const int cu0 = ct0 * UT, nU = ((((int)b + 1) * a.T16[k]) / a.G[k] - ct0) * UT;
            auto start = [&](int w) { return cu0 + ((w * nU) >> 4); };
            int w = warp;
            while (w > 0 && start(w) > tu0) --w;
            for (; w < MK_TW && start(w) < tu1; ++w) {
              const int s0w = start(w), s1w = start(w + 1);
              if (max(s0w, tu0) >= min(s1w, tu1)) continue;
              if (w == warp) {
                v0 += acc0;
                v1 += acc1;
              } else {
                const float* qp = part_s + ((size_t)(w * 2 + (s0w >= tu0 ? 0 : 1)) * 16 + g);
                v0 += qp[0];
                v1 += qp[8];
              }
            }
          }
        }
        if (have) {
          // epilogue of rows tile*16 + g (+8) in lanes t == 0; paired rows from lane + 4
          v0 /= 15.f;
          v1 /= 15.f;
          const int rows = a.rows[k];
          const int row0 = tile * 16;
          if (k == 1 || k == 3) {
            if (t == 0) {
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                const int row = row0 + g + 8 * hh;
                if (row < rows) a.x[row] = a.x[row] + (hh ? v1 : v0);
              }
            }
          } else {
            const float n0 = __shfl_down_sync(0xffffffffu, v0, 4), n1 = __shfl_down_sync(0xffffffffu, v1, 4);
            if (t == 0 && !(g & 1)) {
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                const int row = row0 + g + 8 * hh;
                if (row + 1 >= rows) continue;
                const float x1 = hh ? v1 : v0, x2 = hh ? n1 : n0;
                if (k == 2) {
                  // rows 2i = gate_i, 2i+1 = up_i (chat.py:300-302, the +-40 clip)
                  const float e = expf(-fminf(fmaxf(x1, -40.f), 40.f));
                  a.ffn_buf[row >> 1] = x1 / (1.0f + e) * x2;
                } else {
                  const int half = HD / 2;
                  const int qrows = a.nh * HD, krows = a.nkv * HD;
                  const size_t blk = ep_blk, off = ep_off;
                  KT* kcache = reinterpret_cast<KT*>(a.kpool) + (size_t)l * a.layer_elems;
                  KT* vcache = reinterpret_cast<KT*>(a.vpool) + (size_t)l * a.layer_elems;
                  if (row < qrows + krows) {
                    const bool isq = row < qrows;
                    const int rr = isq ? row : row - qrows;
                    const int hq = rr / HD, pp = (rr % HD) >> 1;
                    const float c = a.cos_t[(size_t)ep_pos * half + pp], s = a.sin_t[(size_t)ep_pos * half + pp];
                    // rotate-half RoPE, fp32 products rounded separately (chat.py:99-100)
                    const float o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
                    const float o2 = __fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c));
                    if (isq) {
                      a.q_buf[(size_t)hq * HD + pp] = o1;
                      a.q_buf[(size_t)hq * HD + pp + half] = o2;
                    } else {
                      const size_t base = ((blk * a.nkv + hq) * a.bs + off) * HD;
                      kcache[base + pp] = to_kv<KT>(o1);
                      kcache[base + pp + half] = to_kv<KT>(o2);
                    }
                  } else {
                    const float vv[2] = {x1, x2};
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                      const int rr = row + e - qrows - krows;
                      const size_t idx = ((blk * a.nkv + rr / HD) * a.bs + off) * HD + rr % HD;
                      vcache[idx] = to_kv<KT>(vv[e]);
                    }
                  }
                }
              }
            }
          }
        }
        acc0 = acc1 = 0.f;
        ++tile;
      }
      // every tile of this CTA is written: one release per CTA and GEMV
      __syncthreads();
      if (tid == 0) {
        __threadfence();
        red_release(done + 4 * l + k, 1u);
      }
    }
  }

  // ---- LM head (chat.py:388, no final norm) with the argmax fused ----------
  if (ok && cta_wait(a, done + 4 * (L - 1) + 3, (unsigned)a.G[3], &go_flag)) {
    unsigned long long best = 0ull;
    const int K = a.d, n8 = K / 8, n_tasks = (a.vocab + 1) / 2;
    for (int task = (int)b * MK_TW + warp; task < n_tasks; task += G * MK_TW) {
      const int row0 = task * 2;
      float acc[2] = {0.f, 0.f};
      for (int c = lane; c < n8; c += 32) {
        const float4* xp = reinterpret_cast<const float4*>(a.x + (size_t)c * 8);
        const float4 xa = xp[0], xc = xp[1];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int row = min(row0 + r, a.vocab - 1);
          const uint4 wv = ldg_stream(a.head + (size_t)row * K + (size_t)c * 8);
          const __half2* hp = reinterpret_cast<const __half2*>(&wv);
          const float2 w0 = __half22float2(hp[0]), w1 = __half22float2(hp[1]);
          const float2 w2 = __half22float2(hp[2]), w3 = __half22float2(hp[3]);
          float s = acc[r];
          s = fmaf(xa.x, w0.x, s); s = fmaf(xa.y, w0.y, s);
          s = fmaf(xa.z, w1.x, s); s = fmaf(xa.w, w1.y, s);
          s = fmaf(xc.x, w2.x, s); s = fmaf(xc.y, w2.y, s);
          s = fmaf(xc.z, w3.x, s); s = fmaf(xc.w, w3.y, s);
          acc[r] = s;
        }
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float v = warp_sum(acc[r]);
        const int row = row0 + r;
        if (row < a.vocab) {
          const unsigned u = __float_as_uint(v);
          const unsigned ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
          const unsigned long long key = ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)row);
          best = key > best ? key : best;
          if (lane == r) a.logits[row] = v;
        }
      }
    }
    if (lane == 0 && best) atomicMax(a.amax_key, best);
    __threadfence();
    __syncthreads();
    if (tid == 0) last_flag = atomicAdd(a.sync + 2, 1u) == G - 1;
    __syncthreads();
    if (last_flag && tid == 0 && a.greedy) {
      // the next step's token and parameters (greedy_commit_kernel)
      __threadfence();
      const unsigned long long key = atomicAdd(a.amax_key, 0ull);
      const int tok = (int)(0xFFFFFFFFu - (unsigned)(key & 0xFFFFFFFFull));
      a.tokens[0] = tok;
      a.chain_tokens[*a.chain_count] = tok;
      *a.chain_count += 1;
      a.Pd->t_prev += 1;
      a.Pd->t_tot += 1;
      a.rowpos[0] += 1;
      const int sp = (a.Pd->t_tot + 63) / 64;
      a.Pd->n_splits = sp < 1 ? 1 : (sp > a.max_splits ? a.max_splits : sp);
    }
  }

  // after an abort some issued units were never consumed: let this warp's
  // copies in flight land (bounded) before the CTA releases its shared memory
  if (lane == 0)
    for (unsigned s = consumed; s < issued; ++s) mbar_wait_bounded(&bars[s % MK_TS], (s / MK_TS) & 1u);
  __syncwarp();
}

}  // namespace

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct MkPlan {
  MkArgs a;
  MkLayer* layers_dev = nullptr;
  size_t smem = 0;
  int grid = 0;
  size_t sync_words = 0;
};

static int mk_plan_weight(MkArgs& a, int k, const lumina_weight* w) {
  if (!w || !w->mma || w->bits != 4 || w->group != 64 || !w->fp16_scales) return LUMINA_E_UNSUPPORTED;
  a.rows[k] = w->rows;
  a.cols[k] = w->cols;
  a.T16[k] = w->rows_pad / 16;
  a.P[k] = w->n_chunks / 2;
  a.ng[k] = w->n_groups;
  a.UT[k] = (a.P[k] + MK_KS - 1) / MK_KS;
  return LUMINA_OK;
}

int decode_mk_prepare(void** plan_out, const MkSetup& s) {
  *plan_out = nullptr;
  if (s.hd * (s.kv_fp16 ? 2 : 4) != MK_ROWB) return LUMINA_E_UNSUPPORTED;
  if (s.block_size < MK_AK) return LUMINA_E_UNSUPPORTED;  // an attention unit spans at most two pages
  if (s.nh % s.nkv || s.d % 8) return LUMINA_E_UNSUPPORTED;
  MkPlan* pl = new MkPlan();
  MkArgs& a = pl->a;
  a = MkArgs{};
  a.n_layer = s.n_layer;
  a.d = s.d;
  a.nh = s.nh;
  a.nkv = s.nkv;
  a.hd = s.hd;
  a.ffn = s.ffn;
  a.eps = s.eps;
  a.sdiv = std::max(sqrtf((float)s.hd), 1e-6f);  // max(hd ** 0.5, 1e-6), chat.py:278
  std::vector<MkLayer> hl(s.n_layer);
  for (int l = 0; l < s.n_layer; ++l) {
    for (int k = 0; k < 4; ++k) {
      const lumina_weight* w = s.w[l][k];
      if (mk_plan_weight(a, k, w)) {
        delete pl;
        return LUMINA_E_UNSUPPORTED;
      }
      hl[l].w[k].codes = w->codes;
      hl[l].w[k].scales = w->scales;
    }
    hl[l].in_norm = s.in_norm[l];
    hl[l].post_norm = s.post_norm[l];
  }
  const int sms = sm_count();
  a.Pmax = 0;
  int per_max = 1;
  for (int k = 0; k < 4; ++k) {
    a.per[k] = (a.T16[k] + sms - 1) / sms;
    a.G[k] = (a.T16[k] + a.per[k] - 1) / a.per[k];
    a.Pmax = std::max(a.Pmax, a.P[k]);
    per_max = std::max(per_max, a.per[k]);
  }
  // shared memory: B fragments (between the qkv and o GEMVs: the attention
  // warp partials), (sx, -15 sum q), tile counters,
  // partials, rings, mbarriers
  size_t off = std::max((size_t)a.Pmax * 2 * 64, (size_t)MK_TW * (s.hd + 2) * 4);
  off = (off + 15) / 16 * 16;
  a.off_fq = (int)off;
  off += (size_t)a.Pmax * 8;
  a.off_cnt = (int)off;
  off += (size_t)per_max * 4;
  off = (off + 15) / 16 * 16;
  a.off_part = (int)off;
  off += (size_t)MK_TW * 2 * 16 * 4;
  off = (off + 127) / 128 * 128;
  a.off_ring = (int)off;
  off += (size_t)MK_TW * MK_TS * MK_STAGE;
  a.off_bars = (int)off;
  off += (size_t)MK_TW * MK_TS * 8;
  pl->smem = off;
  if (pl->smem > 227 * 1024 - 1024) {
    delete pl;
    return LUMINA_E_UNSUPPORTED;
  }
  pl->sync_words = 4 + 5 * (size_t)s.n_layer + (size_t)s.n_layer * s.nh;
  if (cudaMalloc(&pl->layers_dev, hl.size() * sizeof(MkLayer)) != cudaSuccess) {
    cudaGetLastError();
    delete pl;
    set_error("decode_mk: allocation failed");
    return LUMINA_E_OOM;
  }
  cudaMemcpy(pl->layers_dev, hl.data(), hl.size() * sizeof(MkLayer), cudaMemcpyHostToDevice);
  a.layers = pl->layers_dev;
  *plan_out = pl;
  return LUMINA_OK;
}

size_t decode_mk_sync_words(const void* plan) { return static_cast<const MkPlan*>(plan)->sync_words; }

size_t decode_mk_part_floats(int nh, int hd, int max_seq) {
  const size_t cmax = (size_t)(max_seq + MK_AK - 1) / MK_AK;
  return (size_t)nh * cmax * (hd + 2);
}

void decode_mk_free(void* plan) {
  MkPlan* pl = static_cast<MkPlan*>(plan);
  if (!pl) return;
  if (pl->layers_dev) cudaFree(pl->layers_dev);
  delete pl;
}

int decode_mk_launch(void* plan, const MkRun& r, cudaStream_t s) {
  MkPlan* pl = static_cast<MkPlan*>(plan);
  MkArgs a = pl->a;
  a.x = r.x;
  a.q_buf = r.q_buf;
  a.attn = r.attn;
  a.ffn_buf = r.ffn_buf;
  a.kpool = r.kpool;
  a.vpool = r.vpool;
  a.layer_elems = r.layer_elems;
  a.kv_fp16 = r.kv_fp16;
  a.bt = r.bt;
  a.bs = r.bs;
  a.cos_t = r.cos_t;
  a.sin_t = r.sin_t;
  a.Pd = r.P;
  a.rowpos = r.rowpos;
  a.tokens = r.tokens;
  a.embed = r.embed;
  a.embed_rows = r.embed_rows;
  a.head = r.head;
  a.vocab = r.vocab;
  a.logits = r.logits;
  a.amax_key = r.amax_key;
  a.greedy = r.greedy;
  a.chain_tokens = r.chain_tokens;
  a.chain_count = r.chain_count;
  a.max_splits = r.max_splits;
  a.cmax = (r.max_seq + MK_AK - 1) / MK_AK;
  a.part_o = r.part;
  a.part_ml = r.part + (size_t)a.nh * a.cmax * a.hd;
  a.sync = r.sync;
  a.fault = fault_flag_ptr();
  if (!a.fault) {
    set_error("decode_mk: fault flag unavailable");
    return LUMINA_E_CUDA;
  }
  auto kern = r.kv_fp16 ? decode_mk_kernel<__half> : decode_mk_kernel<float>;
  static size_t configured[2] = {0, 0};
  size_t& conf = configured[r.kv_fp16 ? 1 : 0];
  if (pl->smem > conf) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl->smem);
    if (e != cudaSuccess) {
      set_error("decode_mk attribute: %s", cudaGetErrorString(e));
      return LUMINA_E_CUDA;
    }
    conf = pl->smem;
  }
  if (!pl->grid) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, MK_TW * 32, pl->smem) != cudaSuccess ||
        per_sm < 1) {
      cudaGetLastError();
      set_error("decode_mk: the kernel does not fit on an SM");
      return LUMINA_E_UNSUPPORTED;
    }
    pl->grid = sm_count();
  }
  // the kernel's key-split arithmetic is 32-bit: splits x units < 2^31
  if ((long long)a.cmax * pl->grid >= (1ll << 31)) {
    set_error("decode_mk: context %d too long for the persistent step", r.max_seq);
    return LUMINA_E_UNSUPPORTED;
  }
  LUMINA_CUDA_TRY(cudaMemsetAsync(r.sync, 0, pl->sync_words * 4, s));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl->grid);
  cfg.blockDim = dim3(MK_TW * 32);
  cfg.dynamicSmemBytes = pl->smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) {
    set_error("decode_mk launch: %s", cudaGetErrorString(e));
    return LUMINA_E_CUDA;
  }
  return LUMINA_OK;
}

}  // namespace lumina
