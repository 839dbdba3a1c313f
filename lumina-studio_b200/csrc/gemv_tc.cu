// Decode GEMV for int4 weights on the tensor pipe (batch 1, 2 or 4).
//
// Arithmetic. The activation row is quantized per 64-column pair (one
// scale group when group = 64): q = rint(x * fp32(32639/amax)), clamped to
// +-32639, so that q = 256*qh + ql with qh = (q + 128) >> 8 and ql both
// signed bytes. One mma.sync.m16n8k32 (u8 codes x s8) then takes the high
// and the low bytes of a batch row as two B columns (2b, 2b+1), and a second
// one accumulates the pair's other 32 columns, so for a 16-row tile the C
// fragment holds Dh = sum c*qh and Dl = sum c*ql over the 64 columns, exact.
// Per row and pair: T = 2*(256*Dh + Dl) - 15*sum(q), y += T * sx * s, and
// y /= 15 at the end (adapters/lumina.py:135-139: level = (2c - 15) / 15).
// Narrow codes stored one per nibble (int3 / int2 / binary, the same
// layout) use their own level count L = 2^bits - 1 in place of 15.
// The A operand takes the code bytes straight from the fragment layout
// (weights.cuh, mma = 1): low nibbles = the tile's rows 0..7, high nibbles =
// rows 8..15 times 16; that factor 16 is folded exactly into the fp32 scale.
// C lane (g, t) holds rows g and g+8 of batch row t, so an epilogue lane
// never needs another lane's value. B columns beyond the batch (lanes with
// g >= 2*NB) read any valid column: they only feed C columns that are never
// used, so every lane walks the tables with the same compile-time stride.
//
// Work split. Each CTA owns whole 16-row tiles (an equal share, with as few
// CTAs as that share allows), so no partial sum ever leaves the SM. A unit
// is (tile, KS pairs), KS a compile-time 8, 6 or 4 so the unrolled pair loop
// addresses shared memory with immediate offsets; a CTA's units in
// tile-major order are cut into equal runs, one per warp. A warp streams its
// units through a ring of TS shared-memory stages that one lane fills with
// cp.async.bulk (the codes and the scales of a unit are two contiguous
// spans; completion on an mbarrier per stage); the first stages are
// requested before griddepcontrol.wait. A tile split between warps is
// summed in shared memory: each warp stores its partial and adds its unit
// count to the tile's counter, and the warp that completes the count adds
// the partials in unit order (so the result does not depend on which warp
// finishes last) and applies the epilogue.
#include "gemv_impl.cuh"
#include "tc_act.cuh"

namespace lumina {

namespace {

constexpr int TW = 16;          // warps per CTA
constexpr int TW_SHIFT = 4;     // log2(TW)
constexpr int TS = 3;           // ring stages per warp

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

struct TcArgs {
  const uint8_t* codes;
  const uint8_t* scales;
  int rows, cols;
  int P;        // 64-column pairs per row (codes padded to whole pairs)
  int ng;       // scale groups per row
  int gsh;      // log2(group / 64); KS is a multiple of 2^gsh
  int T16;      // 16-row tiles
  int UT;       // units per tile
  int MT;       // most tiles of one CTA
  int stage_bytes;
  int x_bytes;  // shared bytes before the rings
  const float* x;
  int ldx;
  const float* norm_w;
  float eps;
  float* y;
  int ldy;
  const float* resid;
  int ldr;
  RopeKV rk;
  int nb;       // live batch rows (<= NB)
  int* fault;
  long long spin;  // polls before a wait on a ring stage gives up (wait_spin_limit())
  L2Prefetch pf;   // the next kernel's bytes, pulled into L2 while this one runs
  int lv;          // levels - 1 of the codes: 15 (int4), 7, 3, 1 (narrow codes one per nibble)
};

// The fused tensor-parallel exchange of a launch, a kernel parameter of its
// own so that the kernels outside an exchange (TPX false, every one-GPU
// launch) carry neither its bytes nor its code.
template <bool TPX>
struct TpParam {
  TcTp v;
};
template <>
struct TpParam<false> {};

__device__ __forceinline__ unsigned long long tc_global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned tc_ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void tc_st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <typename ST>
__device__ __forceinline__ void load_scale_pair(const uint8_t* p, float& s0, float& s1) {
  if constexpr (sizeof(ST) == 2) {
    const __half2 h = *reinterpret_cast<const __half2*>(p);
    s0 = __low2float(h);
    s1 = __high2float(h);
  } else {
    const float2 f = *reinterpret_cast<const float2*>(p);
    s0 = f.x;
    s1 = f.y;
  }
}

// Epilogue of one finished 16-row tile for batch row t (lane t of each row
// group g): v0 = row g, v1 = row g + 8, already / L. Paired epilogues (rows
// 2i, 2i+1) take the odd row from the neighbouring row group's lane.
// ep_s: the operands staged in shared memory by the prologue -- residual
// rows [res0, res0 + MT*16) of each batch row (EPI_RESID), or the RoPE
// cos / sin rows of each batch row's position (EPI_ROPE_KV).
template <int NB, int EPI, bool TPX>
__device__ __forceinline__ void tc_epilogue(const TcArgs& a, const TpParam<TPX>& tp, int row0, float v0, float v1,
                                            int lane, const int* kv_blk, const int* kv_off, const float* ep_s,
                                            int res0) {
  const int g = lane >> 2, t = lane & 3;
  const bool live = t < NB && t < a.nb;
  if constexpr (EPI == EPI_STORE || EPI == EPI_RESID) {
    if (!live) return;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = row0 + g + 8 * h;
      if (row < a.rows) {
        float v = h ? v1 : v0;
        if constexpr (EPI == EPI_RESID) v = ep_s[t * (a.MT * 16) + (row - res0)] + v;
        if constexpr (TPX && EPI == EPI_STORE) {
          // every rank's receive slot for this rank (peer stores over NVLink)
          for (int r = 0; r < tp.v.tp; ++r) tp.v.push[r][(size_t)t * tp.v.ld + row] = v;
        } else {
          a.y[(size_t)t * a.ldy + row] = v;
        }
      }
    }
  } else {
    // row 2i lives in row group g = 2i (mod 8), row 2i+1 in g + 1: even-g
    // lanes take the odd row's value from lane + 4
    const float n0 = __shfl_down_sync(0xffffffffu, v0, 4), n1 = __shfl_down_sync(0xffffffffu, v1, 4);
    if (!live || (g & 1)) return;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = row0 + g + 8 * h;  // even
      if (row + 1 >= a.rows) continue;
      const float x1 = h ? v1 : v0, x2 = h ? n1 : n0;
      if constexpr (EPI == EPI_SWIGLU) {
        // rows 2i = gate_i, 2i+1 = up_i (chat.py:300-302, the +-40 clip)
        const float e = expf(-fminf(fmaxf(x1, -40.f), 40.f));
        a.y[(size_t)t * a.ldy + (row >> 1)] = x1 / (1.0f + e) * x2;
      } else {
        // fused q/k/v rows: [q heads (RoPE pairs adjacent)][k heads (pairs adjacent)][v]
        const RopeKV& k = a.rk;
        const int qrows = k.nh * k.hd, krows = k.nkv * k.hd, half = k.hd / 2;
        const size_t blk = kv_blk[t], off = kv_off[t];
        if (row < qrows + krows) {
          const bool isq = row < qrows;
          const int rr = isq ? row : row - qrows;
          const int hh = rr / k.hd, p = (rr % k.hd) >> 1;
          const float c = ep_s[t * half + p], s = ep_s[(NB + t) * half + p];
          // rotate-half RoPE, fp32 products rounded separately (chat.py:99-100)
          const float o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
          const float o2 = __fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c));
          if (isq) {
            float* q = k.q_out + (size_t)t * qrows + (size_t)hh * k.hd;
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
    }
  }
}

template <int NB, typename ST, int EPI, bool NORM, int KS, bool TPX>
__global__ void __launch_bounds__(TW * 32, 1)
gemv_tc_kernel(TcArgs a, TpParam<TPX> tp) {
  constexpr int ES = sizeof(ST);
  constexpr int NC = 2 * NB;   // B columns: (high, low) bytes per batch row
  constexpr int SG = 16 * ES;  // scale bytes of one group of a tile: 8 x (row g, row g+8)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int P = a.P;

  // this CTA's tiles and units, this warp's run
  const int G = gridDim.x;
  const int ctile0 = (blockIdx.x * a.T16) / G, ctile1 = ((blockIdx.x + 1) * a.T16) / G;
  const int cu0 = ctile0 * a.UT, cu1 = ctile1 * a.UT;
  const int nU = cu1 - cu0;
  const int wu0 = cu0 + ((warp * nU) >> TW_SHIFT), wu1 = cu0 + (((warp + 1) * nU) >> TW_SHIFT);
  const int n_mine = wu1 - wu0;

  extern __shared__ __align__(128) uint8_t smem[];
  // [B fragments: P x NC x 4 lanes x 16 B][(sx, -L*sum q): P x NB x 8 B]
  // [tile counters: MT ints][partials: TW x 2 x 16 x NB floats]
  // [rings: TW x TS x stage_bytes][mbarriers: TW x TS]
  uint4* xb = reinterpret_cast<uint4*>(smem);
  int2* fq = reinterpret_cast<int2*>(xb + (size_t)P * NC * 4);
  int* cnt_s = reinterpret_cast<int*>(fq + (size_t)P * NB);
  float* part_s = reinterpret_cast<float*>(cnt_s + a.MT);
  float* ep_s = part_s + TW * 2 * 16 * NB;  // staged epilogue operands (see tc_epilogue)
  uint8_t* ring = smem + a.x_bytes + (size_t)warp * TS * a.stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.x_bytes + (size_t)TW * TS * a.stage_bytes) + warp * TS;
  __shared__ float red[NB * TW];
  __shared__ int ep_blk[NB], ep_off[NB];

  // lane 0: unit j of this warp's run into stage j % TS (two bulk copies
  // completing on the stage's mbarrier); units are issued in order, so the
  // (tile, unit-in-tile) of the next one is tracked, not divided out
  int i_tile = 0, i_ku = 0;
  if (n_mine > 0) {
    i_tile = wu0 / a.UT;
    i_ku = wu0 - i_tile * a.UT;
  }
  const uint64_t pol = l2_evict_first_policy();
  auto issue = [&](int j) {
    const int tile = i_tile, p0 = i_ku * KS, np = min(P - p0, KS);
    if (++i_ku == a.UT) {
      i_ku = 0;
      ++i_tile;
    }
    const int G0 = p0 >> a.gsh, G1 = ((p0 + np - 1) >> a.gsh) + 1;
    uint8_t* st = ring + (size_t)(j % TS) * a.stage_bytes;
    const uint32_t cb = (uint32_t)np * 512u, sb = (uint32_t)(G1 - G0) * SG;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_expect_tx(&bars[j % TS], cb + sb);
    bulk_g2s_hint(st, a.codes + ((size_t)tile * P + p0) * 512, cb, &bars[j % TS], pol);
    bulk_g2s_hint(st + KS * 512, a.scales + ((size_t)tile * a.ng + G0) * SG, sb, &bars[j % TS], pol);
  };

  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < TS; ++i) mbar_init(&bars[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  // 1) weights never depend on the previous kernel: the first stages go out
  //    before the dependency wait
  if (lane == 0) {
    for (int j = 0; j < min(TS, n_mine); ++j) issue(j);
    l2_prefetch_share(a.pf, blockIdx.x * TW + warp, G * TW);
  }
  // norm weights never depend on the previous kernel either
  float wpre[TQ_CH][8];
  if constexpr (NORM) tq_preload<NB>(wpre, a.norm_w, a.cols, P);
  if constexpr (EPI == EPI_ROPE_KV) {
    // the KV slot and the rotation of each batch row: positions, KV length
    // and block table are set before the step (host copy or the previous
    // step's commit kernel), not by the kernels this one waits for
    const int half = a.rk.hd / 2;
    if (threadIdx.x < NB && threadIdx.x < a.nb) {
      const int tt = *a.rk.t_prev + a.rk.row_base + threadIdx.x;
      ep_blk[threadIdx.x] = a.rk.block_table[tt / a.rk.bs];
      ep_off[threadIdx.x] = tt % a.rk.bs;
    }
    for (int i = threadIdx.x; i < a.nb * half; i += blockDim.x) {
      const int t = i / half, p = i - t * half;
      const size_t o = (size_t)a.rk.row_pos[t] * half + p;
      ep_s[i] = a.rk.cos_t[o];
      ep_s[NB * half + i] = a.rk.sin_t[o];
    }
  }
  pdl_launch_dependents();
  pdl_wait();

  // 2) activation rows -> B fragments in shared memory; the residual rows
  //    of this CTA's tiles stream into shared memory meanwhile (cp.async)
  for (int i = threadIdx.x; i < a.MT; i += blockDim.x) cnt_s[i] = 0;
  if constexpr (EPI == EPI_RESID) {
    const int r0 = ctile0 * 16, nr = min(ctile1 * 16, a.rows) - r0;
    for (int i = threadIdx.x; i < a.nb * nr; i += blockDim.x) {
      const int t = i / nr, r = i - t * nr;
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(ep_s + t * (a.MT * 16) + r)),
                   "l"(a.resid + (size_t)t * a.ldr + r0 + r)
                   : "memory");
    }
    cp_async_commit();
  }
  if constexpr (TPX && NORM) {
    // every rank's rows of this exchange have landed once its flag holds the
    // epoch this rank's own producer (the kernel waited for above) set
    __shared__ int tp_ok;
    if (threadIdx.x == 0) {
      const unsigned ep = *reinterpret_cast<volatile const unsigned*>(tp.v.epoch);
      const unsigned long long t0 = tc_global_ns();
      int ok = 1;
      for (int r = 0; r < tp.v.tp && ok; ++r)
        while ((int)(tc_ld_acquire_sys(tp.v.in_flags + r) - ep) < 0)
          if (tc_global_ns() - t0 >= tp.v.timeout_ns) {
            atomicOr(a.fault, 4);
            ok = 0;
            break;
          }
      tp_ok = ok;
    }
    __syncthreads();
    TqSum sum;
    if (tp_ok) {
#pragma unroll
      for (int r = 0; r < TQ_MAX_ADD; ++r) sum.add[r] = r < tp.v.tp ? tp.v.add[r] : nullptr;
      sum.n_add = tp.v.tp;
      sum.xout = tp.v.xout;
    }
    tq_run<NB, TW, NORM>(a.x, a.ldx, a.nb, a.cols, P, a.norm_w, a.eps, wpre, xb, fq, red, a.lv, &sum);
  } else {
    tq_run<NB, TW, NORM>(a.x, a.ldx, a.nb, a.cols, P, a.norm_w, a.eps, wpre, xb, fq, red, a.lv);
  }
  if constexpr (EPI == EPI_RESID) cp_async_wait<0>();
  __syncthreads();

  // 3) this warp's units
  const uint4* xbl = xb + (g & (NC - 1)) * 4 + t;  // column g, or any valid one
  const int2* fql = fq + (t & (NB - 1));           // batch row t, or any valid one
  float acc0 = 0.f, acc1 = 0.f;  // rows g, g+8 of batch row t
  int failed = -1;  // the unit a wait gave up on
  int tile = 0, ku = 0;
  if (n_mine > 0) {
    tile = wu0 / a.UT;
    ku = wu0 - tile * a.UT;
  }
  for (int j = 0; j < n_mine; ++j) {
    const int p0 = ku * KS, np = min(P - p0, KS);
    // every lane polls the stage's mbarrier (lane-0 polling plus a shuffle
    // measured 2% slower per token here)
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bars[j % TS], (uint32_t)((j / TS) & 1), a.spin))) {
      failed = j;
      break;
    }
    const uint8_t* st = ring + (size_t)(j % TS) * a.stage_bytes;
    const uint4* cw = reinterpret_cast<const uint4*>(st) + lane;
    const uint8_t* sl = st + KS * 512 + g * 2 * ES;
    const uint4* bp = xbl + (size_t)p0 * (NC * 4);
    const int2* fp = fql + (size_t)p0 * NB;
    auto pair = [&](int i) {
      const uint4 wq = cw[i * 32];
      const uint4 bq = bp[i * NC * 4];
      const int2 fv = fp[i * NB];
      float s0, s1;
      load_scale_pair<ST>(sl + (i >> a.gsh) * SG, s0, s1);
      int c[4];
      mma_first(c, wq.x & 0x0F0F0F0Fu, wq.x & 0xF0F0F0F0u, wq.y & 0x0F0F0F0Fu, wq.y & 0xF0F0F0F0u, bq.x, bq.y);
      mma_acc(c, wq.z & 0x0F0F0F0Fu, wq.z & 0xF0F0F0F0u, wq.w & 0x0F0F0F0Fu, wq.w & 0xF0F0F0F0u, bq.z, bq.w);
      const float fx = __int_as_float(fv.x);
      const int T0 = c[0] * 512 + c[1] * 2 + fv.y;
      const int T1 = c[2] * 512 + c[3] * 2 + fv.y * 16;  // rows g+8 carry codes * 16
      acc0 = fmaf((float)T0, fx * s0, acc0);
      acc1 = fmaf((float)T1, fx * (s1 * 0.0625f), acc1);
    };
    if (np == KS) {
#pragma unroll
      for (int i = 0; i < KS; ++i) pair(i);
    } else {
      for (int i = 0; i < np; ++i) pair(i);  // the short last unit of a row
    }
    __syncwarp();  // every lane is done with stage j % TS
    if (lane == 0 && j + TS < n_mine) issue(j + TS);

    // end of this warp's run over `tile`?
    const bool tile_end = j + 1 == n_mine || ku + 1 == a.UT;
    if (++ku == a.UT) ku = 0;
    if (!tile_end) continue;
    const int tu0 = tile * a.UT, tu1 = tu0 + a.UT;  // the tile lies inside this CTA's range
    float v0 = acc0, v1 = acc1;
    bool have = true;  // this warp holds the tile's sum
    if (wu0 > tu0 || wu1 < tu1) {
      // several warps: partial -> shared slot (0: the tile this warp's run
      // starts in, 1: the one it ends in); arrivals count units, so the warp
      // that completes the tile's units sums the slots
      float* ps = part_s + ((size_t)(warp * 2 + (wu0 >= tu0 ? 0 : 1)) * 16 + g) * NB + (t & (NB - 1));
      if (t < NB) {
        ps[0] = acc0;
        ps[8 * NB] = acc1;
      }
      __threadfence_block();
      __syncwarp();
      const int mine = min(wu1, tu1) - max(wu0, tu0);
      int old = 0;
      if (lane == 0) old = atomicAdd(&cnt_s[tile - ctile0], mine);
      old = __shfl_sync(0xffffffffu, old, 0);
      have = old + mine == a.UT;
      if (have) {
        __threadfence_block();
        v0 = v1 = 0.f;
        // the contributing warps are contiguous: from the first whose run
        // holds tu0, in order (= the tile's units in order)
        auto start = [&](int w) { return cu0 + ((w * nU) >> TW_SHIFT); };
        int w = warp;
        while (w > 0 && start(w) > tu0) --w;
        for (; w < TW && start(w) < tu1; ++w) {
          const int s0w = start(w), s1w = start(w + 1);
          if (max(s0w, tu0) >= min(s1w, tu1)) continue;
          if (w == warp) {
            v0 += acc0;
            v1 += acc1;
          } else {
            const float* qs = part_s + ((size_t)(w * 2 + (s0w >= tu0 ? 0 : 1)) * 16 + g) * NB + (t & (NB - 1));
            v0 += qs[0];
            v1 += qs[8 * NB];
          }
        }
      }
    }
    if (have) tc_epilogue<NB, EPI, TPX>(a, tp, tile * 16, v0 / (float)a.lv, v1 / (float)a.lv, lane, ep_blk, ep_off, ep_s, ctile0 * 16);
    acc0 = acc1 = 0.f;
    ++tile;
  }
  if (failed >= 0) {
    // a stage did not land in time: record it, and let this warp's units
    // still in flight land before the CTA's shared memory is released. Units
    // failed .. failed + TS - 1 (those issued) occupy distinct stages; unit j
    // completes phase j / TS of stage j % TS. These waits take the full limit.
    if (lane == 0) {
      atomicOr(a.fault, 2);
      const int issued = min(n_mine, failed + TS);
      for (int j = failed; j < issued; ++j) mbar_wait_bounded(&bars[j % TS], (uint32_t)((j / TS) & 1));
    }
    __syncwarp();
  }
  if constexpr (TPX && EPI == EPI_STORE) {
    // the exchange is published once every CTA's rows are out: the last CTA
    // to take a ticket (every CTA takes one, a failed one too, so the
    // counter returns to zero) advances the epoch and flags every rank
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      const int tk = atomicAdd(tp.v.ticket, 1);
      if (tk == (int)gridDim.x - 1) {
        *tp.v.ticket = 0;
        __threadfence_system();
        const unsigned ep = *tp.v.epoch + 1u;
        *tp.v.epoch = ep;
        for (int r = 0; r < tp.v.tp; ++r) tc_st_release_sys(tp.v.flags[r], ep);
      }
    }
  }
}

template <int NB, typename ST, int EPI, bool NORM, int KS, bool TPX>
int launch_tc(const TcArgs& a, const TcTp* tpx, size_t smem, int grid, cudaStream_t s) {
  auto kern = gemv_tc_kernel<NB, ST, EPI, NORM, KS, TPX>;
  const int rc = set_smem_limit((const void*)kern, smem, "gemv_tc");
  if (rc) return rc;
  TpParam<TPX> tp{};
  if constexpr (TPX) tp.v = *tpx;
  const cudaError_t e = launch_pdl(kern, dim3(grid), dim3(TW * 32), smem, s, a, tp);
  if (e != cudaSuccess) {
    set_error("gemv_tc launch: %s", cudaGetErrorString(e));
    return LUMINA_E_CUDA;
  }
  return LUMINA_OK;
}

// a fused exchange (tpx non-null) has a producing side (o_proj, down_proj:
// EPI_STORE without a norm) and consuming sides (normalizing q/k/v and
// gate/up); the one-GPU kernels are the TPX = false instances
template <int NB, typename ST, int KS>
int tc_epi(const TcArgs& a, const TcTp* tpx, size_t smem, int grid, int epi, bool norm, cudaStream_t s) {
  switch (epi) {
    case EPI_STORE:
      if (norm) return tpx ? LUMINA_E_UNSUPPORTED : launch_tc<NB, ST, EPI_STORE, true, KS, false>(a, tpx, smem, grid, s);
      return tpx ? launch_tc<NB, ST, EPI_STORE, false, KS, true>(a, tpx, smem, grid, s)
                 : launch_tc<NB, ST, EPI_STORE, false, KS, false>(a, tpx, smem, grid, s);
    case EPI_RESID:
      return norm || tpx ? LUMINA_E_UNSUPPORTED : launch_tc<NB, ST, EPI_RESID, false, KS, false>(a, tpx, smem, grid, s);
    case EPI_SWIGLU:
      if (!norm) return LUMINA_E_UNSUPPORTED;
      return tpx ? launch_tc<NB, ST, EPI_SWIGLU, true, KS, true>(a, tpx, smem, grid, s)
                 : launch_tc<NB, ST, EPI_SWIGLU, true, KS, false>(a, tpx, smem, grid, s);
    default:
      if (!norm) return LUMINA_E_UNSUPPORTED;
      return tpx ? launch_tc<NB, ST, EPI_ROPE_KV, true, KS, true>(a, tpx, smem, grid, s)
                 : launch_tc<NB, ST, EPI_ROPE_KV, true, KS, false>(a, tpx, smem, grid, s);
  }
}

template <int KS>
int tc_nb(const TcArgs& a, const TcTp* tpx, size_t smem, int grid, int nb, bool fp16, int epi, bool norm,
          cudaStream_t s) {
  if (fp16) {
    switch (nb) {
      case 1: return tc_epi<1, __half, KS>(a, tpx, smem, grid, epi, norm, s);
      case 2: return tc_epi<2, __half, KS>(a, tpx, smem, grid, epi, norm, s);
      default: return tc_epi<4, __half, KS>(a, tpx, smem, grid, epi, norm, s);
    }
  }
  switch (nb) {
    case 1: return tc_epi<1, float, KS>(a, tpx, smem, grid, epi, norm, s);
    case 2: return tc_epi<2, float, KS>(a, tpx, smem, grid, epi, norm, s);
    default: return tc_epi<4, float, KS>(a, tpx, smem, grid, epi, norm, s);
  }
}

}  // namespace

int gemv_tc_launch(const lumina_weight* w, const float* x, int ldx, int batch, const float* norm_w, float eps,
                   float* y, int ldy, int epi, const float* resid, int ldr, cudaStream_t s, const RopeKV* rk,
                   const L2Prefetch* pf, const TcTp* tp) {
  if (!w->mma || (w->group % 64) || batch < 1 || batch > 4) return LUMINA_E_UNSUPPORTED;
  const int gp = w->group / 64;
  if ((gp & (gp - 1)) || gp > 4) return LUMINA_E_UNSUPPORTED;  // groups of 64, 128, 256 (a unit holds whole groups)
  if ((epi == EPI_SWIGLU || epi == EPI_ROPE_KV) && (w->rows & 1)) {
    set_error("gemv: paired epilogue needs an even row count");
    return LUMINA_E_ARG;
  }
  int* fault = fault_flag_ptr();
  if (!fault) {
    set_error("gemv_tc: fault flag unavailable");
    return LUMINA_E_CUDA;
  }
  const int NB = batch == 1 ? 1 : batch == 2 ? 2 : 4;
  TcArgs a{};
  a.codes = w->codes;
  a.scales = w->scales;
  a.rows = w->rows;
  a.cols = w->cols;
  a.P = w->n_chunks / 2;
  a.ng = w->n_groups;
  a.gsh = gp == 1 ? 0 : gp == 2 ? 1 : 2;
  a.T16 = w->rows_pad / 16;
  a.x = x;
  a.ldx = ldx;
  a.norm_w = norm_w;
  a.eps = eps;
  a.y = y;
  a.ldy = ldy;
  a.resid = resid;
  a.ldr = ldr;
  if (rk) a.rk = *rk;
  a.nb = batch;
  a.lv = (1 << w->bits) - 1;
  a.fault = fault;
  a.spin = wait_spin_limit();
  if (pf) a.pf = *pf;
  const TcTp* tpx = nullptr;
  if (tp && tp->tp > 1) {
    const bool producer = tp->push[0] != nullptr, consumer = tp->in_flags != nullptr;
    if (producer == consumer || (producer && (epi != EPI_STORE || norm_w)) ||
        (consumer && (!norm_w || (epi != EPI_SWIGLU && epi != EPI_ROPE_KV))) || tp->tp > TCTP_MAX) {
      set_error("gemv_tc: a fused exchange needs a storing producer or a normalizing consumer");
      return LUMINA_E_ARG;
    }
    tpx = tp;
  }
  const int es = w->fp16_scales ? 2 : 4;
  // whole tiles per CTA: the smallest grid with the smallest per-CTA share
  const int per = (a.T16 + sm_count() - 1) / sm_count();
  const int grid = (a.T16 + per - 1) / per;
  a.MT = per;
  const size_t budget = 227 * 1024 - 1024;
  const bool norm = norm_w != nullptr;
  // units of 8 pairs when the TS-stage rings fit next to the activation
  // tables, else of 6 or 4 (a unit holds whole scale groups: 2^gsh | KS)
  for (int ks : {8, 6, 4}) {
    if (ks % gp) continue;
    a.UT = (a.P + ks - 1) / ks;
    const int ep_floats = epi == EPI_RESID ? a.MT * 16 * NB : epi == EPI_ROPE_KV && rk ? 2 * NB * (rk->hd / 2) : 0;
    a.x_bytes = (a.P * 2 * NB * 64 + a.P * NB * 8 + a.MT * 4 + TW * 2 * 16 * NB * 4 + ep_floats * 4 + 127) / 128 * 128;
    const int groups = std::max(1, ks >> a.gsh);
    a.stage_bytes = (ks * 512 + groups * 16 * es + 127) / 128 * 128;
    const size_t smem = (size_t)a.x_bytes + (size_t)TW * TS * a.stage_bytes + TW * TS * 8;
    if (smem > budget) continue;
    if (ks == 8) return tc_nb<8>(a, tpx, smem, grid, NB, w->fp16_scales, epi, norm, s);
    if (ks == 6) return tc_nb<6>(a, tpx, smem, grid, NB, w->fp16_scales, epi, norm, s);
    return tc_nb<4>(a, tpx, smem, grid, NB, w->fp16_scales, epi, norm, s);
  }
  return LUMINA_E_UNSUPPORTED;
}

}  // namespace lumina
