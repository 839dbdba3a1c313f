// Multi-row projection (prompt prefill, tree verification) on the 5th-gen
// tensor cores: Y[m, n] = sum_k X[m, k] * W[n, k] for M token rows.
//
// The reference computes fp32 x @ W16 with W16 the fp16-rounded dequantized
// weight (adapters/lumina.py:135-150, chat.py:140, chat.py:239-243 at sq > 1).
// Here W16 is rebuilt on the fly: each K step, the CTA's threads read the
// int4 codes of 128 weight rows x 64 columns (the tensor-core fragment layout
// of weights.cuh, one 16-byte load per thread) and their group scales, and
// write fp16(s * level(c)) into shared memory in the 128-byte-swizzled
// K-major layout that tcgen05.mma reads. The fp32 activations are carried as
// two fp16 planes, x = hi + lo with hi = fp16(x) and lo = fp16(x - hi)
// (act_f16_kernel: RMSNorm fused, K padded to 64), so the product keeps the
// fp32 activations to about 2^-22 relative (one fp16 plane alone rounds them
// to 2^-11, which compounds through the layers of a long prefill). Both
// planes of BN token rows arrive by one TMA box with the same swizzle and
// form a B operand of 2 BN rows. One thread issues tcgen05.mma.kind::f16
// (M = 128 weight rows, N = 2 BN, K = 16, four per K step) accumulating in
// fp32 in tensor memory across the whole K; the epilogue adds column m of
// the hi half to column m of the lo half. tcgen05.commit frees a stage
// when its MMAs have read it. The K loop keeps STAGES stages in flight: while
// the tensor pipe works on step kb, the threads dequantize step kb + STAGES
// - 1 into the stage that step kb - 1 released. After the last step the
// accumulator goes from tensor memory to registers (tcgen05.ld, one TMEM lane
// per weight row per thread) and through the epilogue (store, residual add,
// SwiGLU over interleaved gate/up rows, or the store of q/k/v rows in their
// original order for the RoPE + KV append kernel).
//
// A grid of fewer (row, token) tiles than the GPU has SMs -- few token rows
// (tree verification) or few weight rows (o_proj, down) -- also splits K:
// CTA z of a tile takes K steps [z P / ks, (z + 1) P / ks), writes its fp32
// partial tile to a workspace, and the CTA that draws the tile's last ticket
// adds the ks partials in z order and runs the epilogue.
//
// Waits are bounded: a wait that gives up sets bit 3 of the device fault
// word; the CTA then stops issuing work, lets its TMA loads and MMAs in flight
// finish (waiting with the default limit), frees its tensor memory and exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "gemv_impl.cuh"

namespace lumina {

namespace {

constexpr int G5_BM = 128;                 // weight rows per CTA (the MMA's M)
constexpr int G5_BK = 64;                  // K per stage: one 128-byte swizzle row of fp16
constexpr int G5_SA = 4;                   // weight stages
constexpr int G5_DEQ_WARPS = 8;            // dequantize (one 16-row tile each), then run the epilogue
constexpr int G5_THREADS = 32 * (G5_DEQ_WARPS + 1);  // + the control warp (TMA, MMA, TMEM)
constexpr int G5_A_BYTES = G5_BM * G5_BK * 2;
constexpr int G5_MIN_SPLIT_STEPS = 8;      // K steps per CTA when K is split
constexpr double G5_CTA_OVERHEAD = 4.0;    // a CTA's fixed cost, in K steps

// activation stages (a deeper ring for narrow token tiles, whose stages are
// small) and the shared memory of one CTA
template <int BN>
struct G5Cfg {
  static constexpr int SB = BN <= 32 ? 8 : BN <= 64 ? 6 : 4;
  static constexpr int B_BYTES = 2 * BN * 128;  // hi rows, then lo rows
  static constexpr size_t SMEM = (size_t)G5_SA * G5_A_BYTES + (size_t)SB * B_BYTES + (2 * G5_SA + 2 * SB + 1) * 8 + 1024;
};

// named barrier 1 over the 8 dequantizing warps (the control warp is elsewhere)
__device__ __forceinline__ void g5_bar() { asm volatile("bar.sync 1, %0;" ::"n"(32 * G5_DEQ_WARPS) : "memory"); }
__device__ __forceinline__ bool g5_bar_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(32 * G5_DEQ_WARPS)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

struct G5Args {
  const uint8_t* codes;
  const uint8_t* scales;
  int rows;     // weight rows (N of the projection)
  int P;        // K steps (64-column pairs)
  int ng;       // scale groups per row
  int gsh;      // log2(group / 64)
  int T16;      // 16-row tiles of the weight
  int M;        // token rows
  float* y;
  int ldy;
  const float* resid;
  int ldr;
  int epi;      // G5_STORE, G5_RESID, G5_SWIGLU
  int qk_rows;  // rows < qk_rows hold RoPE pairs adjacent (fused q/k/v): stored at their original index
  int hd;
  int* fault;
  long long spin;
  int ks;       // K splits (grid z)
  float* ws;    // ks > 1: partial tiles, [z][M][rows]
  int* cnt;     // ks > 1: one ticket counter per (row tile, token tile)
};

// ---- tcgen05 / TMA building blocks -----------------------------------------
__device__ __forceinline__ void tc05_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc05_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (stride byte offset), leading byte offset 16 (unused with
// this swizzle), descriptor version 1
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// instruction descriptor, kind::f16: fp16 A and B (K-major), fp32 D, M x N
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tc05_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, int accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
      : "memory");
}
// the mbarrier completes one arrival once every tcgen05 op this thread issued so far is done
__device__ __forceinline__ void tc05_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// box {64 columns, 128 rows} at (c0, c1): a dense fp16 weight tile
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// box {64 columns, BN rows, 2 planes} at (c0, c1, 0)
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(0), "r"(smem_u32(bar))
      : "memory");
}

// 16 fp32 columns of this warp's 32 TMEM lanes (one lane = one row per thread)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- dequantization of one K step ------------------------------------------
// Thread (warp T, lane L = 4g + t) owns the 16-byte fragment word of 16-row
// tile T at each K step: rows 16T + g (low nibbles) and 16T + g + 8 (high
// nibbles), columns 32(j >> 1) + 16(j & 1) + 4t + q of byte q of word j.
// The word and the two rows' group scales are loaded G5_PD steps before they
// are dequantized (a register queue), so no step waits on its own load. Step
// p lives in slot p mod G5_PD for its whole time in the queue: every slot is
// named by a constant, so no queue entry is ever moved -- moving a register
// whose load is still in flight would wait for that load.
// Each run of four columns becomes one 8-byte store of four fp16 values at
// the 128-byte-swizzled position: row r at r * 128, 16-byte chunk
// (col / 8) XOR (r mod 8).
constexpr int G5_PD = 8;  // K steps between a code load and its use

struct G5Frag {
  uint4 q;
  float s0, s1;
};

template <typename ST>
__device__ __forceinline__ G5Frag g5_load(const G5Args& a, int n0, int kb, int kb_end, int tid) {
  const int T = tid >> 5, L = tid & 31, g = L >> 2;
  const int gt = (n0 >> 4) + T;
  G5Frag f{make_uint4(0u, 0u, 0u, 0u), 0.f, 0.f};
  if (gt < a.T16 && kb < kb_end) {
    f.q = ldg_stream(a.codes + (((size_t)gt * a.P + kb) * 32 + L) * 16);
    const uint8_t* sp = a.scales + (((size_t)gt * a.ng + (kb >> a.gsh)) * 8 + g) * 2 * sizeof(ST);
    if constexpr (sizeof(ST) == 2) {
      const __half2 h = *reinterpret_cast<const __half2*>(sp);
      f.s0 = __low2float(h);
      f.s1 = __high2float(h);
    } else {
      const float2 v = *reinterpret_cast<const float2*>(sp);
      f.s0 = v.x;
      f.s1 = v.y;
    }
  }
  return f;
}

__device__ __forceinline__ void g5_dequant(const G5Frag& fr, uint8_t* As, int tid) {
  const int T = tid >> 5, L = tid & 31, g = L >> 2, t = L & 3;
  const int r0 = 16 * T + g, r1 = r0 + 8;
  // w = s * (-1 + c * 2/15) = c * (2s/15) - s (adapters/lumina.py:135-139), in fp32, then fp16
  const float k0 = fr.s0 * (2.0f / 15.0f), k1 = fr.s1 * (2.0f / 15.0f);
  const uint32_t words[4] = {fr.q.x, fr.q.y, fr.q.z, fr.q.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c0 = (j >> 1) * 32 + (j & 1) * 16 + t * 4;
    const uint32_t lo = words[j] & 0x0F0F0F0Fu, hi = (words[j] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t src = h ? hi : lo;
      const float kk = h ? k1 : k0, ss = h ? fr.s1 : fr.s0;
      float f[4];
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        // 0x4B0000cc = 2^23 + c as fp32
        const float m = __int_as_float((int)__byte_perm(src, 0x4B000000u, 0x7440u + b)) - 8388608.0f;
        f[b] = fmaf(m, kk, -ss);
      }
      const __half2 p0 = __floats2half2_rn(f[0], f[1]), p1 = __floats2half2_rn(f[2], f[3]);
      const int r = h ? r1 : r0;
      uint8_t* dst = As + r * 128 + (((c0 >> 3) ^ (r & 7)) << 4) + ((c0 & 7) << 1);
      asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(smem_u32(dst)), "r"(*reinterpret_cast<const uint32_t*>(&p0)),
                   "r"(*reinterpret_cast<const uint32_t*>(&p1))
                   : "memory");
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor pipe
}

// the register queue over K steps [begin, end): local step p in slot p % G5_PD
template <typename ST>
struct G5Queue {
  G5Frag e[G5_PD];
  int begin, end;
  __device__ __forceinline__ void init(const G5Args& a, int n0, int begin_, int end_, int tid) {
    begin = begin_;
    end = end_;
#pragma unroll
    for (int i = 0; i < G5_PD; ++i) e[i] = g5_load<ST>(a, n0, begin + i, end, tid);
  }
  template <int SLOT>
  __device__ __forceinline__ void pop_at(const G5Args& a, uint8_t* As, int n0, int tid, int p) {
    g5_dequant(e[SLOT], As, tid);
    e[SLOT] = g5_load<ST>(a, n0, begin + p + G5_PD, end, tid);
  }
  // dequantize local step p (steps are popped in order) into As and load
  // step p + G5_PD into its slot
  __device__ __forceinline__ void pop(const G5Args& a, uint8_t* As, int n0, int tid, int p) {
    static_assert(G5_PD == 8, "one case per slot");
    switch (p & (G5_PD - 1)) {
      case 0: pop_at<0>(a, As, n0, tid, p); break;
      case 1: pop_at<1>(a, As, n0, tid, p); break;
      case 2: pop_at<2>(a, As, n0, tid, p); break;
      case 3: pop_at<3>(a, As, n0, tid, p); break;
      case 4: pop_at<4>(a, As, n0, tid, p); break;
      case 5: pop_at<5>(a, As, n0, tid, p); break;
      case 6: pop_at<6>(a, As, n0, tid, p); break;
      default: pop_at<7>(a, As, n0, tid, p); break;
    }
  }
};

// RoPE pair permutation of the fused q/k/v weight: row 2p + e of a head is
// the original row p + e * hd / 2
__device__ __forceinline__ int g5_orig_row(const G5Args& a, int row) {
  if (row >= a.qk_rows) return row;
  const int h = row / a.hd, rr = row - h * a.hd;
  return h * a.hd + (rr >> 1) + (rr & 1) * (a.hd >> 1);
}

// epilogue of 16 token columns mb .. mb + 15 of this thread's weight row
// (every lane of the warp calls it: SwiGLU takes the up row from lane + 1)
__device__ __forceinline__ void g5_emit(const G5Args& a, int row, int mb, const float (&v)[16], int lane) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int m = mb + j;
    if (a.epi == G5_SWIGLU) {
      const float up = __shfl_down_sync(0xffffffffu, v[j], 1);
      if (m < a.M && !(lane & 1) && row + 1 < a.rows) {
        const float gt = v[j];
        const float e = expf(-fminf(fmaxf(gt, -40.f), 40.f));  // chat.py:300-302
        a.y[(size_t)m * a.ldy + (row >> 1)] = gt / (1.0f + e) * up;
      }
    } else if (m < a.M && row < a.rows) {
      if (a.epi == G5_RESID)
        a.y[(size_t)m * a.ldy + row] = a.resid[(size_t)m * a.ldr + row] + v[j];
      else
        a.y[(size_t)m * a.ldy + g5_orig_row(a, row)] = v[j];
    }
  }
}

// One CTA: 8 dequantizing warps (warp T rebuilds 16-row tile T of each K
// step into the weight stage, then runs the epilogue) and a control warp
// whose lane 0 moves the activation tiles by TMA and issues the MMAs. The
// two sides meet only at mbarriers: full_a (the 8 warps wrote a weight
// stage), full_b (an activation stage landed), empty_a / empty_b (the MMAs
// of a step finished reading its stages, tcgen05.commit), accum (every MMA
// done). No CTA-wide barrier sits in the K loop, so every warp runs ahead
// as far as its stages allow.
//
// DENSE: the weight is an fp16 matrix (the LM head) whose 128 x 64 tiles
// arrive by TMA (tensor map tmw, same swizzle) instead of being rebuilt from
// codes; ST is then unused and the 8 warps only run the epilogue.
template <int BN, typename ST, bool DENSE>
__global__ void __launch_bounds__(G5_THREADS, 1)
gemm_tc05_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw, G5Args a) {
  static_assert(2 * BN <= 256, "hi and lo planes form one MMA of N = 2 BN <= 256");
  using C = G5Cfg<BN>;
  constexpr int SA = G5_SA, SB = C::SB;
  constexpr uint32_t IDESC = idesc_f16(G5_BM, 2 * BN);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* Bst = smem + SA * G5_A_BYTES;                                  // activation stages
  uint64_t* full_a = reinterpret_cast<uint64_t*>(Bst + SB * C::B_BYTES);  // weight stage written / landed
  uint64_t* empty_a = full_a + SA;                                        // weight stage read by its MMAs
  uint64_t* full_b = empty_a + SA;                                        // activation stage landed
  uint64_t* empty_b = full_b + SB;                                        // activation stage read
  uint64_t* accum = empty_b + SB;                                         // every MMA done
  __shared__ uint32_t tmem_base;
  __shared__ int abort_s, last_s;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * G5_BM, m0 = blockIdx.y * BN;
  // this CTA's K steps: kb0 + p for p < KB
  const int z = blockIdx.z;
  const int kb0 = (int)((long long)a.P * z / a.ks), KB = (int)((long long)a.P * (z + 1) / a.ks) - kb0;

  if (tid == 0) {
    for (int i = 0; i < SA; ++i) {
      mbar_init(&full_a[i], DENSE ? 1 : G5_DEQ_WARPS);
      mbar_init(&empty_a[i], 1);
    }
    for (int i = 0; i < SB; ++i) {
      mbar_init(&full_b[i], 1);
      mbar_init(&empty_b[i], 1);
    }
    mbar_init(accum, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    abort_s = 0;
  }
  if (warp == G5_DEQ_WARPS) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(2 * BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc05_fence_before();
  __syncthreads();
  tc05_fence_after();
  const uint32_t tmem = tmem_base;
  pdl_launch_dependents();
  volatile int* abort_v = &abort_s;

  if (warp < G5_DEQ_WARPS) {
    // ---- dequantizing warps: weights never depend on the previous kernel,
    // so they stream from the first instruction
    if constexpr (!DENSE) {
      G5Queue<ST> wq;
      wq.init(a, n0, kb0, kb0 + KB, tid);
      for (int p = 0; p < KB; ++p) {
        const int s = p % SA;
        if (p >= SA) {
          // the stage's previous step (p - SA) must have been read by its MMAs
          const bool freed = mbar_wait_bounded(&empty_a[s], (uint32_t)((p / SA - 1) & 1), a.spin);
          if (!__all_sync(0xffffffffu, freed)) {
            if (lane == 0) {
              atomicOr(a.fault, 8);
              *abort_v = 1;
            }
            break;
          }
        }
        if (*abort_v) break;
        wq.pop(a, smem + s * G5_A_BYTES, n0, tid, p);  // ends with the async-proxy fence
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_a[s]);
      }
    }
  } else if (lane == 0) {
    // ---- control thread: activation (and, DENSE, weight) tiles by TMA, MMAs
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmx) : "memory");
    int a_issued = 0, a_landed = 0, b_issued = 0, b_landed = 0;
    if constexpr (DENSE) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tmw) : "memory");
      for (int p = 0; p < SA && p < KB; ++p, ++a_issued) {
        mbar_expect_tx(&full_a[p], G5_A_BYTES);
        tma_load_2d(smem + p * G5_A_BYTES, &tmw, (kb0 + p) * G5_BK, n0, &full_a[p]);
      }
    }
    pdl_wait();  // the activation rows come from the previous kernel
    for (int p = 0; p < SB && p < KB; ++p, ++b_issued) {
      mbar_expect_tx(&full_b[p], C::B_BYTES);
      tma_load_3d(Bst + p * C::B_BYTES, &tmx, (kb0 + p) * G5_BK, m0, &full_b[p]);
    }
    for (int p = 0; p < KB; ++p) {
      const int sa = p % SA, sb = p % SB;
      bool ok = mbar_wait_bounded(&full_a[sa], (uint32_t)((p / SA) & 1), a.spin);
      if (ok && DENSE) ++a_landed;
      ok = ok && mbar_wait_bounded(&full_b[sb], (uint32_t)((p / SB) & 1), a.spin);
      if (ok) ++b_landed;
      if (!ok || *abort_v) {
        if (!ok) atomicOr(a.fault, 8);
        *abort_v = 1;
        break;
      }
      tc05_fence_after();
      const uint32_t sa_addr = smem_u32(smem + sa * G5_A_BYTES), sb_addr = smem_u32(Bst + sb * C::B_BYTES);
#pragma unroll
      for (int kk = 0; kk < G5_BK / 16; ++kk)
        tc05_mma(tmem, smem_desc_sw128(sa_addr + kk * 32), smem_desc_sw128(sb_addr + kk * 32), IDESC, (p | kk) != 0);
      tc05_commit(&empty_a[sa]);
      tc05_commit(&empty_b[sb]);
      // refill the stages of step p - 1 (its MMAs were issued one step ago)
      // with step p - 1 + SB (activations) and, DENSE, p - 1 + SA (weights)
      if (p >= 1) {
        const int q = p - 1;
        const bool nb = q + SB < KB, na = DENSE && q + SA < KB;
        if (nb || na) {
          bool freed = true;
          if (nb) freed = mbar_wait_bounded(&empty_b[q % SB], (uint32_t)((q / SB) & 1), a.spin);
          if (freed && na) freed = mbar_wait_bounded(&empty_a[q % SA], (uint32_t)((q / SA) & 1), a.spin);
          if (!freed) {
            atomicOr(a.fault, 8);
            *abort_v = 1;
            break;
          }
          if (nb) {
            mbar_expect_tx(&full_b[q % SB], C::B_BYTES);
            tma_load_3d(Bst + (q % SB) * C::B_BYTES, &tmx, (kb0 + q + SB) * G5_BK, m0, &full_b[q % SB]);
            ++b_issued;
          }
          if (na) {
            mbar_expect_tx(&full_a[q % SA], G5_A_BYTES);
            tma_load_2d(smem + (q % SA) * G5_A_BYTES, &tmw, (kb0 + q + SA) * G5_BK, n0, &full_a[q % SA]);
            ++a_issued;
          }
        }
      }
    }
    if (*abort_v) {
      // let every tile load in flight land before the stages go away
      for (int i = b_landed; i < b_issued; ++i) mbar_wait_bounded(&full_b[i % SB], (uint32_t)((i / SB) & 1));
      for (int i = a_landed; i < a_issued; ++i) mbar_wait_bounded(&full_a[i % SA], (uint32_t)((i / SA) & 1));
    }
    tc05_commit(accum);  // completes once every MMA issued above is done
  }

  if (warp < G5_DEQ_WARPS) {
    // ---- epilogue (the 8 warps; named barrier 1 spans them only)
    const bool done = mbar_wait_bounded(accum, 0u, MBAR_SPIN_LIMIT);
    tc05_fence_after();
    pdl_wait();  // outputs and residual rows may belong to earlier kernels
    if (!done && lane == 0) atomicOr(a.fault, 8);
    const bool all_ok = g5_bar_and(done && !*abort_v);
    // warp w reads TMEM lanes 32 (w % 4) .. + 31 (weight rows) and token
    // columns [BN/2 (w / 4), BN/2 (w / 4 + 1)) of both planes
    const int quarter = warp & 3, half = warp >> 2;
    const int row = n0 + 32 * quarter + lane;
    constexpr int COLS = BN / 2;
    if (a.ks == 1) {
      if (all_ok) {
        for (int c0 = half * COLS; c0 < (half + 1) * COLS; c0 += 16) {
          float v[16], lo[16];
          const uint32_t ta = tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)c0;
          __syncwarp();
          tmem_ld16(ta, v);
          tmem_ld16(ta + (uint32_t)BN, lo);
          if (m0 + c0 >= a.M) continue;  // warp-uniform: the loads above are collective
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] += lo[j];
          g5_emit(a, row, m0 + c0, v, lane);
        }
      }
    } else {
      // split K: the partial tile to ws[z][m][row]; every CTA of the tile
      // takes a ticket (an aborted CTA too, so the counter returns to zero)
      if (all_ok) {
        for (int c0 = half * COLS; c0 < (half + 1) * COLS; c0 += 16) {
          float v[16], lo[16];
          const uint32_t ta = tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)c0;
          __syncwarp();
          tmem_ld16(ta, v);
          tmem_ld16(ta + (uint32_t)BN, lo);
          if (row < a.rows) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int m = m0 + c0 + j;
              if (m < a.M) a.ws[((size_t)z * a.M + m) * a.rows + row] = v[j] + lo[j];
            }
          }
        }
      }
      __threadfence();
      g5_bar();
      const int tile = blockIdx.y * gridDim.x + blockIdx.x;
      if (tid == 0) last_s = atomicAdd(&a.cnt[tile], 1) == a.ks - 1;
      g5_bar();
      if (last_s) {
        __threadfence();
        for (int c0 = half * COLS; c0 < (half + 1) * COLS; c0 += 16) {
          if (m0 + c0 >= a.M) break;  // warp-uniform
          float v[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + c0 + j;
            float acc = 0.f;
            if (m < a.M && row < a.rows)
              for (int zz = 0; zz < a.ks; ++zz) acc += __ldcg(a.ws + ((size_t)zz * a.M + m) * a.rows + row);
            v[j] = acc;
          }
          g5_emit(a, row, m0 + c0, v, lane);
        }
        if (tid == 0) a.cnt[tile] = 0;
      }
    }
  }
  tc05_fence_before();
  __syncthreads();
  if (warp == G5_DEQ_WARPS) {
    // no MMA may still write the accumulator when it is freed (the epilogue's
    // wait can only have given up on a failed CTA)
    if (lane == 0) mbar_wait_bounded(accum, 0u, MBAR_SPIN_LIMIT);
    __syncwarp();
    tc05_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN) : "memory");
  }
}

// fp32 rows (optionally RMS-normalized, chat.py:63-66) -> two planes of fp16
// rows of Kpad columns, hi = fp16(v) at out[m], lo = fp16(v - hi) at
// out[M + m]; zeros past K
template <bool NORM>
__global__ void __launch_bounds__(256) act_f16_kernel(const float* __restrict__ x, int ldx, int K, int Kpad, int M,
                                                      const float* __restrict__ nw, float eps, __half* __restrict__ out) {
  __shared__ float red[8];
  const int m = blockIdx.x, tid = threadIdx.x;
  pdl_launch_dependents();
  pdl_wait();
  const float* xr = x + (size_t)m * ldx;
  float rinv = 1.f;
  if constexpr (NORM) {
    float ss = 0.f;
    for (int k = tid; k < K; k += 256) ss = fmaf(xr[k], xr[k], ss);
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += red[w];
    rinv = 1.0f / sqrtf(tot / (float)K + eps);
  }
  __half* o = out + (size_t)m * Kpad;
  __half* ol = out + (size_t)(M + m) * Kpad;
  for (int k = 2 * tid; k < Kpad; k += 512) {
    float v0 = 0.f, v1 = 0.f;
    if (k < K) v0 = NORM ? (xr[k] * rinv) * nw[k] : xr[k];
    if (k + 1 < K) v1 = NORM ? (xr[k + 1] * rinv) * nw[k + 1] : xr[k + 1];
    const __half2 hi = __floats2half2_rn(v0, v1);
    *reinterpret_cast<__half2*>(o + k) = hi;
    *reinterpret_cast<__half2*>(ol + k) = __floats2half2_rn(v0 - __low2float(hi), v1 - __high2float(hi));
  }
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::mutex mu;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      cudaGetLastError();
  }
  return fn;
}

template <int BN, typename ST, bool DENSE = false>
int g5_launch(const CUtensorMap& map, const G5Args& a, cudaStream_t s, const CUtensorMap* wmap = nullptr) {
  auto kern = gemm_tc05_kernel<BN, ST, DENSE>;
  const size_t smem = G5Cfg<BN>::SMEM;
  const int rc = set_smem_limit((const void*)kern, smem, "gemm_tc05");
  if (rc) return rc;
  const dim3 grid((a.rows + G5_BM - 1) / G5_BM, (a.M + BN - 1) / BN, a.ks);
  const cudaError_t e = launch_pdl(kern, grid, dim3(G5_THREADS), smem, s, map, wmap ? *wmap : map, a);
  if (e != cudaSuccess) {
    set_error("gemm_tc05 launch: %s", cudaGetErrorString(e));
    return LUMINA_E_CUDA;
  }
  return LUMINA_OK;
}

template <typename ST>
int g5_bn(const CUtensorMap& map, const G5Args& a, int bn, cudaStream_t s) {
  switch (bn) {
    case 32: return g5_launch<32, ST>(map, a, s);
    case 64: return g5_launch<64, ST>(map, a, s);
    default: return g5_launch<128, ST>(map, a, s);
  }
}

// per-device fp16 activation rows for lumina_gemm_rows (grown on demand)
int x16_scratch(int device, size_t elems, __half** out) {
  static std::mutex mu;
  static __half* buf[64] = {};
  static size_t cap[64] = {};
  if (device < 0 || device >= 64) {
    set_error("gemm_rows: bad device %d", device);
    return LUMINA_E_ARG;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (cap[device] < elems) {
    if (buf[device]) {
      cudaDeviceSynchronize();  // queued work may still read the smaller buffer
      cudaFree(buf[device]);
      buf[device] = nullptr;
      cap[device] = 0;
    }
    const size_t want = std::max(elems, (size_t)1 << 20);
    if (cudaMalloc(&buf[device], want * 2) != cudaSuccess) {
      cudaGetLastError();
      set_error("gemm_rows: cudaMalloc of %zu bytes failed", want * 2);
      return LUMINA_E_OOM;
    }
    cap[device] = want;
  }
  *out = buf[device];
  return LUMINA_OK;
}

// 1) the activation rows -> fp16 hi and lo planes (RMSNorm fused when
// norm_w is given); 2) the token tile and K splits; 3) the planes' tensor map
int g5_prepare(const float* x, int ldx, int M, int K, int P, const float* norm_w, float eps, __half* x16, int rows,
               const SplitWork* sw, cudaStream_t s, int* bn_out, int* ks_out, CUtensorMap* map) {
  auto encode = tensor_map_encoder();
  if (!encode) {
    set_error("gemm_tc05: cuTensorMapEncodeTiled unavailable");
    return LUMINA_E_CUDA;
  }
  const int Kpad = P * 64;
  {
    const cudaError_t e = norm_w ? launch_pdl(act_f16_kernel<true>, dim3(M), dim3(256), 0, s, x, ldx, K, Kpad, M,
                                              norm_w, eps, x16)
                                 : launch_pdl(act_f16_kernel<false>, dim3(M), dim3(256), 0, s, x, ldx, K, Kpad, M,
                                              norm_w, eps, x16);
    if (e != cudaSuccess) {
      set_error("act_f16 launch: %s", cudaGetErrorString(e));
      return LUMINA_E_CUDA;
    }
  }
  // the token tile: the smallest that covers M (at most 128: the two planes
  // make N = 2 BN), halved (not below 64) while the grid leaves SMs idle --
  // weights of few 128-row tiles (o_proj, down: 32) would otherwise run on a
  // fraction of the GPU
  int bn = M <= 32 ? 32 : M <= 64 ? 64 : 128;
  const int row_tiles = (rows + G5_BM - 1) / G5_BM;
  while (bn > 64 && row_tiles * ((M + bn - 1) / bn) < sm_count()) bn /= 2;
  // K splits: one CTA per SM, so a grid of `tiles` x ks CTAs runs in
  // ceil(tiles ks / SMs) waves of P / ks steps (plus about G5_CTA_OVERHEAD
  // steps of pipeline fill and epilogue each); take the ks with the fewest
  // step-times, at least G5_MIN_SPLIT_STEPS K steps per CTA, partials
  // within the workspace
  const int tiles = row_tiles * ((M + bn - 1) / bn);
  int ks = 1;
  if (sw && sw->ws && sw->cnt && tiles <= sw->cnt_n) {
    const int sms = sm_count();
    double best = 1e30;
    for (int k = 1; k <= std::max(1, P / G5_MIN_SPLIT_STEPS); ++k) {
      if (k > 1 && (size_t)k * M * rows > sw->ws_elems) break;
      const double t = (double)((tiles * k + sms - 1) / sms) * ((double)P / k + G5_CTA_OVERHEAD);
      if (t < best - 1e-9) {
        best = t;
        ks = k;
      }
    }
  }
  // the fp16 planes as a 3-D tensor (K innermost, rows, plane), boxes of
  // 64 x BN x 2, 128-byte swizzle: a stage holds BN hi rows then BN lo rows
  const cuuint64_t dims[3] = {(cuuint64_t)Kpad, (cuuint64_t)M, 2};
  const cuuint64_t strides[2] = {(cuuint64_t)Kpad * 2, (cuuint64_t)M * Kpad * 2};
  const cuuint32_t box[3] = {(cuuint32_t)G5_BK, (cuuint32_t)bn, 2};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult cr = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, x16, dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) {
    set_error("gemm_tc05: tensor map encode failed (%d)", (int)cr);
    return LUMINA_E_CUDA;
  }
  *bn_out = bn;
  *ks_out = ks;
  return LUMINA_OK;
}

}  // namespace

int split_scratch(int device, SplitWork* out) {
  static std::mutex mu;
  static SplitWork work[64];
  if (device < 0 || device >= 64) {
    set_error("split workspace: bad device %d", device);
    return LUMINA_E_ARG;
  }
  std::lock_guard<std::mutex> lk(mu);
  SplitWork& sw = work[device];
  if (!sw.ws) {
    float* ws = nullptr;
    int* cnt = nullptr;
    if (cudaMalloc(&ws, SPLIT_WS_ELEMS * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&cnt, SPLIT_COUNTERS * sizeof(int)) != cudaSuccess ||
        cudaMemset(cnt, 0, SPLIT_COUNTERS * sizeof(int)) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {  // zeroed before any stream uses it
      cudaGetLastError();
      if (ws) cudaFree(ws);
      if (cnt) cudaFree(cnt);
      set_error("split workspace: cudaMalloc failed");
      return LUMINA_E_OOM;
    }
    sw.ws = ws;
    sw.ws_elems = SPLIT_WS_ELEMS;
    sw.cnt = cnt;
    sw.cnt_n = SPLIT_COUNTERS;
  }
  *out = sw;
  return LUMINA_OK;
}

size_t gemm_tc05_x16_elems(int rows, int cols) { return 2 * (size_t)rows * (size_t)((cols + 63) / 64 * 64); }

int gemm_tc05_launch(const lumina_weight* w, const float* x, int ldx, int M, const float* norm_w, float eps,
                     __half* x16, float* y, int ldy, int epi, const float* resid, int ldr, int qk_rows, int hd,
                     cudaStream_t s, const SplitWork* sw) {
  if (!w->mma || w->bits != 4 || (w->group % 64) || M < 1) return LUMINA_E_UNSUPPORTED;
  const int gp = w->group / 64;
  if ((gp & (gp - 1)) || gp > 4) return LUMINA_E_UNSUPPORTED;
  if (epi != G5_STORE && epi != G5_RESID && epi != G5_SWIGLU) return LUMINA_E_UNSUPPORTED;
  if (epi == G5_SWIGLU && (w->rows & 1)) {
    set_error("gemm_tc05: SwiGLU needs an even row count");
    return LUMINA_E_ARG;
  }
  int* fault = fault_flag_ptr();
  if (!fault) {
    set_error("gemm_tc05: fault flag unavailable");
    return LUMINA_E_CUDA;
  }
  const int P = w->n_chunks / 2;
  int bn = 0, ks = 1;
  CUtensorMap map;
  if (const int rc = g5_prepare(x, ldx, M, w->cols, P, norm_w, eps, x16, w->rows, sw, s, &bn, &ks, &map)) return rc;
  G5Args a{};
  a.codes = w->codes;
  a.scales = w->scales;
  a.rows = w->rows;
  a.P = P;
  a.ng = w->n_groups;
  a.gsh = gp == 1 ? 0 : gp == 2 ? 1 : 2;
  a.T16 = w->rows_pad / 16;
  a.M = M;
  a.y = y;
  a.ldy = ldy;
  a.resid = resid;
  a.ldr = ldr;
  a.epi = epi;
  a.qk_rows = qk_rows;
  a.hd = hd > 0 ? hd : 1;
  a.fault = fault;
  a.spin = wait_spin_limit();
  a.ks = ks;
  a.ws = ks > 1 ? sw->ws : nullptr;
  a.cnt = ks > 1 ? sw->cnt : nullptr;
  return w->fp16_scales ? g5_bn<__half>(map, a, bn, s) : g5_bn<float>(map, a, bn, s);
}

int dense_tc05_launch(const __half* W, int rows, int K, const float* x, int ldx, int M, __half* x16, float* y,
                      int ldy, cudaStream_t s, const SplitWork* sw) {
  if (M < 1 || rows < 1 || K < 1 || (K % 8)) return LUMINA_E_UNSUPPORTED;
  auto encode = tensor_map_encoder();
  int* fault = fault_flag_ptr();
  if (!encode || !fault) {
    set_error("gemm_tc05 (dense): tensor map encoder or fault flag unavailable");
    return LUMINA_E_CUDA;
  }
  const int P = (K + G5_BK - 1) / G5_BK;
  int bn = 0, ks = 1;
  CUtensorMap map, wmap;
  if (const int rc = g5_prepare(x, ldx, M, K, P, nullptr, 0.f, x16, rows, sw, s, &bn, &ks, &map)) return rc;
  // the weight rows as a 2-D tensor (K innermost), 64 x 128 boxes; columns
  // past K and rows past `rows` read as zeros
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {(cuuint32_t)G5_BK, (cuuint32_t)G5_BM};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult cr = encode(&wmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(W), dims, strides, box,
                             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) {
    set_error("gemm_tc05 (dense): tensor map encode failed (%d)", (int)cr);
    return LUMINA_E_CUDA;
  }
  G5Args a{};
  a.rows = rows;
  a.P = P;
  a.M = M;
  a.y = y;
  a.ldy = ldy;
  a.epi = G5_STORE;
  a.hd = 1;
  a.fault = fault;
  a.spin = wait_spin_limit();
  a.ks = ks;
  a.ws = ks > 1 ? sw->ws : nullptr;
  a.cnt = ks > 1 ? sw->cnt : nullptr;
  switch (bn) {
    case 32: return g5_launch<32, float, true>(map, a, s, &wmap);
    case 64: return g5_launch<64, float, true>(map, a, s, &wmap);
    default: return g5_launch<128, float, true>(map, a, s, &wmap);
  }
}

}  // namespace lumina

extern "C" int lumina_gemm_rows(const lumina_weight* w, const float* x_dev, int rows, int ldx, float* y_dev, int ldy,
                                void* stream) {
  using namespace lumina;
  LUMINA_CHECK_ARG(w && x_dev && y_dev, "gemm_rows: null pointer");
  LUMINA_CHECK_ARG(rows >= 1, "gemm_rows: %d rows", rows);
  LUMINA_CHECK_ARG(ldx >= w->cols && ldy >= w->rows, "gemm_rows: ldx %d / ldy %d smaller than (%d, %d)", ldx, ldy,
                   w->cols, w->rows);
  if (!w->mma || w->bits != 4) {
    set_error("gemm_rows: built for int4 weights in the tensor-core fragment layout");
    return LUMINA_E_UNSUPPORTED;
  }
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != w->device) cudaSetDevice(w->device);
  __half* x16 = nullptr;
  SplitWork sw;
  int rc = x16_scratch(w->device, gemm_tc05_x16_elems(rows, w->cols), &x16);
  if (!rc) rc = split_scratch(w->device, &sw);
  if (!rc)
    rc = gemm_tc05_launch(w, x_dev, ldx, rows, nullptr, 0.f, x16, y_dev, ldy, G5_STORE, nullptr, 0, 0, 0,
                          (cudaStream_t)stream, &sw);
  if (prev >= 0 && prev != w->device) cudaSetDevice(prev);
  return rc;
}
