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
constexpr int G5_DEQ_WARPS = 8;            // dequantize (one 16-row tile each), then run the epilogue
constexpr int G5_MMA_WARP = G5_DEQ_WARPS;  // tensor memory and the MMAs
constexpr int G5_THREADS = 32 * (G5_DEQ_WARPS + 2);  // + the MMA warp + the TMA warp
constexpr int G5_A_BYTES = G5_BM * G5_BK * 2;
constexpr int G5_MIN_SPLIT_STEPS = 8;      // K steps per CTA when K is split
constexpr double G5_CTA_OVERHEAD = 4.0;    // a CTA's fixed cost, in K steps

// A stage holds G5_KS K steps: [weight tiles | activation tiles], G5_KS of
// each. S stages, code chunks of CK steps, RC chunk slots per dequantizing
// warp; shared memory of one CTA: [stages][code rings][mbarriers]
constexpr int G5_KS = 2;
template <int BN>
struct G5Cfg {
  static constexpr int B_BYTES = 2 * BN * 128;  // one step's activations: hi rows, then lo rows
  static constexpr int STAGE = G5_KS * (G5_A_BYTES + B_BYTES);
  static constexpr int S = BN <= 32 ? 3 : 2;
  static constexpr int CK = BN <= 64 ? 4 : 2;
  static constexpr int RC = BN <= 64 ? 4 : 3;
  static constexpr int RING_SLOT = CK * 512 + CK * 16 * 4;  // G5Ring<CK>::SLOT
  static constexpr int RING_BYTES = 8 * RC * RING_SLOT;
  static constexpr int N_BARS = 3 * S + 1 + 8 * RC;
  static constexpr size_t SMEM = (size_t)S * STAGE + RING_BYTES + N_BARS * 8 + 1024;
  static_assert(SMEM <= 227 * 1024, "shared memory of one CTA");
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
// Each run of four columns becomes one 8-byte store of four fp16 values at
// the 128-byte-swizzled position: row r at r * 128, 16-byte chunk
// (col / 8) XOR (r mod 8).
//
// The codes and scales reach shared memory by bulk asynchronous copies, not
// by loads of the dequantizing threads: every step ends with a release (the
// async-proxy fence and the mbarrier arrive that hand the stage to the MMA),
// and a release waits for the thread's own loads still in flight -- with
// the weights loaded by the threads themselves, every step would wait one
// HBM latency. Lane 0 of warp T streams tile T's codes through a ring of
// RC chunks of CK steps (tile T's codes of consecutive K steps are
// contiguous, 512 bytes a step, and so are its scale groups), each chunk
// completing an mbarrier; the warp reads a step's word and scales with
// shared loads.
struct G5Frag {
  uint4 q;
  float s0, s1;
};

// a chunk slot of CK steps: codes, then up to CK scale groups of 16 rows
template <int CK>
struct G5Ring {
  static constexpr int CODE_BYTES = CK * 512;
  static constexpr int SLOT = CODE_BYTES + CK * 16 * 4;
};

// chunk c (local) of this warp's tile: steps [c CK, min((c + 1) CK, KB)) of
// the CTA's range starting at kb0, and the scale groups they use
template <typename ST, int CK>
__device__ __forceinline__ void g5_fetch(const G5Args& a, int gt, int kb0, int KB, int c, uint8_t* slot,
                                         uint64_t* bar) {
  const int p0 = c * CK, ns = min(CK, KB - p0);
  const int g0 = (kb0 + p0) >> a.gsh, g1 = (kb0 + p0 + ns - 1) >> a.gsh;
  const uint32_t cb = (uint32_t)ns * 512u, sb = (uint32_t)(g1 - g0 + 1) * 16u * (uint32_t)sizeof(ST);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the warp's reads of the slot come first
  mbar_expect_tx(bar, cb + sb);
  bulk_g2s(slot, a.codes + ((size_t)gt * a.P + kb0 + p0) * 512, cb, bar);
  bulk_g2s(slot + G5Ring<CK>::CODE_BYTES, a.scales + ((size_t)gt * a.ng + g0) * 16 * sizeof(ST), sb, bar);
}

// local step p's fragment from its chunk slot
template <typename ST, int CK>
__device__ __forceinline__ G5Frag g5_read(const G5Args& a, const uint8_t* slot, int kb0, int p, int lane) {
  const int g = lane >> 2, i = p % CK;
  const int grp = ((kb0 + p) >> a.gsh) - ((kb0 + p - i) >> a.gsh);
  G5Frag f;
  f.q = *reinterpret_cast<const uint4*>(slot + i * 512 + lane * 16);
  const uint8_t* sp = slot + G5Ring<CK>::CODE_BYTES + (grp * 8 + g) * 2 * sizeof(ST);
  if constexpr (sizeof(ST) == 2) {
    const __half2 h = *reinterpret_cast<const __half2*>(sp);
    f.s0 = __low2float(h);
    f.s1 = __high2float(h);
  } else {
    const float2 v = *reinterpret_cast<const float2*>(sp);
    f.s0 = v.x;
    f.s1 = v.y;
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
}

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

// One CTA, three roles that meet only at mbarriers (no CTA-wide barrier in
// the K loop, so every warp runs ahead as far as the stages allow):
//  * warps 0-7 dequantize (warp T rebuilds 16-row tile T of each K step into
//    the stage's weight tile) and later run the epilogue;
//  * warp 8 owns the tensor memory, and its lane 0 issues the MMAs: one wait
//    on the stage's `full` barrier, four tcgen05.mma, one tcgen05.commit to
//    the stage's `empty` barrier per K step;
//  * warp 9's lane 0 moves the activation tiles (and, DENSE, the weight
//    tiles) by TMA, counting their bytes on the same `full` barrier.
// A stage is [weight tile | activation tile]. `tiles` completes when the
// stage's TMA bytes landed; warp 0 waits for it before it arrives on `full`,
// which completes when the 8 dequantizing warps arrived; `empty` completes
// when the step's MMAs have read the stage. Each mbarrier wait costs a couple
// of hundred cycles even when its phase is already complete, so the MMA
// thread, which sets the pace, waits once per step (DENSE: on `tiles`).
//
// DENSE: the weight is an fp16 matrix (the LM head) whose 128 x 64 tiles
// arrive by TMA (tensor map tmw, same swizzle) instead of being rebuilt from
// codes; ST is then unused and the 8 warps only run the epilogue.
template <int BN, typename ST, bool DENSE>
__global__ void __launch_bounds__(G5_THREADS, 1)
gemm_tc05_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw, G5Args a) {
  static_assert(2 * BN <= 256, "hi and lo planes form one MMA of N = 2 BN <= 256");
  using C = G5Cfg<BN>;
  constexpr int S = C::S;
  constexpr uint32_t IDESC = idesc_f16(G5_BM, 2 * BN);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* Ring = smem + S * C::STAGE;                                  // code rings, RC slots per warp
  uint64_t* full = reinterpret_cast<uint64_t*>(Ring + C::RING_BYTES);   // weight tile written (8 warps)
  uint64_t* tiles = full + S;                                           // the stage's TMA bytes landed
  uint64_t* empty = tiles + S;                                          // stage read by its MMAs
  uint64_t* accum = empty + S;                                          // every MMA done
  uint64_t* chunk = accum + 1;                                          // code chunk landed, RC per warp
  __shared__ uint32_t tmem_base;
  __shared__ int abort_s, last_s;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * G5_BM, m0 = blockIdx.y * BN;
  // this CTA's K steps: kb0 + p for p < KB
  const int z = blockIdx.z;
  const int kb0 = (int)((long long)a.P * z / a.ks), KB = (int)((long long)a.P * (z + 1) / a.ks) - kb0;

  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], G5_DEQ_WARPS);
      mbar_init(&tiles[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(accum, 1);
    for (int i = 0; i < G5_DEQ_WARPS * C::RC; ++i) mbar_init(&chunk[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    abort_s = 0;
  }
  if (warp == G5_MMA_WARP) {
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

  const int NS = (KB + G5_KS - 1) / G5_KS;  // stages (the last may hold one step)
  if (warp < G5_DEQ_WARPS) {
    // ---- dequantizing warps: weights never depend on the previous kernel,
    // so they stream from the first instruction
    if constexpr (!DENSE) {
      constexpr int RC = C::RC, CK = C::CK;
      uint8_t* ring = Ring + warp * RC * C::RING_SLOT;
      uint64_t* cbar = chunk + warp * RC;
      const int gt = (n0 >> 4) + warp;  // this warp's 16-row tile
      const bool have = gt < a.T16;     // tiles past the weight dequantize zeros
      const int NC = (KB + CK - 1) / CK;
      int issued = 0, landed = 0;  // chunks requested (lane 0) / seen complete
      if (have && lane == 0)
        for (; issued < RC && issued < NC; ++issued)
          g5_fetch<ST, CK>(a, gt, kb0, KB, issued, ring + issued * C::RING_SLOT, &cbar[issued]);
      for (int p = 0; p < KB; ++p) {
        const int q = p / G5_KS, sub = p % G5_KS, s = q % S, c = p / CK, i = p % CK;
        const uint8_t* slot = ring + (c % RC) * C::RING_SLOT;
        if (sub == 0 && q >= S) {
          // the stage's previous occupant (stage q - S) must have been read by its MMAs
          if (!mbar_wait_warp(&empty[s], (uint32_t)((q / S - 1) & 1), a.spin, lane)) {
            if (lane == 0) {
              atomicOr(a.fault, 8);
              *abort_v = 1;
            }
            break;
          }
          if (*abort_v) break;
        }
        G5Frag fr{make_uint4(0u, 0u, 0u, 0u), 0.f, 0.f};
        if (have) {
          if (i == 0) {
            if (!mbar_wait_warp(&cbar[c % RC], (uint32_t)((c / RC) & 1), a.spin, lane)) {
              if (lane == 0) {
                atomicOr(a.fault, 8);
                *abort_v = 1;
              }
              break;
            }
            landed = c + 1;
          }
          fr = g5_read<ST, CK>(a, slot, kb0, p, lane);
        }
        g5_dequant(fr, smem + s * C::STAGE + sub * G5_A_BYTES, tid);
        const bool stage_done = sub == G5_KS - 1 || p == KB - 1;
        const bool chunk_end = have && (i == CK - 1 || p == KB - 1);
        if (!stage_done && !chunk_end) continue;  // nothing to hand over after this step
        // the stage's weight tiles become visible to the tensor pipe
        if (stage_done) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        if (stage_done && warp == 0) {
          // the stage's activation tiles must have landed before `full`
          if (!mbar_wait_warp(&tiles[s], (uint32_t)((q / S) & 1), a.spin, lane)) {
            if (lane == 0) {
              atomicOr(a.fault, 8);
              *abort_v = 1;
            }
            break;
          }
        }
        __syncwarp();
        if (lane == 0) {
          if (stage_done) mbar_arrive(&full[s]);
          // the chunk's last step is read: its slot takes chunk c + RC
          if (chunk_end && issued < NC) {
            g5_fetch<ST, CK>(a, gt, kb0, KB, issued, ring + (issued % RC) * C::RING_SLOT, &cbar[issued % RC]);
            ++issued;
          }
        }
      }
      // a warp that stopped early lets its chunk copies in flight land first
      if (have && lane == 0)
        for (int c = landed; c < issued; ++c) mbar_wait_bounded(&cbar[c % RC], (uint32_t)((c / RC) & 1));
    }
  } else if (warp == G5_MMA_WARP) {
    // ---- MMA thread: one wait and one commit per stage of G5_KS steps
    if (lane == 0) {
      for (int q = 0; q < NS; ++q) {
        const int s = q % S;
        if (!mbar_wait_bounded(DENSE ? &tiles[s] : &full[s], (uint32_t)((q / S) & 1), a.spin) || *abort_v) {
          if (!*abort_v) atomicOr(a.fault, 8);
          *abort_v = 1;
          break;
        }
        tc05_fence_after();
        const uint32_t st = smem_u32(smem + s * C::STAGE);
        const int nsub = min(G5_KS, KB - q * G5_KS);
        for (int sub = 0; sub < nsub; ++sub) {
          const uint32_t sa = st + sub * G5_A_BYTES, sb = st + G5_KS * G5_A_BYTES + sub * C::B_BYTES;
#pragma unroll
          for (int kk = 0; kk < G5_BK / 16; ++kk)
            tc05_mma(tmem, smem_desc_sw128(sa + kk * 32), smem_desc_sw128(sb + kk * 32), IDESC,
                     (q | sub | kk) != 0);
        }
        tc05_commit(&empty[s]);
      }
      tc05_commit(accum);  // completes once every MMA issued above is done
    }
  } else if (lane == 0) {
    // ---- TMA thread: a stage is refilled once the MMAs of its previous
    // occupant are done; the bytes count on the stage's `tiles` barrier
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmx) : "memory");
    if (DENSE) asm volatile("prefetch.tensormap [%0];" ::"l"(&tmw) : "memory");
    pdl_wait();  // the activation rows come from the previous kernel
    int issued = 0;
    for (; issued < NS; ++issued) {
      const int s = issued % S;
      if (issued >= S && !mbar_wait_bounded(&empty[s], (uint32_t)((issued / S - 1) & 1), a.spin)) {
        atomicOr(a.fault, 8);
        *abort_v = 1;
        break;
      }
      if (*abort_v) break;
      uint8_t* st = smem + s * C::STAGE;
      const int k0 = kb0 + issued * G5_KS, nsub = min(G5_KS, KB - issued * G5_KS);
      mbar_expect_tx(&tiles[s], (uint32_t)nsub * (C::B_BYTES + (DENSE ? G5_A_BYTES : 0)));
      for (int sub = 0; sub < nsub; ++sub) {
        tma_load_3d(st + G5_KS * G5_A_BYTES + sub * C::B_BYTES, &tmx, (k0 + sub) * G5_BK, m0, &tiles[s]);
        if (DENSE) tma_load_2d(st + sub * G5_A_BYTES, &tmw, (k0 + sub) * G5_BK, n0, &tiles[s]);
      }
    }
    // an aborted CTA lets the loads in flight land before the stages go away
    // (`tiles` phases complete on the bytes alone; older phases completed
    // before their stage was refilled)
    if (*abort_v)
      for (int i = issued > S ? issued - S : 0; i < issued; ++i)
        mbar_wait_bounded(&tiles[i % S], (uint32_t)((i / S) & 1));
  }

  if (warp < G5_DEQ_WARPS) {
    // ---- epilogue (the 8 warps; named barrier 1 spans them only)
    const bool done = mbar_wait_warp(accum, 0u, MBAR_SPIN_LIMIT, lane);
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
  if (warp == G5_MMA_WARP) {
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
