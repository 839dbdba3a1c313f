// Attention of several query rows at once (prompt prefill, tree
// verification): chat.py:264-281 with sq > 1 -- scores q.K^T / sqrt(hd), key
// j visible to row r iff its position (j itself for a cached key, else the
// position of the input row it came from) is <= row r's position, plus
// min(0, bias[r, j]) when a bias is given (the tree ancestry mask of
// eagle.py:259-291), softmax over the keys, times V. A positive bias entry
// (which the reference never passes) admits the key whatever its position:
// several sequences sharing one cache, whose rows sit side by side.
//
// One CTA per (head, block of AR_BR = 64 query rows), four warps of 16 rows
// each (with 16 or 32 rows in all, the warps split each key tile instead:
// the key groups of attn_rows_kernel's G). The CTA streams the keys in tiles of AR_BC = 64 through shared
// memory (double-buffered; fp16 cache rows by cp.async, fp32 cache rows
// converted to fp16 on the way), so every K/V row is read once per 64 query
// rows. Each warp computes its 16 x 64 score tile with mma.sync m16n8k16
// (fp16 inputs, fp32 accumulation), masks it, keeps an online softmax per
// row in registers (fp32, the running maximum subtracted), and multiplies the
// probabilities with the V tile on the tensor pipe (the score accumulators
// become the A fragments directly). The fp32 operands q and p enter the
// tensor pipe as two fp16 parts, v = hi + lo with hi = fp16(v) and
// lo = fp16(v - hi), each multiplied with the same K or V fragment, so they
// keep about 22 bits; the fp16 cache is used as stored (an fp32 cache is
// rounded to fp16 in the tile). The output rows are divided by their
// softmax sums at the end.
//
// Few rows (tree verification: 31 rows, one row block per head) would leave
// most SMs idle, so the key tiles also split over gridDim.z CTAs: CTA z takes
// tiles [z nkt / ks, (z + 1) nkt / ks), writes its unnormalized output rows
// and per-row (max, sum) to a workspace, and the CTA that draws the last
// ticket of its (head, row block) merges the ks states in z order:
// M = max_z m_z, out = sum_z o_z e^(m_z - M) / sum_z l_z e^(m_z - M).
#include "model.cuh"

namespace lumina {

namespace {

constexpr int AR_BR = 64;   // query rows per CTA
constexpr int AR_BC = 64;   // keys per tile
constexpr int AR_THREADS = 128;
constexpr int AR_MIN_SPLIT_TILES = 4;  // key tiles per CTA when the keys are split
constexpr int AR_CTAS_PER_SM = 2;      // resident CTAs per SM (registers, shared memory)

template <int HD>
struct ArCfg {
  static constexpr int ROW = HD * 2 + 16;  // padded fp16 row (bytes): ldmatrix phases hit distinct banks
  static constexpr int Q_BYTES = AR_BR * ROW;  // q hi + lo staged in one K/V buffer (2 KV_BYTES)
  static constexpr int KV_BYTES = AR_BC * ROW;
  static constexpr int B_BYTES = AR_BR * AR_BC * 4;  // bias tile (fp32)
  // [2 x (K, V)][kpos 2 x AR_BC ints][bias 2 x tile]; two CTAs fit on an SM
  static constexpr int SMEM_NOBIAS = 4 * KV_BYTES + 2 * AR_BC * 4;
  static constexpr int SMEM_BIAS = SMEM_NOBIAS + 2 * B_BYTES;
};

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// 4-byte asynchronous copy global -> shared; src_bytes 0 writes a zero and
// reads nothing
__device__ __forceinline__ void cp_async4(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src), "r"(src_bytes)
               : "memory");
}
// (a, b) -> fp16 pair (hi) and the fp16 pair of the remainders (lo)
__device__ __forceinline__ uint32_t pack_hl(float a, float b, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(a, b);
  const __half2 l = __floats2half2_rn(a - __low2float(h), b - __high2float(h));
  lo = *reinterpret_cast<const uint32_t*>(&l);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// G key groups: with few rows (G = 4: up to 16 rows, G = 2: up to 32) warp
// w takes rows 16 (w % RW) .. + 15 of the block and keys (w / RW) KPW ..
// + KPW - 1 of every tile, RW = 4 / G, KPW = 64 / G, so every warp has
// work; the G per-warp softmax states of a row merge in shared memory in
// key-group order after the key loop. G = 1 is the one-group kernel.
template <int HD, typename KT, int G>
__global__ void __launch_bounds__(AR_THREADS, AR_CTAS_PER_SM)
attn_rows_kernel(const float* __restrict__ q, int nh, int nkv, const KT* __restrict__ kcache,
                 const KT* __restrict__ vcache, const int* __restrict__ block_table, int bs,
                 const int* __restrict__ row_pos, const float* __restrict__ bias, const DevParams* __restrict__ P,
                 float* __restrict__ out, float sdiv, float* __restrict__ ws, int* __restrict__ cnt) {
  using C = ArCfg<HD>;
  constexpr int NKK = HD / 16;  // k-steps of q.K^T
  constexpr int NDT = HD / 8;   // n-tiles of P.V
  constexpr int RW = 4 / G;     // row warps
  constexpr int KPW = AR_BC / G, NTW = KPW / 8, NPW = KPW / 16;  // a warp's keys, n-tiles, 16-key steps
  const int h = blockIdx.x, r0 = blockIdx.y * AR_BR;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rw = warp % RW, kg = warp / RW;  // row warp, key group
  const int g = lane >> 2, t = lane & 3;
  pdl_launch_dependents();
  pdl_wait();
  const int n = P->n, T = P->t_tot, t_prev = P->t_prev, bias_ld = P->bias_ld;
  if (r0 >= n) return;
  const int kvh = h / (nh / nkv);
  const size_t bstride = (size_t)nkv * bs * HD;

  extern __shared__ __align__(16) uint8_t sm[];
  uint8_t* KVs = sm;  // [buf][K | V]
  int* kpos_s = reinterpret_cast<int*>(sm + 4 * C::KV_BYTES);  // [buf][AR_BC]
  float* bias_s = reinterpret_cast<float*>(kpos_s + 2 * AR_BC);             // [buf][AR_BR][AR_BC]

  // tile kt of K, V (and positions, bias) into buffer kt & 1; this CTA's
  // tiles are [kt0, kt1)
  const int nkt = (T + AR_BC - 1) / AR_BC;
  const int ks = gridDim.z, z = blockIdx.z;
  const int kt0 = (int)((long long)nkt * z / ks), kt1 = (int)((long long)nkt * (z + 1) / ks);
  auto load_tile = [&](int kt) {
    const int b = kt & 1;
    uint8_t* ks = KVs + (size_t)b * 2 * C::KV_BYTES;
    uint8_t* vs = ks + C::KV_BYTES;
    const int j0 = kt * AR_BC;
    if constexpr (sizeof(KT) == 2) {
      // thread tid copies 16-byte chunk tid % CH of keys tid / CH + it * KSTEP;
      // the page numbers of those keys are read first, all at once (each
      // cp.async below is a memory-clobbering asm that would otherwise make
      // every page-table read wait for the previous copy's issue)
      constexpr int CH = HD * 2 / 16, IT = AR_BC * CH / AR_THREADS, KSTEP = AR_THREADS / CH;
      static_assert(AR_BC * CH % AR_THREADS == 0 && AR_THREADS % CH == 0, "whole chunks per thread");
      const int ch = tid % CH, jt = tid / CH;
      int page[IT];
#pragma unroll
      for (int it = 0; it < IT; ++it) {
        const int key = j0 + jt + it * KSTEP;
        page[it] = key < T ? block_table[key / bs] : 0;
      }
#pragma unroll
      for (int it = 0; it < IT; ++it) {
        const int j = jt + it * KSTEP, key = j0 + j;
        uint8_t* kd = ks + j * C::ROW + ch * 16;
        uint8_t* vd = vs + j * C::ROW + ch * 16;
        if (key < T) {
          const size_t base = (size_t)page[it] * bstride + ((size_t)kvh * bs + key % bs) * HD;
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(kd)),
                       "l"(reinterpret_cast<const uint8_t*>(kcache + base) + ch * 16) : "memory");
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(vd)),
                       "l"(reinterpret_cast<const uint8_t*>(vcache + base) + ch * 16) : "memory");
        } else {
          *reinterpret_cast<uint4*>(kd) = make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(vd) = make_uint4(0u, 0u, 0u, 0u);
        }
      }
    } else {
      // fp32 cache rows: 4 values per load, rounded to fp16 into the tile
      constexpr int CH = HD / 4;
      for (int i = tid; i < AR_BC * CH; i += AR_THREADS) {
        const int j = i / CH, ch = i - j * CH, key = j0 + j;
        uint2 kh = make_uint2(0u, 0u), vh = make_uint2(0u, 0u);
        if (key < T) {
          const size_t base = (size_t)block_table[key / bs] * bstride + ((size_t)kvh * bs + key % bs) * HD;
          const float4 kf = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(kcache) + base + ch * 4);
          const float4 vf = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(vcache) + base + ch * 4);
          kh = make_uint2(pack_h2(kf.x, kf.y), pack_h2(kf.z, kf.w));
          vh = make_uint2(pack_h2(vf.x, vf.y), pack_h2(vf.z, vf.w));
        }
        *reinterpret_cast<uint2*>(ks + j * C::ROW + ch * 8) = kh;
        *reinterpret_cast<uint2*>(vs + j * C::ROW + ch * 8) = vh;
      }
    }
    // key positions and the bias tile also arrive by cp.async (4-byte copies:
    // bias rows of bias_ld floats need not be 16-byte aligned), so no thread
    // waits on a load here; out-of-range bias entries are zero-filled
    for (int j = tid; j < AR_BC; j += AR_THREADS) {
      const int key = j0 + j;
      int* dst = &kpos_s[b * AR_BC + j];
      if (key >= T || key < t_prev)
        *dst = key >= T ? 0x7fffffff : key;
      else
        cp_async4(dst, row_pos + (key - t_prev), 4);
    }
    if (bias) {
      float* bt = bias_s + (size_t)b * AR_BR * AR_BC;
      for (int i = tid; i < AR_BR * AR_BC; i += AR_THREADS) {
        const int rr = i / AR_BC, j = i - rr * AR_BC, row = r0 + rr, key = j0 + j;
        const bool in = row < n && key < T;
        cp_async4(bt + i, in ? bias + (size_t)row * bias_ld + key : bias, in ? 4 : 0);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  if (kt0 < kt1) load_tile(kt0);
  // q rows of the block -> fp16 hi and lo parts (rows past n are zero),
  // staged in the K/V buffer that tile kt0 does not use, then held in
  // registers for the whole key loop
  static_assert(2 * C::Q_BYTES <= 2 * C::KV_BYTES, "q hi and lo fit in one K/V buffer");
  uint8_t* Qs = KVs + (size_t)((kt0 + 1) & 1) * 2 * C::KV_BYTES;  // fp16(q)
  uint8_t* Ql = Qs + C::Q_BYTES;                                    // fp16(q - fp16(q))
  for (int i = tid; i < AR_BR * (HD / 4); i += AR_THREADS) {
    const int rr = i / (HD / 4), c4 = i - rr * (HD / 4), row = r0 + rr;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (row < n) v = *reinterpret_cast<const float4*>(q + ((size_t)row * nh + h) * HD + c4 * 4);
    uint32_t l0, l1;
    const uint32_t h0 = pack_hl(v.x, v.y, l0), h1 = pack_hl(v.z, v.w, l1);
    *reinterpret_cast<uint2*>(Qs + rr * C::ROW + c4 * 8) = make_uint2(h0, h1);
    *reinterpret_cast<uint2*>(Ql + rr * C::ROW + c4 * 8) = make_uint2(l0, l1);
  }
  const int ra = r0 + 16 * rw + g, rb = ra + 8;  // this lane's two rows
  const int pa = ra < n ? row_pos[ra] : -1, pb = rb < n ? row_pos[rb] : -1;
  __syncthreads();
  uint32_t qa[NKK][4], ql[NKK][4];
#pragma unroll
  for (int kk = 0; kk < NKK; ++kk) {
    const int off = (16 * rw + (lane & 15)) * C::ROW + (16 * kk + 8 * (lane >> 4)) * 2;
    ldsm_x4(qa[kk], Qs + off);
    ldsm_x4(ql[kk], Ql + off);
  }
  __syncthreads();  // the staging buffer is free for tile kt0 + 1

  float o[NDT][4];
#pragma unroll
  for (int i = 0; i < NDT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float ma = -INFINITY, mb = -INFINITY, la = 0.f, lb = 0.f;

  for (int kt = kt0; kt < kt1; ++kt) {
    if (kt + 1 < kt1) {
      load_tile(kt + 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    // a warp whose 16 rows are all past n (tree verification: 31 rows in a
    // 64-row block) only helps load the tiles
    if (r0 + 16 * rw < n) {
      const int b = kt & 1;
      const uint8_t* ks = KVs + (size_t)b * 2 * C::KV_BYTES;
      const uint8_t* vs = ks + C::KV_BYTES;
      const int* kp = kpos_s + b * AR_BC;
      const float* bt = bias_s + (size_t)b * AR_BR * AR_BC;
      // scores: 16 rows x this warp's KPW keys, n-tile nt = keys kg KPW +
      // 8nt .. + 7; the k-step loop is outside so that consecutive MMAs feed
      // different accumulators (a chain of dependent mma.sync would stall
      // on each)
      float s[NTW][4];
#pragma unroll
      for (int nt = 0; nt < NTW; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < NKK; ++kk) {
        // matrices of pair np: keys 16np.. x dims lo / hi, keys 16np+8.. x dims lo / hi
        uint32_t kb[NPW][4];
#pragma unroll
        for (int np = 0; np < NPW; ++np) {
          const int key = kg * KPW + 16 * np + (lane & 7) + 8 * (lane >> 4);
          ldsm_x4(kb[np], ks + key * C::ROW + (16 * kk + 8 * ((lane >> 3) & 1)) * 2);
        }
#pragma unroll
        for (int np = 0; np < NPW; ++np) {
          mma_f16(s[2 * np], qa[kk], kb[np][0], kb[np][1]);
          mma_f16(s[2 * np + 1], qa[kk], kb[np][2], kb[np][3]);
        }
#pragma unroll
        for (int np = 0; np < NPW; ++np) {
          mma_f16(s[2 * np], ql[kk], kb[np][0], kb[np][1]);
          mma_f16(s[2 * np + 1], ql[kk], kb[np][2], kb[np][3]);
        }
      }
      // mask, scale, online softmax (rows a = g, b = g + 8 of this warp)
      float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < NTW; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = kg * KPW + 8 * nt + 2 * t + (e & 1);
          const bool rowb = e >= 2;
          const int rp = rowb ? pb : pa;
          // a positive bias admits the key whatever its position (rows of
          // one sequence among several sharing the cache); otherwise the
          // position rule and min(0, bias) as the reference applies them
          const float bv = bias ? bt[(16 * rw + g + (rowb ? 8 : 0)) * AR_BC + j] : 0.f;
          float v = -INFINITY;
          if (rp >= 0 && (kp[j] <= rp || bv > 0.f)) {
            v = __fdiv_rn(s[nt][e], sdiv);
            v += fminf(0.f, bv);
          }
          s[nt][e] = v;
          if (rowb) mxb = fmaxf(mxb, v); else mxa = fmaxf(mxa, v);
        }
      }
      mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 1));
      mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 2));
      mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 1));
      mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 2));
      const float na = fmaxf(ma, mxa), nb = fmaxf(mb, mxb);
      const float aa = na == -INFINITY ? 1.f : expf(ma - na), ab = nb == -INFINITY ? 1.f : expf(mb - nb);
      float sa = 0.f, sb = 0.f;
#pragma unroll
      for (int nt = 0; nt < NTW; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const bool rowb = e >= 2;
          const float m = rowb ? nb : na;
          const float p = s[nt][e] == -INFINITY ? 0.f : expf(s[nt][e] - m);
          s[nt][e] = p;
          if (rowb) sb += p; else sa += p;
        }
      }
      sa += __shfl_xor_sync(0xffffffffu, sa, 1);
      sa += __shfl_xor_sync(0xffffffffu, sa, 2);
      sb += __shfl_xor_sync(0xffffffffu, sb, 1);
      sb += __shfl_xor_sync(0xffffffffu, sb, 2);
      la = la * aa + sa;
      lb = lb * ab + sb;
      ma = na;
      mb = nb;
#pragma unroll
      for (int i = 0; i < NDT; ++i) {
        o[i][0] *= aa;
        o[i][1] *= aa;
        o[i][2] *= ab;
        o[i][3] *= ab;
      }
      // P.V: k-step kk = this warp's keys 16kk .. 16kk + 15 (score n-tiles
      // 2kk, 2kk + 1), tile keys kg KPW + 16kk ..
#pragma unroll
      for (int kk = 0; kk < NPW; ++kk) {
        uint32_t pa4[4], pl4[4];
        pa4[0] = pack_hl(s[2 * kk][0], s[2 * kk][1], pl4[0]);
        pa4[1] = pack_hl(s[2 * kk][2], s[2 * kk][3], pl4[1]);
        pa4[2] = pack_hl(s[2 * kk + 1][0], s[2 * kk + 1][1], pl4[2]);
        pa4[3] = pack_hl(s[2 * kk + 1][2], s[2 * kk + 1][3], pl4[3]);
#pragma unroll
        for (int nd = 0; nd < NDT; nd += 4) {
          // matrices (transposed): keys 16kk.. / 16kk+8.. x dims 8nd.., then
          // dims 8(nd+1)..; two such pairs, so that an accumulator's hi and lo
          // products are four MMAs apart
          uint32_t vb[2][4];
#pragma unroll
          for (int u = 0; u < 2; ++u)
            ldsm_x4_t(vb[u], vs + (kg * KPW + 16 * kk + (lane & 15)) * C::ROW +
                                 (8 * (nd + 2 * u) + 8 * (lane >> 4)) * 2);
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            mma_f16(o[nd + 2 * u], pa4, vb[u][0], vb[u][1]);
            mma_f16(o[nd + 2 * u + 1], pa4, vb[u][2], vb[u][3]);
          }
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            mma_f16(o[nd + 2 * u], pl4, vb[u][0], vb[u][1]);
            mma_f16(o[nd + 2 * u + 1], pl4, vb[u][2], vb[u][3]);
          }
        }
      }
    }
    __syncthreads();  // buffer b is free for tile kt + 2
  }
  if constexpr (G > 1) {
    // key groups 1 .. G-1 leave their states in the free K/V buffers; the
    // group-0 warp of each row warp adds them in group order
    constexpr int SLOT = (4 * NDT + 4) * 32;  // floats: o, then (ma, la, mb, lb), lane-minor
    float* st = reinterpret_cast<float*>(KVs);
    if (kg > 0) {
      float* my = st + (size_t)((kg - 1) * RW + rw) * SLOT;
#pragma unroll
      for (int nd = 0; nd < NDT; ++nd)
#pragma unroll
        for (int e = 0; e < 4; ++e) my[(4 * nd + e) * 32 + lane] = o[nd][e];
      my[(4 * NDT + 0) * 32 + lane] = ma;
      my[(4 * NDT + 1) * 32 + lane] = la;
      my[(4 * NDT + 2) * 32 + lane] = mb;
      my[(4 * NDT + 3) * 32 + lane] = lb;
    }
    __syncthreads();
    if (kg == 0) {
#pragma unroll 1
      for (int q = 1; q < G; ++q) {
        const float* ot = st + (size_t)((q - 1) * RW + rw) * SLOT;
        const float qma = ot[(4 * NDT + 0) * 32 + lane], qla = ot[(4 * NDT + 1) * 32 + lane];
        const float qmb = ot[(4 * NDT + 2) * 32 + lane], qlb = ot[(4 * NDT + 3) * 32 + lane];
        const float na = fmaxf(ma, qma), nb = fmaxf(mb, qmb);
        const float fa0 = na == -INFINITY ? 0.f : expf(ma - na), fa1 = na == -INFINITY ? 0.f : expf(qma - na);
        const float fb0 = nb == -INFINITY ? 0.f : expf(mb - nb), fb1 = nb == -INFINITY ? 0.f : expf(qmb - nb);
        la = la * fa0 + qla * fa1;
        lb = lb * fb0 + qlb * fb1;
#pragma unroll
        for (int nd = 0; nd < NDT; ++nd) {
          o[nd][0] = o[nd][0] * fa0 + ot[(4 * nd + 0) * 32 + lane] * fa1;
          o[nd][1] = o[nd][1] * fa0 + ot[(4 * nd + 1) * 32 + lane] * fa1;
          o[nd][2] = o[nd][2] * fb0 + ot[(4 * nd + 2) * 32 + lane] * fb1;
          o[nd][3] = o[nd][3] * fb0 + ot[(4 * nd + 3) * 32 + lane] * fb1;
        }
        ma = na;
        mb = nb;
      }
    }
  }
  // only the group-0 warps hold final states from here on
  const bool writer = kg == 0;
  const bool va = writer && ra < n, vb = writer && rb < n;  // rows this lane writes
  // out[row][h][d] = o / l: lane holds rows a (o[.][0..1]) and b (o[.][2..3]), dims 8nd + 2t, +1
  if (ks == 1) {
    const float ia = la > 0.f ? 1.f / la : 0.f, ib = lb > 0.f ? 1.f / lb : 0.f;
#pragma unroll
    for (int nd = 0; nd < NDT; ++nd) {
      const int d = 8 * nd + 2 * t;
      if (va)
        *reinterpret_cast<float2*>(out + ((size_t)ra * nh + h) * HD + d) = make_float2(o[nd][0] * ia, o[nd][1] * ia);
      if (vb)
        *reinterpret_cast<float2*>(out + ((size_t)rb * nh + h) * HD + d) = make_float2(o[nd][2] * ib, o[nd][3] * ib);
    }
    return;
  }
  // split keys: state z of (row, head) at part_o[(z n + row) nh + h][HD] and
  // part_ml[(z n + row) nh + h] = (m, l)
  float* part_o = ws;
  float2* part_ml = reinterpret_cast<float2*>(ws + (size_t)ks * n * nh * HD);
  const size_t ia_idx = ((size_t)z * n + ra) * nh + h, ib_idx = ((size_t)z * n + rb) * nh + h;
#pragma unroll
  for (int nd = 0; nd < NDT; ++nd) {
    const int d = 8 * nd + 2 * t;
    if (va) *reinterpret_cast<float2*>(part_o + ia_idx * HD + d) = make_float2(o[nd][0], o[nd][1]);
    if (vb) *reinterpret_cast<float2*>(part_o + ib_idx * HD + d) = make_float2(o[nd][2], o[nd][3]);
  }
  if (t == 0) {
    if (va) part_ml[ia_idx] = make_float2(ma, la);
    if (vb) part_ml[ib_idx] = make_float2(mb, lb);
  }
  __threadfence();
  __syncthreads();
  __shared__ int last_s;
  const int tile = blockIdx.y * nh + h;
  if (tid == 0) last_s = atomicAdd(&cnt[tile], 1) == ks - 1;
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  // merge in z order
  float Ma = -INFINITY, Mb = -INFINITY;
  for (int zz = 0; zz < ks; ++zz) {
    if (va) Ma = fmaxf(Ma, __ldcg(&part_ml[((size_t)zz * n + ra) * nh + h].x));
    if (vb) Mb = fmaxf(Mb, __ldcg(&part_ml[((size_t)zz * n + rb) * nh + h].x));
  }
  float accA[NDT][2], accB[NDT][2], La = 0.f, Lb = 0.f;
#pragma unroll
  for (int nd = 0; nd < NDT; ++nd) accA[nd][0] = accA[nd][1] = accB[nd][0] = accB[nd][1] = 0.f;
  for (int zz = 0; zz < ks; ++zz) {
    const size_t ja = ((size_t)zz * n + ra) * nh + h, jb = ((size_t)zz * n + rb) * nh + h;
    if (va && Ma != -INFINITY) {
      const float2 ml = __ldcg(&part_ml[ja]);
      const float f = ml.x == -INFINITY ? 0.f : expf(ml.x - Ma);
      La += ml.y * f;
#pragma unroll
      for (int nd = 0; nd < NDT; ++nd) {
        const float2 v = __ldcg(reinterpret_cast<const float2*>(part_o + ja * HD + 8 * nd + 2 * t));
        accA[nd][0] += v.x * f;
        accA[nd][1] += v.y * f;
      }
    }
    if (vb && Mb != -INFINITY) {
      const float2 ml = __ldcg(&part_ml[jb]);
      const float f = ml.x == -INFINITY ? 0.f : expf(ml.x - Mb);
      Lb += ml.y * f;
#pragma unroll
      for (int nd = 0; nd < NDT; ++nd) {
        const float2 v = __ldcg(reinterpret_cast<const float2*>(part_o + jb * HD + 8 * nd + 2 * t));
        accB[nd][0] += v.x * f;
        accB[nd][1] += v.y * f;
      }
    }
  }
  const float ia = La > 0.f ? 1.f / La : 0.f, ib = Lb > 0.f ? 1.f / Lb : 0.f;
#pragma unroll
  for (int nd = 0; nd < NDT; ++nd) {
    const int d = 8 * nd + 2 * t;
    if (va)
      *reinterpret_cast<float2*>(out + ((size_t)ra * nh + h) * HD + d) = make_float2(accA[nd][0] * ia, accA[nd][1] * ia);
    if (vb)
      *reinterpret_cast<float2*>(out + ((size_t)rb * nh + h) * HD + d) = make_float2(accB[nd][0] * ib, accB[nd][1] * ib);
  }
  if (tid == 0) cnt[tile] = 0;
}

template <int HD, typename KT, int G>
int launch_rows(const float* q, int nh, int nkv, const void* kc, const void* vc, const int* bt, int bs,
                const int* row_pos, const float* bias, const DevParams* P, float* out, int max_n, float sdiv,
                int t_tot, const SplitWork* sw, cudaStream_t s) {
  auto kern = attn_rows_kernel<HD, KT, G>;
  const size_t smem = bias ? ArCfg<HD>::SMEM_BIAS : ArCfg<HD>::SMEM_NOBIAS;
  const int rc = set_smem_limit((const void*)kern, smem, "attention (rows)");
  if (rc) return rc;
  // key splits while heads x row blocks leave SMs idle: as many as one wave
  // of CTAs holds (AR_CTAS_PER_SM per SM), at least AR_MIN_SPLIT_TILES key
  // tiles per CTA, the states within the workspace
  const int rb = (max_n + AR_BR - 1) / AR_BR, tiles = nh * rb;
  const int nkt = (t_tot + AR_BC - 1) / AR_BC;
  int ks = 1;
  if (sw && sw->ws && sw->cnt && tiles < sm_count() && tiles <= sw->cnt_n) {
    ks = std::min(AR_CTAS_PER_SM * sm_count() / tiles, nkt / AR_MIN_SPLIT_TILES);
    while (ks > 1 && (size_t)ks * max_n * nh * (HD + 2) > sw->ws_elems) --ks;
    ks = std::max(ks, 1);
  }
  const dim3 grid(nh, rb, ks);
  const cudaError_t e = launch_pdl(kern, grid, dim3(AR_THREADS), smem, s, q, nh, nkv, (const KT*)kc, (const KT*)vc,
                                   bt, bs, row_pos, bias, P, out, sdiv, ks > 1 ? sw->ws : nullptr,
                                   ks > 1 ? sw->cnt : nullptr);
  if (e != cudaSuccess) {
    set_error("attention (rows) launch: %s", cudaGetErrorString(e));
    return LUMINA_E_CUDA;
  }
  return LUMINA_OK;
}

// few rows leave warps of the 64-row block idle: split each tile's keys
// over them instead (4 key groups up to 16 rows, 2 up to 32)
template <int HD, typename KT>
int launch_rows_g(const float* q, int nh, int nkv, const void* kc, const void* vc, const int* bt, int bs,
                  const int* row_pos, const float* bias, const DevParams* P, float* out, int max_n, float sdiv,
                  int t_tot, const SplitWork* sw, cudaStream_t s) {
  if (max_n <= 16)
    return launch_rows<HD, KT, 4>(q, nh, nkv, kc, vc, bt, bs, row_pos, bias, P, out, max_n, sdiv, t_tot, sw, s);
  if (max_n <= 32)
    return launch_rows<HD, KT, 2>(q, nh, nkv, kc, vc, bt, bs, row_pos, bias, P, out, max_n, sdiv, t_tot, sw, s);
  return launch_rows<HD, KT, 1>(q, nh, nkv, kc, vc, bt, bs, row_pos, bias, P, out, max_n, sdiv, t_tot, sw, s);
}

}  // namespace

int launch_attention_rows(bool fp16, int hd, const float* q, int nh, int nkv, const void* kc, const void* vc,
                          const int* bt, int bs, const int* row_pos, const float* bias, const DevParams* P, float* out,
                          int max_n, int t_tot, const SplitWork* sw, cudaStream_t s) {
  const float sdiv = std::max(sqrtf((float)hd), 1e-6f);  // max(hd ** 0.5, 1e-6), chat.py:278
  if (hd == 128)
    return fp16 ? launch_rows_g<128, __half>(q, nh, nkv, kc, vc, bt, bs, row_pos, bias, P, out, max_n, sdiv, t_tot,
                                             sw, s)
                : launch_rows_g<128, float>(q, nh, nkv, kc, vc, bt, bs, row_pos, bias, P, out, max_n, sdiv, t_tot,
                                            sw, s);
  if (hd == 64)
    return fp16 ? launch_rows_g<64, __half>(q, nh, nkv, kc, vc, bt, bs, row_pos, bias, P, out, max_n, sdiv, t_tot,
                                            sw, s)
                : launch_rows_g<64, float>(q, nh, nkv, kc, vc, bt, bs, row_pos, bias, P, out, max_n, sdiv, t_tot,
                                           sw, s);
  set_error("attention: head_dim %d not built (64, 128)", hd);
  return LUMINA_E_UNSUPPORTED;
}

}  // namespace lumina
