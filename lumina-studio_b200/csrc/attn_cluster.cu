// Single-query decode attention over the paged KV cache (chat.py:264-281
// with one new row: every key up to the row is visible, no bias).
//
// One thread-block cluster of ATTNC_CLUSTER CTAs per head. CTA r of the
// cluster takes keys [r*T/CS, (r+1)*T/CS) and streams them through a
// double-buffered shared-memory ring of ATTNC_CHUNK keys (cp.async, 16
// bytes per copy; K rows padded by 16 bytes so that lanes reading
// consecutive keys hit distinct banks). Only the new row (and q) come from
// the preceding q/k/v kernel; the key count and block table are fixed for
// the whole step, so both ring chunks are requested before the dependency
// wait without the new row, which is read after it. The CTA keeps an online
// softmax: scores
// with lanes along keys and two warps per half of the head dimension, the
// chunk's max / exponentials in one warp, P.V with threads along dimension
// pairs. The CTAs' (max, sum, unnormalized output) meet in distributed
// shared memory: rank 0 merges them in rank order (deterministic) after a
// cluster barrier and writes the head's output; a second barrier keeps every
// CTA's shared memory alive until rank 0 has read it. No global workspace,
// counters or atomics.
#include <cooperative_groups.h>

#include "model.cuh"

namespace lumina {

namespace {

namespace cg = cooperative_groups;

template <int HD, typename KT>
struct AttnCfg {
  static constexpr int ES = sizeof(KT);
  static constexpr int KROW = HD * ES + 16;  // padded K row (bytes)
  static constexpr int VROW = HD * ES;
  static constexpr int CH = HD * ES / 16;    // 16-byte chunks per row
  static constexpr int BUF = ATTNC_CHUNK * (KROW + VROW);
  static constexpr int DP = HD / 2, NPH = 128 / DP;  // P.V: dim pairs x key phases
  static constexpr int SMEM = 2 * BUF + HD * 4 + 2 * ATTNC_CHUNK * 4 + NPH * HD * 4 + HD * 4 + 16;
};

template <int HD, typename KT>
__global__ void __launch_bounds__(128)
attnc_kernel(const float* __restrict__ q, int nh, int nkv, const KT* __restrict__ kcache,
             const KT* __restrict__ vcache, const int* __restrict__ block_table, int bs,
             const DevParams* __restrict__ P, float* __restrict__ out, float sdiv, L2Prefetch pf) {
  using C = AttnCfg<HD, KT>;
  constexpr int CK = ATTNC_CHUNK, CS = ATTNC_CLUSTER;
  cg::cluster_group cluster = cg::this_cluster();
  const int r = (int)cluster.block_rank();
  const int h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_launch_dependents();
  // set before the step (host copy or the previous step's commit kernel)
  const int T = P->t_tot, knew = P->t_prev;
  const int k0 = (r * T) / CS, k1 = ((r + 1) * T) / CS, nk = k1 - k0;
  const int kvh = h / (nh / nkv);
  const size_t bstride = (size_t)nkv * bs * HD;

  extern __shared__ __align__(16) uint8_t sm[];
  uint8_t* buf = sm;                                                   // [2][CK][KROW + VROW]
  float* qs = reinterpret_cast<float*>(sm + 2 * C::BUF);               // [HD]
  float* sc = qs + HD;                                                 // [2][CK]
  float* po = sc + 2 * CK;                                             // [NPH][HD]
  float* oc = po + C::NPH * HD;                                        // [HD] this CTA's output
  float* ml = oc + HD;                                                 // m, l, alpha
  // chunk c's K rows at buf + (c & 1) * BUF, V rows after the K rows
  // one commit group per call (possibly empty); before the dependency wait
  // (pre) the new row is left out
  auto issue = [&](int c, bool pre) {
    uint8_t* ks = buf + (size_t)(c & 1) * C::BUF;
    uint8_t* vs = ks + (size_t)CK * C::KROW;
    const int j0 = k0 + c * CK, n = min(CK, k1 - j0);
    for (int i = tid; i < n * C::CH; i += 128) {
      const int j = i / C::CH, ch = i - j * C::CH;
      const int key = j0 + j;
      if (pre && key == knew) continue;
      const int blk = block_table[key / bs], off = key % bs;
      const size_t base = (size_t)blk * bstride + ((size_t)kvh * bs + off) * HD;
      const uint8_t* kp = reinterpret_cast<const uint8_t*>(kcache + base) + ch * 16;
      const uint8_t* vp = reinterpret_cast<const uint8_t*>(vcache + base) + ch * 16;
      const uint32_t kd = (uint32_t)__cvta_generic_to_shared(ks + (size_t)j * C::KROW + ch * 16);
      const uint32_t vd = (uint32_t)__cvta_generic_to_shared(vs + (size_t)j * C::VROW + ch * 16);
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(kd), "l"(kp) : "memory");
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(vd), "l"(vp) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  const int nchunks = (nk + CK - 1) / CK;
  issue(0, true);
  issue(1, true);
  if (tid == 0) l2_prefetch_share(pf, h * CS + r, gridDim.y * CS);
  pdl_wait();
  // the new row, when it sits in a chunk requested before the wait
  if (knew >= k0 && knew < k1 && (knew - k0) / CK < 2) {
    const int j = knew - k0, c = j / CK, jj = j - c * CK;
    uint8_t* ks = buf + (size_t)(c & 1) * C::BUF;
    uint8_t* vs = ks + (size_t)CK * C::KROW;
    const int blk = block_table[knew / bs], off = knew % bs;
    const size_t base = (size_t)blk * bstride + ((size_t)kvh * bs + off) * HD;
    for (int ch = tid; ch < C::CH; ch += 128) {
      *reinterpret_cast<uint4*>(ks + (size_t)jj * C::KROW + ch * 16) =
          __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(kcache + base) + ch * 16));
      *reinterpret_cast<uint4*>(vs + (size_t)jj * C::VROW + ch * 16) =
          __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(vcache + base) + ch * 16));
    }
  }
  for (int d = tid; d < HD; d += 128) qs[d] = q[(size_t)h * HD + d];
  if (tid == 0) {
    ml[0] = -INFINITY;
    ml[1] = 0.f;
  }
  const int dp = tid % C::DP, kp = tid / C::DP;
  float o0 = 0.f, o1 = 0.f;  // dims 2dp, 2dp+1 over keys of phase kp
  for (int c = 0; c < nchunks; ++c) {
    asm volatile("cp.async.wait_group 1;" ::: "memory");  // chunk c landed (c + 1 may be in flight)
    __syncthreads();
    const uint8_t* ks = buf + (size_t)(c & 1) * C::BUF;
    const uint8_t* vs = ks + (size_t)CK * C::KROW;
    const int n = min(CK, nk - c * CK);
    // half-dots: warp w takes dims (w & 1) * HD/2 .. and keys (w >> 1) * 32 + lane
    {
      const int hf = warp & 1;
      for (int j = (warp >> 1) * 32 + lane; j < n; j += 64) {
        const uint4* kr = reinterpret_cast<const uint4*>(ks + (size_t)j * C::KROW + hf * (HD / 2) * C::ES);
        const float* qh = qs + hf * (HD / 2);
        float d = 0.f;
#pragma unroll
        for (int cc = 0; cc < (HD / 2) * C::ES / 16; ++cc) {
          const uint4 w = kr[cc];
          if constexpr (C::ES == 2) {
            const __half2* hh = reinterpret_cast<const __half2*>(&w);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __half22float2(hh[e]);
              d = fmaf(qh[cc * 8 + 2 * e], f.x, d);
              d = fmaf(qh[cc * 8 + 2 * e + 1], f.y, d);
            }
          } else {
            d = fmaf(qh[cc * 4], __uint_as_float(w.x), d);
            d = fmaf(qh[cc * 4 + 1], __uint_as_float(w.y), d);
            d = fmaf(qh[cc * 4 + 2], __uint_as_float(w.z), d);
            d = fmaf(qh[cc * 4 + 3], __uint_as_float(w.w), d);
          }
        }
        sc[hf * CK + j] = d;
      }
    }
    __syncthreads();
    // online softmax over the chunk (warp 0): scores -> p, running max / sum
    if (warp == 0) {
      float m = -INFINITY;
      for (int j = lane; j < n; j += 32) {
        const float s = __fdiv_rn(sc[j] + sc[CK + j], sdiv);
        sc[j] = s;
        m = fmaxf(m, s);
      }
      m = warp_max(m);
      const float m_old = ml[0], m_new = fmaxf(m_old, m);
      float l = 0.f;
      for (int j = lane; j < n; j += 32) {
        const float p = expf(sc[j] - m_new);
        sc[j] = p;
        l += p;
      }
      l = warp_sum(l);
      __syncwarp();
      if (lane == 0) {
        const float alpha = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
        ml[0] = m_new;
        ml[1] = ml[1] * alpha + l;
        ml[2] = alpha;
      }
    }
    __syncthreads();
    // P.V, the running output rescaled by alpha
    {
      const float alpha = ml[2];
      o0 *= alpha;
      o1 *= alpha;
      for (int j = kp; j < n; j += C::NPH) {
        const float p = sc[j];
        float2 v;
        if constexpr (C::ES == 2) {
          v = __half22float2(*reinterpret_cast<const __half2*>(vs + (size_t)j * C::VROW + dp * 4));
        } else {
          v = *reinterpret_cast<const float2*>(vs + (size_t)j * C::VROW + dp * 8);
        }
        o0 = fmaf(p, v.x, o0);
        o1 = fmaf(p, v.y, o1);
      }
    }
    __syncthreads();  // the buffer of chunk c is free for chunk c + 2
    if (c + 2 < nchunks) issue(c + 2, false);
    else asm volatile("cp.async.commit_group;" ::: "memory");
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  po[kp * HD + 2 * dp] = o0;
  po[kp * HD + 2 * dp + 1] = o1;
  __syncthreads();
  for (int d = tid; d < HD; d += 128) {
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < C::NPH; ++i) acc += po[i * HD + d];
    oc[d] = acc;
  }
  // every CTA's (m, l, o) -> rank 0 over distributed shared memory
  cluster.sync();
  if (r == 0) {
    float M = -INFINITY;
#pragma unroll
    for (int rr = 0; rr < CS; ++rr) M = fmaxf(M, cluster.map_shared_rank(ml, rr)[0]);
    float L = 0.f, wgt[CS];
#pragma unroll
    for (int rr = 0; rr < CS; ++rr) {
      const float* mr = cluster.map_shared_rank(ml, rr);
      wgt[rr] = mr[0] == -INFINITY ? 0.f : expf(mr[0] - M);
      L += wgt[rr] * mr[1];
    }
    for (int d = tid; d < HD; d += 128) {
      float acc = 0.f;
#pragma unroll
      for (int rr = 0; rr < CS; ++rr)
        if (wgt[rr] != 0.f) acc = fmaf(wgt[rr], cluster.map_shared_rank(oc, rr)[d], acc);
      out[(size_t)h * HD + d] = acc / L;
    }
  }
  cluster.sync();  // rank 0 is done reading the other CTAs' shared memory
}

template <int HD, typename KT>
int launch_one(const float* q, int nh, int nkv, const void* kc, const void* vc, const int* bt, int bs,
               const DevParams* P, float* out, float sdiv, cudaStream_t s, const L2Prefetch* pf) {
  auto kern = attnc_kernel<HD, KT>;
  constexpr int smem = AttnCfg<HD, KT>::SMEM;
  const int rc = set_smem_limit((const void*)kern, smem, "attention (cluster)");
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ATTNC_CLUSTER, nh);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = ATTNC_CLUSTER;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const L2Prefetch none;
  const cudaError_t e =
      cudaLaunchKernelEx(&cfg, kern, q, nh, nkv, (const KT*)kc, (const KT*)vc, bt, bs, P, out, sdiv, pf ? *pf : none);
  if (e != cudaSuccess) {
    set_error("attention (cluster) launch: %s", cudaGetErrorString(e));
    return LUMINA_E_CUDA;
  }
  return LUMINA_OK;
}

}  // namespace

int launch_attention_cluster(bool fp16, int hd, const float* q, int nh, int nkv, const void* kc, const void* vc,
                             const int* bt, int bs, const DevParams* P, float* out, cudaStream_t s,
                             const L2Prefetch* pf) {
  const float sdiv = std::max(sqrtf((float)hd), 1e-6f);  // max(hd ** 0.5, 1e-6), chat.py:278
  if (hd == 128) return fp16 ? launch_one<128, __half>(q, nh, nkv, kc, vc, bt, bs, P, out, sdiv, s, pf)
                             : launch_one<128, float>(q, nh, nkv, kc, vc, bt, bs, P, out, sdiv, s, pf);
  if (hd == 64) return fp16 ? launch_one<64, __half>(q, nh, nkv, kc, vc, bt, bs, P, out, sdiv, s, pf)
                            : launch_one<64, float>(q, nh, nkv, kc, vc, bt, bs, P, out, sdiv, s, pf);
  set_error("attention: head_dim %d not built (64, 128)", hd);
  return LUMINA_E_UNSUPPORTED;
}

}  // namespace lumina
