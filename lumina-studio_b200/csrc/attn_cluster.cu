// Single-query decode attention over the paged KV cache (chat.py:264-281
// with one new row: every key up to the row is visible, no bias).
//
// One thread-block cluster of ATTNC_CLUSTER CTAs per head; CTA r takes keys
// [r T / CS, (r + 1) T / CS) and each of its four warps a quarter of those.
// A warp streams its keys 16 at a time through its own double buffer of
// shared memory (cp.async, 16 bytes per copy; K rows padded by 16 bytes so
// that the eight lanes of a shared-memory phase hit distinct banks). Lane
// (h = lane / 16, j = lane % 16) forms the half-dot of head-dimension half h
// with key j and one shuffle completes the score; the warp keeps its own
// online softmax (fp32, the running max subtracted) and its output rows (4
// dimensions per lane for head_dim 128), so no CTA barrier runs inside the key
// loop. Only the new row (and q) come from the preceding q/k/v kernel; the
// key count and block table are fixed for the whole step, so the first two
// chunks are requested before the dependency wait without the new row, which
// is read after it. The four warps' (max, sum, output) merge in shared
// memory; the CTAs' merge in distributed shared memory, rank 0 adding them in
// rank order (deterministic) after a cluster barrier, a second barrier
// keeping every CTA's shared memory alive until rank 0 has read it. No
// global workspace, counters or atomics.
#include <cooperative_groups.h>

#include "model.cuh"

namespace lumina {

namespace {

namespace cg = cooperative_groups;

template <int HD, typename KT>
struct AttnCfg {
  static constexpr int ES = sizeof(KT);
  static constexpr int CK = 16;              // keys per warp chunk
  static constexpr int KROW = HD * ES + 16;  // padded K row (bytes)
  static constexpr int VROW = HD * ES;
  static constexpr int CH = HD * ES / 16;    // 16-byte pieces per row
  static constexpr int WBUF = CK * (KROW + VROW);
  static constexpr int DPL = HD / 32;        // output dims per lane
  // [4 warps][2 buffers][WBUF] | wm[4] wl[4] | wo[4][HD] | oc[HD] | ml[4]
  static constexpr int SMEM = 4 * 2 * WBUF + 8 * 4 + 4 * HD * 4 + HD * 4 + 16;
};

// One thread-block cluster of ATTNC_CLUSTER CTAs per head; CTA r takes keys
// [r T / CS, (r + 1) T / CS) and each of its four warps a quarter of them.
// A warp streams its keys 16 at a time through its own double buffer
// (cp.async), lanes (half h = lane / 16, key j = lane % 16) form half-dots
// that one shuffle completes, and the warp keeps its own online softmax and
// output (4 dims per lane), so no CTA barrier runs inside the key loop. The
// four warps then merge in shared memory, and rank 0 merges the CTAs in rank
// order over distributed shared memory.
template <int HD, typename KT>
__global__ void __launch_bounds__(128)
attnc_kernel(const float* __restrict__ q, int nh, int nkv, const KT* __restrict__ kcache,
             const KT* __restrict__ vcache, const int* __restrict__ block_table, int bs,
             const DevParams* __restrict__ P, float* __restrict__ out, float sdiv, L2Prefetch pf) {
  using C = AttnCfg<HD, KT>;
  constexpr int CS = ATTNC_CLUSTER, CK = C::CK, HH = HD / 2;
  cg::cluster_group cluster = cg::this_cluster();
  const int r = (int)cluster.block_rank();
  const int h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_launch_dependents();
  const int T = P->t_tot, knew = P->t_prev;
  const int k0 = (r * T) / CS, k1 = ((r + 1) * T) / CS, nk = k1 - k0;
  const int w0 = k0 + (warp * nk) / 4, w1 = k0 + ((warp + 1) * nk) / 4, nw = w1 - w0;
  const int kvh = h / (nh / nkv);
  const size_t bstride = (size_t)nkv * bs * HD;

  extern __shared__ __align__(16) uint8_t sm[];
  uint8_t* wbuf = sm + (size_t)warp * 2 * C::WBUF;
  float* wm = reinterpret_cast<float*>(sm + 4 * 2 * C::WBUF);
  float* wl = wm + 4;
  float* wo = wl + 4;     // [4][HD]
  float* oc = wo + 4 * HD;
  float* ml = oc + HD;    // m, l of this CTA

  auto issue = [&](int c, bool pre) {
    uint8_t* ks = wbuf + (size_t)(c & 1) * C::WBUF;
    uint8_t* vs = ks + (size_t)CK * C::KROW;
    const int j0 = w0 + c * CK, n = min(CK, w1 - j0);
    for (int i = lane; i < n * C::CH; i += 32) {
      const int j = i / C::CH, ch = i - j * C::CH;
      const int key = j0 + j;
      if (pre && key == knew) continue;
      const int blk = block_table[key / bs], off = key % bs;
      const size_t base = (size_t)blk * bstride + ((size_t)kvh * bs + off) * HD;
      const uint32_t kd = (uint32_t)__cvta_generic_to_shared(ks + (size_t)j * C::KROW + ch * 16);
      const uint32_t vd = (uint32_t)__cvta_generic_to_shared(vs + (size_t)j * C::VROW + ch * 16);
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(kd),
                   "l"(reinterpret_cast<const uint8_t*>(kcache + base) + ch * 16) : "memory");
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(vd),
                   "l"(reinterpret_cast<const uint8_t*>(vcache + base) + ch * 16) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  const int nch = (nw + CK - 1) / CK;
  issue(0, true);
  issue(1, true);
  if (tid == 0) l2_prefetch_share(pf, h * CS + r, gridDim.y * CS);
  pdl_wait();
  // the new row, when it sits in a chunk requested before the wait
  if (knew >= w0 && knew < w1 && (knew - w0) / CK < 2) {
    const int jj = knew - w0, c = jj / CK, j = jj - c * CK;
    uint8_t* ks = wbuf + (size_t)(c & 1) * C::WBUF;
    uint8_t* vs = ks + (size_t)CK * C::KROW;
    const int blk = block_table[knew / bs], off = knew % bs;
    const size_t base = (size_t)blk * bstride + ((size_t)kvh * bs + off) * HD;
    for (int ch = lane; ch < C::CH; ch += 32) {
      *reinterpret_cast<uint4*>(ks + (size_t)j * C::KROW + ch * 16) =
          __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(kcache + base) + ch * 16));
      *reinterpret_cast<uint4*>(vs + (size_t)j * C::VROW + ch * 16) =
          __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(vcache + base) + ch * 16));
    }
  }
  const int hf = lane >> 4, kj = lane & 15;
  float qh[HH];
#pragma unroll
  for (int d = 0; d < HH; d += 4) {
    const float4 f = __ldg(reinterpret_cast<const float4*>(q + (size_t)h * HD + hf * HH + d));
    qh[d] = f.x;
    qh[d + 1] = f.y;
    qh[d + 2] = f.z;
    qh[d + 3] = f.w;
  }
  float m_run = -INFINITY, l_run = 0.f, o[C::DPL];
#pragma unroll
  for (int d = 0; d < C::DPL; ++d) o[d] = 0.f;
  for (int c = 0; c < nch; ++c) {
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    __syncwarp();
    const uint8_t* ks = wbuf + (size_t)(c & 1) * C::WBUF;
    const uint8_t* vs = ks + (size_t)CK * C::KROW;
    const int n = min(CK, nw - c * CK);
    float part = 0.f;
    if (kj < n) {
      const uint4* kr = reinterpret_cast<const uint4*>(ks + (size_t)kj * C::KROW + hf * HH * C::ES);
#pragma unroll
      for (int cc = 0; cc < HH * C::ES / 16; ++cc) {
        const uint4 w = kr[cc];
        if constexpr (C::ES == 2) {
          const __half2* hh = reinterpret_cast<const __half2*>(&w);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(hh[e]);
            part = fmaf(qh[cc * 8 + 2 * e], f.x, part);
            part = fmaf(qh[cc * 8 + 2 * e + 1], f.y, part);
          }
        } else {
          part = fmaf(qh[cc * 4], __uint_as_float(w.x), part);
          part = fmaf(qh[cc * 4 + 1], __uint_as_float(w.y), part);
          part = fmaf(qh[cc * 4 + 2], __uint_as_float(w.z), part);
          part = fmaf(qh[cc * 4 + 3], __uint_as_float(w.w), part);
        }
      }
    }
    const float full = part + __shfl_xor_sync(0xffffffffu, part, 16);
    const float sc = kj < n ? __fdiv_rn(full, sdiv) : -INFINITY;
    float mc = sc;
#pragma unroll
    for (int o2 = 8; o2 > 0; o2 >>= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, o2));
    const float m_new = fmaxf(m_run, mc);
    const float alpha = m_run == -INFINITY ? 0.f : expf(m_run - m_new);
    const float p = kj < n ? expf(sc - m_new) : 0.f;
    float ps = p;
#pragma unroll
    for (int o2 = 8; o2 > 0; o2 >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o2);
    l_run = l_run * alpha + ps;
    m_run = m_new;
#pragma unroll
    for (int d = 0; d < C::DPL; ++d) o[d] *= alpha;
    for (int j = 0; j < n; ++j) {
      const float pj = __shfl_sync(0xffffffffu, p, j);
      const uint8_t* vr = vs + (size_t)j * C::VROW + lane * C::DPL * C::ES;
      if constexpr (C::ES == 2) {
        if constexpr (C::DPL == 4) {
          const uint2 raw = *reinterpret_cast<const uint2*>(vr);
          const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
          const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
          o[0] = fmaf(pj, a.x, o[0]);
          o[1] = fmaf(pj, a.y, o[1]);
          o[2] = fmaf(pj, b.x, o[2]);
          o[3] = fmaf(pj, b.y, o[3]);
        } else {
          const float2 a = __half22float2(*reinterpret_cast<const __half2*>(vr));
          o[0] = fmaf(pj, a.x, o[0]);
          o[1] = fmaf(pj, a.y, o[1]);
        }
      } else {
#pragma unroll
        for (int d = 0; d < C::DPL; ++d) o[d] = fmaf(pj, reinterpret_cast<const float*>(vr)[d], o[d]);
      }
    }
    __syncwarp();  // every lane is done with this buffer
    if (c + 2 < nch) issue(c + 2, false);
    else asm volatile("cp.async.commit_group;" ::: "memory");
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  // the four warps -> this CTA's (m, l, o)
  if (lane == 0) {
    wm[warp] = m_run;
    wl[warp] = l_run;
  }
#pragma unroll
  for (int d = 0; d < C::DPL; ++d) wo[warp * HD + lane * C::DPL + d] = o[d];
  __syncthreads();
  {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w]);
    float wg[4], L = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      wg[w] = wm[w] == -INFINITY ? 0.f : expf(wm[w] - M);
      L += wg[w] * wl[w];
    }
    for (int d = tid; d < HD; d += 128) {
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) acc = fmaf(wg[w], wo[w * HD + d], acc);
      oc[d] = acc;
    }
    if (tid == 0) {
      ml[0] = M;
      ml[1] = L;
    }
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
