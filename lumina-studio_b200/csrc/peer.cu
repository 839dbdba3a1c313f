// Tensor-parallel exchange over peer memory (NVLink / NVSwitch): the sum
// after each row-parallel projection (o_proj, down_proj) added into the
// residual stream, and the gather of the vocab-sharded head logits -- one
// kernel each, in place of a library collective plus an add kernel.
//
// Every rank owns one exchange region: [flags: PEER_CTAS x PEER_MAX u32]
// [slot 0][slot 1][slot 2], a slot holding one rank's contribution (slot 0:
// o_proj partial sums, 1: down_proj partials, 2: a logits shard). The regions
// are shared between the ranks' processes with CUDA IPC handles, so each rank
// holds a device pointer to every peer's region.
//
// One exchange: the producing kernel (the GEMV before this one) has written
// this rank's contribution into its own slot. CTA c of the exchange kernel
// waits for that kernel (griddepcontrol.wait), then tells every rank t "my
// slot is complete" by a release store of the exchange's epoch into t's
// flags[c][rank], and waits (acquire loads, bounded by the global timer)
// until its own flags[c][r] hold that epoch for every rank r. It then reads
// its share of every rank's slot over NVLink and either adds their sum (rank
// order, so every rank computes the same bits) into the residual x, or copies
// the shards side by side into the full logits.
//
// Why slots are safe to reuse: ranks run the same exchanges in the same
// order, and epochs grow by one per exchange. A rank rewrites slot p only
// after passing the barrier of a later exchange (which reads other slots),
// and a peer reaches that barrier only after its kernels that read slot p
// have completed. A wait that runs out of time sets bit 2 of the device fault
// word and leaves the output untouched; the host turns that into an error.
#include "model.cuh"

namespace lumina {

namespace {

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// a peer's (or this rank's) slot: never served from a stale L1 line
__device__ __forceinline__ float4 ld_volatile4(const float* p) {
  float4 v;
  asm volatile("ld.volatile.global.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

template <int MODE>
__global__ void __launch_bounds__(PEER_THREADS) peer_exchange_kernel(PeerArgs a) {
  __shared__ unsigned s_epoch;
  __shared__ int s_ok;
  pdl_launch_dependents();
  pdl_wait();  // this rank's slot (the previous kernel's output) is complete
  const int c = blockIdx.x, tid = threadIdx.x;
  if (tid == 0) {
    s_epoch = a.epoch[c] + 1u;
    s_ok = 1;
  }
  __syncthreads();
  const unsigned ep = s_epoch;
  if (tid < a.tp) {
    __threadfence_system();
    st_release_sys(a.flags[tid] + c * PEER_MAX + a.rank, ep);
    const unsigned* f = a.flags[a.rank] + c * PEER_MAX + tid;
    const unsigned long long t0 = global_ns();
    while ((int)(ld_acquire_sys(f) - ep) < 0) {
      if (global_ns() - t0 >= a.timeout_ns) {
        atomicOr(a.fault, 4);
        s_ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  if (tid == 0) a.epoch[c] = ep;
  if (!s_ok) return;
  const size_t n4 = a.n / 4;
  for (size_t i = (size_t)c * PEER_THREADS + tid; i < n4; i += (size_t)PEER_CTAS * PEER_THREADS) {
    if constexpr (MODE == PEER_SUM) {
      float4 s = ld_volatile4(a.slot[0] + 4 * i);
      for (int r = 1; r < a.tp; ++r) {
        const float4 v = ld_volatile4(a.slot[r] + 4 * i);
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
      float4* xo = reinterpret_cast<float4*>(a.out) + i;
      float4 x = *xo;
      x.x += s.x;
      x.y += s.y;
      x.z += s.z;
      x.w += s.w;
      *xo = x;
    } else {
      for (int r = 0; r < a.tp; ++r)
        reinterpret_cast<float4*>(a.out + (size_t)r * a.n)[i] = ld_volatile4(a.slot[r] + 4 * i);
    }
  }
}

}  // namespace

int launch_peer_exchange(const PeerArgs& a, int mode, cudaStream_t s) {
  if (a.n % 4) {
    set_error("peer exchange: %zu floats is not a multiple of 4", a.n);
    return LUMINA_E_ARG;
  }
  const cudaError_t e = mode == PEER_SUM
                            ? launch_pdl(peer_exchange_kernel<PEER_SUM>, dim3(PEER_CTAS), dim3(PEER_THREADS), 0, s, a)
                            : launch_pdl(peer_exchange_kernel<PEER_GATHER>, dim3(PEER_CTAS), dim3(PEER_THREADS), 0,
                                         s, a);
  if (e != cudaSuccess) {
    set_error("peer exchange launch: %s", cudaGetErrorString(e));
    return LUMINA_E_CUDA;
  }
  return LUMINA_OK;
}

}  // namespace lumina
