// Shared definitions for liblumina_cuda (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stddef.h>

#include "lumina_cuda.h"

namespace lumina {

// Per-thread last error text; every C-ABI entry sets it before returning a
// non-zero status (the ctypes layer turns it into {"error": ...}).
void set_error(const char* fmt, ...);
const char* get_error();

#define LUMINA_CUDA_TRY(expr)                                                   \
  do {                                                                          \
    cudaError_t _e = (expr);                                                    \
    if (_e != cudaSuccess) {                                                    \
      ::lumina::set_error("%s: %s (%s:%d)", #expr, cudaGetErrorString(_e),     \
                          __FILE__, __LINE__);                                  \
      return LUMINA_E_CUDA;                                                     \
    }                                                                           \
  } while (0)

#define LUMINA_CHECK_ARG(cond, ...)                                             \
  do {                                                                          \
    if (!(cond)) {                                                              \
      ::lumina::set_error(__VA_ARGS__);                                         \
      return LUMINA_E_ARG;                                                      \
    }                                                                           \
  } while (0)

#define LUMINA_LAUNCH_CHECK()                                                   \
  do {                                                                          \
    cudaError_t _e = cudaGetLastError();                                        \
    if (_e != cudaSuccess) {                                                    \
      ::lumina::set_error("kernel launch: %s (%s:%d)", cudaGetErrorString(_e), \
                          __FILE__, __LINE__);                                  \
      return LUMINA_E_CUDA;                                                     \
    }                                                                           \
  } while (0)

// Streaming, read-only 128-bit load that does not allocate in L1 (weights are
// touched once per GEMV).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// Read-only cached 128-bit load (activations: reused by every row of a warp).
__device__ __forceinline__ uint4 ldg_cached(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Programmatic dependent launch: let the next kernel in the stream start its
// independent prologue, and wait for the previous kernel's writes.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

int sm_count();

// Bytes that the kernel launched next in the stream will stream from HBM,
// pulled into L2 by the running kernel (one bulk prefetch per piece), so that
// HBM keeps streaming across the launch boundary instead of idling while the
// next kernel's CTAs start and issue their first requests. A hint only: it
// moves no data a kernel reads through any path but L2.
struct L2Prefetch {
  const void* p[2] = {nullptr, nullptr};  // contiguous ranges, 16-byte aligned
  unsigned long long n[2] = {0, 0};       // their sizes, multiples of 16 bytes
  // the paged KV rows [0, *len) of one layer: blocks bt[0 .. ceil(*len / bs))
  // of kc and vc, block_bytes each (a multiple of 16)
  const void* kc = nullptr;
  const void* vc = nullptr;
  const int* bt = nullptr;
  const int* len = nullptr;
  int bs = 0;
  unsigned block_bytes = 0;
};

__device__ __forceinline__ void l2_prefetch(const void* p, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Worker w of nw (one thread each) prefetches its share of every range, in
// pieces of at most 64 KB.
__device__ __forceinline__ void l2_prefetch_share(const L2Prefetch& pf, int w, int nw) {
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const unsigned long long n = pf.n[r];
    if (!n) continue;
    const unsigned long long per = ((n + nw - 1) / nw + 15) & ~15ull;
    const unsigned long long s0 = (unsigned long long)w * per;
    if (s0 >= n) continue;
    const unsigned long long len = per < n - s0 ? per : n - s0;
    const char* base = static_cast<const char*>(pf.p[r]) + s0;
    for (unsigned long long o = 0; o < len; o += 65536)
      l2_prefetch(base + o, (unsigned)(len - o < 65536 ? len - o : 65536));
  }
  if (pf.bt) {
    const int nblk = (*pf.len + pf.bs - 1) / pf.bs;
    for (int b = w; b < 2 * nblk; b += nw) {
      const char* base = static_cast<const char*>((b & 1) ? pf.vc : pf.kc) + (size_t)pf.bt[b >> 1] * pf.block_bytes;
      for (unsigned o = 0; o < pf.block_bytes; o += 65536)
        l2_prefetch(base + o, pf.block_bytes - o < 65536u ? pf.block_bytes - o : 65536u);
    }
  }
}

// Raise `func`'s dynamic shared-memory limit to at least `bytes` on the
// current device (cached per kernel and device, thread-safe).
int set_smem_limit(const void* func, size_t bytes, const char* what);

// Polls a kernel makes on a pending shared-memory transfer before it gives up
// and sets the device fault word: WAIT_SPIN_DEFAULT (about a second) unless
// lumina_debug_wait_limit changed it. Passed to kernels as an argument.
constexpr long long WAIT_SPIN_DEFAULT = 1LL << 24;
long long wait_spin_limit();

// Launch a kernel with the programmatic-stream-serialization attribute so that
// it may begin while its predecessor drains (kernels call pdl_wait() before
// touching data the predecessor wrote).
template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern kernel, dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace lumina
