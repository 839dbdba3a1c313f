// int8 fused GEMV family with the TOPS C-ABI semantics (host buffers in and
// out, caller owns every buffer). Replaces kernels/tops_int8.c:
//   tops_gemv_int8   :41-66   out[n] = (sum_b xs[b]*dot32 + tail) * ws[n]
//   tops_gemv_q4_0   :73-106  out[n] = sum_b dot32(x, code-8)*xs[b]*ws[n,b] + tail
//   tops_gemv_fp16   :225-243 out[n] = sum_k x[k]*w[n,k] (fp32 accumulate here;
//                            the NEON kernel accumulates 8 fp16 lanes)
//   tops_gemm_int8   :300-326 out[m,n] = ws[n] * sum_b xs[m,b]*dot32 (tail ignored)
// "tail" = columns past the last whole 32-block, added unscaled exactly as the
// reference kernels do. One warp per output; lane b takes 32-blocks b, b+32...
#include <mutex>

#include "common.cuh"

namespace lumina {

__device__ __forceinline__ int dot32_s8(const int8_t* a, const int8_t* b, bool aligned) {
  int d = 0;
  if (aligned) {
    const int4* pa = reinterpret_cast<const int4*>(a);
    const int4* pb = reinterpret_cast<const int4*>(b);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int4 va = __ldg(pa + q), vb = __ldg(pb + q);
      d = __dp4a(va.x, vb.x, d);
      d = __dp4a(va.y, vb.y, d);
      d = __dp4a(va.z, vb.z, d);
      d = __dp4a(va.w, vb.w, d);
    }
  } else {
    for (int j = 0; j < 32; ++j) d += (int)a[j] * (int)b[j];
  }
  return d;
}

// mode 0: int8 GEMV/GEMM, mode 1: q4_0
template <int MODE>
__global__ void tops_kernel(const int8_t* __restrict__ xq, const float* __restrict__ xs,
                            const uint8_t* __restrict__ wq, const float* __restrict__ ws,
                            float* __restrict__ out, int M, int N, int K, int with_tail) {
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int n_warps = (gridDim.x * blockDim.x) >> 5;
  const int nb = K >> 5;
  for (int task = gw; task < M * N; task += n_warps) {
    const int m = task / N, n = task % N;
    const int8_t* xr = xq + (size_t)m * K;
    const float* xsr = xs + (size_t)m * nb;
    float acc = 0.f;
    if (MODE == 0) {
      const int8_t* wr = reinterpret_cast<const int8_t*>(wq) + (size_t)n * K;
      const bool al = ((K & 15) == 0);
      for (int b = lane; b < nb; b += 32)
        acc = fmaf((float)dot32_s8(xr + 32 * b, wr + 32 * b, al), xsr[b], acc);
    } else {
      const uint8_t* wr = wq + (size_t)n * (K >> 1);
      for (int b = lane; b < nb; b += 32) {
        int d = 0;
        for (int j = 0; j < 16; ++j) {
          const int byte = wr[16 * b + j];
          d += (int)xr[32 * b + 2 * j] * ((byte & 15) - 8) + (int)xr[32 * b + 2 * j + 1] * ((byte >> 4) - 8);
        }
        acc += (float)d * xsr[b] * ws[(size_t)n * nb + b];
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) {
      int tail = 0;
      if (with_tail) {
        for (int k = nb << 5; k < K; ++k) {
          int wv;
          if (MODE == 0) {
            wv = reinterpret_cast<const int8_t*>(wq)[(size_t)n * K + k];
          } else {
            const int byte = wq[(size_t)n * (K >> 1) + (k >> 1)];
            wv = ((k & 1) ? (byte >> 4) : (byte & 15)) - 8;
          }
          tail += (int)xr[k] * wv;
        }
      }
      float v = MODE == 0 ? (acc + (float)tail) * ws[n] : acc + (float)tail;
      out[(size_t)m * N + n] = v;
    }
  }
}

__global__ void fp16_gemv_kernel(const __half* __restrict__ x, const __half* __restrict__ w,
                                 float* __restrict__ out, int N, int K) {
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int n_warps = (gridDim.x * blockDim.x) >> 5;
  for (int n = gw; n < N; n += n_warps) {
    const __half* wr = w + (size_t)n * K;
    float acc = 0.f;
    for (int k = lane; k < K; k += 32) acc = fmaf(__half2float(x[k]), __half2float(wr[k]), acc);
    acc = warp_sum(acc);
    if (lane == 0) out[n] = acc;
  }
}

// growable per-process staging buffer for the host-pointer entries
static std::mutex g_mu;
static void* g_buf = nullptr;
static size_t g_cap = 0;
static int g_dev = -1;

static int staging(size_t bytes, void** out) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (g_buf && (g_cap < bytes || g_dev != dev)) {
    int prev = dev;
    cudaSetDevice(g_dev);
    cudaFree(g_buf);
    cudaSetDevice(prev);
    g_buf = nullptr;
    g_cap = 0;
  }
  if (!g_buf) {
    if (cudaMalloc(&g_buf, bytes) != cudaSuccess) {
      cudaGetLastError();
      set_error("tops staging: cudaMalloc(%zu) failed", bytes);
      return LUMINA_E_OOM;
    }
    g_cap = bytes;
    g_dev = dev;
  }
  *out = g_buf;
  return LUMINA_OK;
}

static size_t al(size_t v) { return (v + 255) & ~size_t(255); }

static int run_tops(int mode, const int8_t* xq, const float* xs, const uint8_t* wq, size_t wbytes,
                    const float* ws, size_t ws_n, float* out, int M, int N, int K, int with_tail) {
  LUMINA_CHECK_ARG(xq && xs && wq && ws && out, "tops: null pointer");
  LUMINA_CHECK_ARG(M > 0 && N > 0 && K > 0, "tops: bad shape M=%d N=%d K=%d", M, N, K);
  const int nb = K >> 5;
  const size_t bx = al((size_t)M * K), bxs = al((size_t)M * (nb ? nb : 1) * 4), bw = al(wbytes),
               bws = al(ws_n * 4), bo = al((size_t)M * N * 4);
  std::lock_guard<std::mutex> lk(g_mu);
  void* base = nullptr;
  int rc = staging(bx + bxs + bw + bws + bo, &base);
  if (rc) return rc;
  char* p = static_cast<char*>(base);
  int8_t* dx = reinterpret_cast<int8_t*>(p);
  float* dxs = reinterpret_cast<float*>(p + bx);
  uint8_t* dw = reinterpret_cast<uint8_t*>(p + bx + bxs);
  float* dws = reinterpret_cast<float*>(p + bx + bxs + bw);
  float* dout = reinterpret_cast<float*>(p + bx + bxs + bw + bws);
  LUMINA_CUDA_TRY(cudaMemcpy(dx, xq, (size_t)M * K, cudaMemcpyHostToDevice));
  if (nb) LUMINA_CUDA_TRY(cudaMemcpy(dxs, xs, (size_t)M * nb * 4, cudaMemcpyHostToDevice));
  LUMINA_CUDA_TRY(cudaMemcpy(dw, wq, wbytes, cudaMemcpyHostToDevice));
  LUMINA_CUDA_TRY(cudaMemcpy(dws, ws, ws_n * 4, cudaMemcpyHostToDevice));
  const long warps = (long)M * N;
  const int blocks = (int)std::min<long>((warps + 7) / 8, 8L * sm_count());
  if (mode == 0)
    tops_kernel<0><<<blocks, 256>>>(dx, dxs, dw, dws, dout, M, N, K, with_tail);
  else
    tops_kernel<1><<<blocks, 256>>>(dx, dxs, dw, dws, dout, M, N, K, with_tail);
  LUMINA_LAUNCH_CHECK();
  LUMINA_CUDA_TRY(cudaMemcpy(out, dout, (size_t)M * N * 4, cudaMemcpyDeviceToHost));
  return LUMINA_OK;
}

}  // namespace lumina

using namespace lumina;

extern "C" {

int lumina_gemv_int8(const int8_t* xq, const float* xs, const int8_t* wq, const float* ws, float* out,
                     int N, int K) {
  return run_tops(0, xq, xs, reinterpret_cast<const uint8_t*>(wq), (size_t)N * K, ws, (size_t)N, out, 1,
                  N, K, 1);
}

int lumina_gemv_q4_0(const int8_t* xq, const float* xs, const uint8_t* wq, const float* ws, float* out,
                     int N, int K) {
  LUMINA_CHECK_ARG(K % 2 == 0, "gemv_q4_0: K=%d must be even", K);
  return run_tops(1, xq, xs, wq, (size_t)N * (K / 2), ws, (size_t)N * (K >> 5), out, 1, N, K, 1);
}

int lumina_gemm_int8(const int8_t* xq, const float* xs, const int8_t* wq, const float* ws, float* out,
                     int M, int N, int K) {
  return run_tops(0, xq, xs, reinterpret_cast<const uint8_t*>(wq), (size_t)N * K, ws, (size_t)N, out, M,
                  N, K, 0);
}

int lumina_gemv_fp16(const void* x, const void* w, float* out, int N, int K) {
  LUMINA_CHECK_ARG(x && w && out && N > 0 && K > 0, "gemv_fp16: bad arguments");
  std::lock_guard<std::mutex> lk(g_mu);
  const size_t bx = al((size_t)K * 2), bw = al((size_t)N * K * 2), bo = al((size_t)N * 4);
  void* base = nullptr;
  int rc = staging(bx + bw + bo, &base);
  if (rc) return rc;
  char* p = static_cast<char*>(base);
  LUMINA_CUDA_TRY(cudaMemcpy(p, x, (size_t)K * 2, cudaMemcpyHostToDevice));
  LUMINA_CUDA_TRY(cudaMemcpy(p + bx, w, (size_t)N * K * 2, cudaMemcpyHostToDevice));
  const int blocks = std::min((N + 7) / 8, 8 * sm_count());
  fp16_gemv_kernel<<<blocks, 256>>>(reinterpret_cast<const __half*>(p), reinterpret_cast<const __half*>(p + bx),
                                    reinterpret_cast<float*>(p + bx + bw), N, K);
  LUMINA_LAUNCH_CHECK();
  LUMINA_CUDA_TRY(cudaMemcpy(out, p + bx + bw, (size_t)N * 4, cudaMemcpyDeviceToHost));
  return LUMINA_OK;
}

}  // extern "C"
