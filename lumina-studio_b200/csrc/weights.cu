// Packed-weight upload, bit-exact unpack / dequant gates, lumina_gemv.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <atomic>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>
#include <vector>

#include "weights.cuh"

namespace lumina {

static thread_local char g_err[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}
const char* get_error() { return g_err; }

// per device, filled on first use (atomics: host threads may race to fill
// a slot; every one of them writes the same value)
int sm_count() {
  static std::atomic<int> n[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  int v = n[dev].load(std::memory_order_relaxed);
  if (!v) {
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    if (v <= 0) v = 148;
    n[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

// Dynamic shared-memory limits are a per-device attribute of a kernel: the
// largest limit granted so far is remembered per (kernel, device), under one
// lock, so a process that launches on several devices (or from several host
// threads) raises the limit on each device it uses.
int set_smem_limit(const void* func, size_t bytes, const char* what) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> granted;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    set_error("%s: no current device", what);
    return LUMINA_E_CUDA;
  }
  std::lock_guard<std::mutex> lk(mu);
  size_t& g = granted[std::make_pair(func, dev)];
  if (bytes <= g) return LUMINA_OK;
  const cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) {
    set_error("%s: shared-memory limit of %zu bytes on device %d: %s", what, bytes, dev, cudaGetErrorString(e));
    return LUMINA_E_CUDA;
  }
  g = bytes;
  return LUMINA_OK;
}

static std::atomic<long long> g_wait_spins{WAIT_SPIN_DEFAULT};
long long wait_spin_limit() { return g_wait_spins.load(std::memory_order_relaxed); }

// RAII device switch: entries run on the object's device and restore the
// caller's current device on return.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// ---------------------------------------------------------------------------
// per-device activation scratch
// ---------------------------------------------------------------------------
struct Scratch {
  void* base = nullptr;
  size_t bytes = 0;
};
static std::mutex g_scratch_mu;
static Scratch g_scratch[64];

static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

static size_t actq_bytes(int batch, int nblk_pad) {
  const size_t n = (size_t)batch * nblk_pad;
  return align256(n * 64) + align256(n * 4) + align256(n * 4);
}

static void carve_actq(void* base, int batch, int nblk_pad, ActQ* out) {
  const size_t n = (size_t)batch * nblk_pad;
  char* p = static_cast<char*>(base);
  out->xq = reinterpret_cast<int16_t*>(p);
  p += align256(n * 64);
  out->sx = reinterpret_cast<float*>(p);
  p += align256(n * 4);
  out->xsum = reinterpret_cast<int*>(p);
  out->nblk_pad = nblk_pad;
}

int scratch_actq(int device, int batch, int nblk_pad, ActQ* out) {
  if (device < 0 || device >= 64) {
    set_error("scratch: bad device %d", device);
    return LUMINA_E_ARG;
  }
  const size_t need = actq_bytes(batch, nblk_pad);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  Scratch& s = g_scratch[device];
  if (s.bytes < need) {
    if (s.base) {
      // a smaller scratch may still be read by queued work on any stream
      cudaDeviceSynchronize();
      cudaFree(s.base);
      s.base = nullptr;
      s.bytes = 0;
    }
    size_t want = std::max(need, (size_t)4 << 20);
    if (cudaMalloc(&s.base, want) != cudaSuccess) {
      cudaGetLastError();
      set_error("scratch: cudaMalloc(%zu) failed", want);
      return LUMINA_E_OOM;
    }
    s.bytes = want;
  }
  carve_actq(s.base, batch, nblk_pad, out);
  return LUMINA_OK;
}

size_t actq_scratch_bytes(int batch, int nblk_pad) { return actq_bytes(batch, nblk_pad); }
void actq_carve(void* base, int batch, int nblk_pad, ActQ* out) { carve_actq(base, batch, nblk_pad, out); }

// ---------------------------------------------------------------------------
// level table: np.linspace(-1, 1, 2^b) in float64 (ptq_ladder.py:58-59)
// ---------------------------------------------------------------------------
static void linspace_levels(int bits, double* out) {
  const int n = 1 << bits;
  const volatile double start = -1.0, stop = 1.0;
  const volatile double step = (stop - start) / (double)(n - 1);
  for (int c = 0; c < n; ++c) {
    volatile double y = (double)c * step;
    out[c] = y + start;
  }
  out[n - 1] = stop;  // numpy sets the endpoint exactly
}

__constant__ double c_levels[4][16];

// The device fault word: a bounded wait gave up in gemv_fused_kernel (bit
// 0), gemv_tc_kernel (bit 1), the tensor-parallel peer exchange (bit 2) or
// gemm_tc05_kernel (bit 3). Kernels only ever OR bits in; the host reads and
// clears it (lumina_fault_status, and every synchronous entry).
__device__ int g_fault_flag;

int* fault_flag_ptr() {
  static std::mutex mu;
  static int* p[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (!p[dev]) {
    void* a = nullptr;
    if (cudaGetSymbolAddress(&a, g_fault_flag) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    p[dev] = static_cast<int*>(a);
  }
  return p[dev];
}

int read_fault_flag(int* out) {
  int* p = fault_flag_ptr();
  if (!p) {
    set_error("fault flag: symbol address unavailable");
    return LUMINA_E_CUDA;
  }
  LUMINA_CUDA_TRY(cudaMemcpy(out, p, sizeof(int), cudaMemcpyDeviceToHost));
  return LUMINA_OK;
}

int clear_fault_async(cudaStream_t s) {
  int* p = fault_flag_ptr();
  if (!p) {
    set_error("fault flag: symbol address unavailable");
    return LUMINA_E_CUDA;
  }
  LUMINA_CUDA_TRY(cudaMemsetAsync(p, 0, sizeof(int), s));
  return LUMINA_OK;
}

int fault_error(const char* what, int word) {
  set_error("%s: a device wait timed out (fault word %#x:%s%s%s%s%s)", what, word,
            (word & 1) ? " gemv_fused_kernel" : "", (word & 2) ? " gemv_tc_kernel" : "",
            (word & 4) ? " peer exchange" : "", (word & 8) ? " gemm_tc05_kernel" : "", (word & 16) ? " gemv_tcb_kernel" : "");
  return LUMINA_E_CUDA;
}

static int ensure_levels() {
  int dev = 0;
  cudaGetDevice(&dev);
  static std::mutex mu;
  static bool done[64] = {false};
  std::lock_guard<std::mutex> lk(mu);
  if (dev >= 0 && dev < 64 && done[dev]) return LUMINA_OK;
  double h[4][16] = {};
  for (int b = 1; b <= 4; ++b) linspace_levels(b, h[b - 1]);
  LUMINA_CUDA_TRY(cudaMemcpyToSymbol(c_levels, h, sizeof(h)));
  if (dev >= 0 && dev < 64) done[dev] = true;
  return LUMINA_OK;
}

// ---------------------------------------------------------------------------
// unpack / dequant gates (read the device layout back to one code per byte)
// ---------------------------------------------------------------------------
__device__ __forceinline__ int device_code(const lumina_weight& w, int r, int k) {
  if (w.mma) {
    int nib = 0;
    const size_t o = mma_code_byte(w, r, k, &nib);
    return (w.codes[o] >> (4 * nib)) & 0xF;
  }
  const int blk = k >> 5, j = k & 31;
  const int cbk = blocks_per_chunk(w.bits);
  const uint8_t* chunk = w.codes + code_offset(w, r, blk / cbk);
  const uint32_t* bw = reinterpret_cast<const uint32_t*>(chunk) + (blk % cbk) * w.bits;
  switch (w.bits) {
    case 4: return (bw[j >> 3] >> (4 * (j & 7))) & 0xF;
    case 2: return (bw[j >> 4] >> (2 * (j & 15))) & 0x3;
    case 1: return (bw[0] >> j) & 0x1;
    default: {  // int3
      const int half = j >> 4, i = j & 15;
      const int lo = (bw[half] >> (2 * i)) & 0x3;
      const int hbit = (bw[2] >> (4 * half + (i >> 2) * 8 + (i & 3))) & 0x1;
      return lo | (hbit << 2);
    }
  }
}

__device__ __forceinline__ float device_scale(const lumina_weight& w, int r, int g) {
  const uint8_t* p = w.scales + (w.mma ? mma_scale_offset(w, r, g) : scale_offset(w, r, g));
  return w.fp16_scales ? __half2float(*reinterpret_cast<const __half*>(p)) : *reinterpret_cast<const float*>(p);
}

__global__ void unpack_kernel(const lumina_weight w, uint8_t* out) {
  const size_t n = (size_t)w.rows * w.cols;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / w.cols), k = (int)(i % w.cols);
    out[i] = (uint8_t)device_code(w, r, k);
  }
}

__global__ void dequant_kernel(const lumina_weight w, float* out) {
  const size_t n = (size_t)w.rows * w.cols;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / w.cols), k = (int)(i % w.cols);
    const int c = device_code(w, r, k);
    const float s = device_scale(w, r, k / w.group);
    // adapters/lumina.py:138-139 (int) / :145-148 (binary, levels are -1/+1)
    out[i] = __double2float_rn(__dmul_rn((double)s, c_levels[w.bits - 1][c]));
  }
}

}  // namespace lumina

using namespace lumina;

// ---------------------------------------------------------------------------
// host-side re-tiling of one file record into the device layout
// ---------------------------------------------------------------------------
static int file_code(int kind, int pack, const uint8_t* rowp, int k) {
  if (pack == LUMINA_PACK_NIBBLE) return (rowp[k >> 1] >> (4 * (k & 1))) & 0xF;
  if (pack == LUMINA_PACK_2BIT) return (rowp[k >> 2] >> (2 * (k & 3))) & 0x3;
  if (kind == LUMINA_KIND_BINARY) return (rowp[k >> 3] >> (k & 7)) & 0x1;
  return rowp[k];
}

extern "C" {

int lumina_cuda_version(void) { return LUMINA_CUDA_VERSION; }

const char* lumina_last_error(void) { return lumina::get_error(); }

int lumina_device_count(int* n) {
  LUMINA_CHECK_ARG(n, "device_count: null out");
  int v = 0;
  cudaError_t e = cudaGetDeviceCount(&v);
  if (e != cudaSuccess) {
    cudaGetLastError();
    *n = 0;
    set_error("cudaGetDeviceCount: %s", cudaGetErrorString(e));
    return LUMINA_E_CUDA;
  }
  *n = v;
  return LUMINA_OK;
}

int lumina_weight_upload(int device, int kind, int group_size, int pack, const uint8_t* codes_host,
                         size_t codes_len, const float* scales_host, size_t n_scales, int rows, int cols,
                         lumina_weight** out) {
  LUMINA_CHECK_ARG(out && codes_host && scales_host, "weight_upload: null pointer");
  *out = nullptr;
  LUMINA_CHECK_ARG(kind >= 1 && kind <= 4, "weight_upload: kind %d not in 1..4", kind);
  LUMINA_CHECK_ARG(rows > 0 && cols > 0, "weight_upload: bad shape (%d, %d)", rows, cols);
  if (group_size <= 0 || group_size % 32) {
    set_error("weight_upload: group_size %d must be a positive multiple of 32", group_size);
    return LUMINA_E_UNSUPPORTED;
  }
  const int expect_pack = kind == 4 ? LUMINA_PACK_NIBBLE : (kind == 2 ? LUMINA_PACK_2BIT : LUMINA_PACK_NONE);
  // the reader honours the flag; int4/int2 may also arrive unpacked (legacy
  // files without the flag, adapters/lumina.py:51,76)
  LUMINA_CHECK_ARG(pack == expect_pack || pack == LUMINA_PACK_NONE,
                   "weight_upload: packed flag %d does not match kind %d", pack, kind);
  const int n_groups = (cols + group_size - 1) / group_size;
  LUMINA_CHECK_ARG(n_scales == (size_t)rows * n_groups,
                   "weight_upload: %zu scales for (%d, %d) at group %d (want %zu)", n_scales, rows, cols,
                   group_size, (size_t)rows * n_groups);
  // file row stride: derived from the blob length like unpack_codes
  // (adapters/lumina.py:53-60) for packed kinds
  int per_byte = 1;
  if (pack == LUMINA_PACK_NIBBLE) per_byte = 2;
  else if (pack == LUMINA_PACK_2BIT) per_byte = 4;
  else if (kind == LUMINA_KIND_BINARY) per_byte = 8;
  LUMINA_CHECK_ARG(codes_len % rows == 0, "weight_upload: codes blob %zu not divisible by %d rows",
                   codes_len, rows);
  const size_t stride = codes_len / rows;
  LUMINA_CHECK_ARG(stride * per_byte >= (size_t)cols, "weight_upload: codes blob too short for %d columns",
                   cols);
  if (pack == LUMINA_PACK_NONE && kind != LUMINA_KIND_BINARY)
    LUMINA_CHECK_ARG(stride == (size_t)cols, "weight_upload: byte-per-code blob is not (%d, %d)", rows, cols);
  if (kind == LUMINA_KIND_BINARY)
    LUMINA_CHECK_ARG(stride == (size_t)(cols + 7) / 8, "weight_upload: sign blob stride %zu for %d columns",
                     stride, cols);

  const int bits = kind;
  lumina_weight L{};
  L.device = device;
  L.bits = bits;
  L.group = group_size;
  L.rows = rows;
  L.cols = cols;
  L.rows_pad = (rows + ROW_PAD - 1) / ROW_PAD * ROW_PAD;
  L.nblk = (cols + 31) / 32;
  const int cbk = blocks_per_chunk(bits), chb = chunk_bytes(bits);
  L.n_chunks = (L.nblk + cbk - 1) / cbk;
  L.row_bytes = L.n_chunks * chb;
  L.n_groups = n_groups;
  // codes: each file row re-packed into device chunks (a plain copy for the
  // kinds whose file layout is the device layout)
  std::vector<uint8_t> dev((size_t)L.rows_pad * L.row_bytes, 0);
  const bool same_layout = (bits == 4 && pack == LUMINA_PACK_NIBBLE) ||
                           (bits == 2 && pack == LUMINA_PACK_2BIT) || bits == 1;
  for (int r = 0; r < rows; ++r) {
    const uint8_t* src = codes_host + (size_t)r * stride;
    uint8_t* dst = dev.data() + (size_t)r * L.row_bytes;
    if (same_layout) {
      const size_t nb = ((size_t)cols * bits + 7) / 8;
      memcpy(dst, src, nb);
      const int tail = (cols * bits) % 8;  // clear bits past the last column
      if (tail) dst[nb - 1] &= (uint8_t)((1u << tail) - 1);
      continue;
    }
    uint32_t* dw = reinterpret_cast<uint32_t*>(dst);
    for (int k = 0; k < cols; ++k) {
      const int c = file_code(kind, pack, src, k);
      if (c > (1 << bits) - 1) {
        set_error("weight_upload: code %d out of range for int%d at (%d, %d)", c, bits, r, k);
        return LUMINA_E_ARG;
      }
      const int blk = k >> 5, j = k & 31;
      uint32_t* bw = dw + (size_t)(blk / cbk) * (chb / 4) + (blk % cbk) * bits;
      switch (bits) {
        case 4: bw[j >> 3] |= (uint32_t)c << (4 * (j & 7)); break;
        case 2: bw[j >> 4] |= (uint32_t)c << (2 * (j & 15)); break;
        case 1: bw[0] |= (uint32_t)c << j; break;
        default: {
          const int half = j >> 4, i = j & 15;
          bw[half] |= (uint32_t)(c & 3) << (2 * i);
          bw[2] |= (uint32_t)((c >> 2) & 1) << (4 * half + (i >> 2) * 8 + (i & 3));
        }
      }
    }
  }
  // scales: fp16 when lossless; rows padded to 16 bytes
  bool fp16 = true;
  for (size_t i = 0; i < n_scales; ++i) {
    const float s = scales_host[i];
    if (!std::isfinite(s)) {
      set_error("weight_upload: non-finite scale at %zu", i);
      return LUMINA_E_ARG;
    }
    if (__half2float(__float2half_rn(s)) != s) fp16 = false;
  }
  L.fp16_scales = fp16 ? 1 : 0;
  const int es = fp16 ? 2 : 4;
  L.spr = (n_groups * es + 15) / 16 * 16;
  std::vector<uint8_t> sdev;
  // int4 goes to the tensor-core fragment layout when LUMINA_INT4_LAYOUT=mma
  // (gemv_tc.cu for batch <= 4, gemv_tcb.cu for 5..32, gemv_mma.cu beyond);
  // a model converts its own int4 projections to that layout when it is
  // finalized. int3 / int2 / binary go there too, one code per nibble, when
  // LUMINA_NARROW_LAYOUT=mma: 4 bits of device memory per code instead of
  // 3 / 2 / 1, for the tensor-pipe GEMVs of lumina_gemv (batch <= 16)
  const char* lay = getenv(bits == 4 ? "LUMINA_INT4_LAYOUT" : "LUMINA_NARROW_LAYOUT");
  const bool want_mma = lay && strcmp(lay, "mma") == 0;
  const int gpw = group_size / 64;
  if (group_size % 64 == 0 && (gpw & (gpw - 1)) == 0 && gpw <= 4 && want_mma) {
    // tensor-core fragment layout (gemv_mma.cu): built from the row-major codes
    L.mma = 1;
    const int nbp = (L.nblk + 1) / 2 * 2;
    const int rows32 = (rows + 31) / 32 * 32;
    std::vector<uint8_t> m((size_t)rows32 * nbp * 16, 0);
    lumina_weight M = L;
    M.n_chunks = nbp;
    M.row_bytes = nbp * 16;
    M.rows_pad = rows32;
    for (int r = 0; r < rows; ++r) {
      const uint8_t* src = dev.data() + (size_t)r * L.row_bytes;  // int4: the nibble row
      const uint8_t* fsrc = codes_host + (size_t)r * stride;       // narrow kinds: the file row
      for (int k = 0; k < cols; ++k) {
        const int c = bits == 4 ? (src[k >> 1] >> (4 * (k & 1))) & 0xF : file_code(kind, pack, fsrc, k);
        int nib = 0;
        const size_t o = mma_code_byte(M, r, k, &nib);
        m[o] |= (uint8_t)(c << (4 * nib));
      }
    }
    sdev.assign((size_t)rows32 * n_groups * es, 0);
    for (int r = 0; r < rows; ++r)
      for (int gi = 0; gi < n_groups; ++gi) {
        const float s = scales_host[(size_t)r * n_groups + gi];
        uint8_t* d = sdev.data() + mma_scale_offset(M, r, gi);
        if (fp16) {
          const __half h = __float2half_rn(s);
          memcpy(d, &h, 2);
        } else {
          memcpy(d, &s, 4);
        }
      }
    dev.swap(m);
    L = M;
  } else {
    sdev.assign((size_t)L.rows_pad * L.spr, 0);
    for (int r = 0; r < rows; ++r)
      for (int gi = 0; gi < n_groups; ++gi) {
        const float s = scales_host[(size_t)r * n_groups + gi];
        uint8_t* d = sdev.data() + scale_offset(L, r, gi);
        if (fp16) {
          const __half h = __float2half_rn(s);
          memcpy(d, &h, 2);
        } else {
          memcpy(d, &s, 4);
        }
      }
  }

  DeviceGuard g(device);
  lumina_weight* w = new lumina_weight(L);
  w->codes = nullptr;
  w->scales = nullptr;
  w->bytes = dev.size() + sdev.size();
  if (cudaMalloc(&w->codes, dev.size()) != cudaSuccess || cudaMalloc(&w->scales, sdev.size()) != cudaSuccess) {
    cudaGetLastError();
    if (w->codes) cudaFree(w->codes);
    delete w;
    set_error("weight_upload: cudaMalloc of %zu bytes failed", dev.size() + sdev.size());
    return LUMINA_E_OOM;
  }
  cudaError_t e1 = cudaMemcpy(w->codes, dev.data(), dev.size(), cudaMemcpyHostToDevice);
  cudaError_t e2 = cudaMemcpy(w->scales, sdev.data(), sdev.size(), cudaMemcpyHostToDevice);
  if (e1 != cudaSuccess || e2 != cudaSuccess) {
    cudaFree(w->codes);
    cudaFree(w->scales);
    delete w;
    set_error("weight_upload: copy failed: %s", cudaGetErrorString(e1 != cudaSuccess ? e1 : e2));
    return LUMINA_E_CUDA;
  }
  *out = w;
  return LUMINA_OK;
}

int lumina_weight_free(lumina_weight* w) {
  if (!w) return LUMINA_OK;
  DeviceGuard g(w->device);
  cudaFree(w->codes);
  cudaFree(w->scales);
  delete w;
  return LUMINA_OK;
}

int lumina_weight_info(const lumina_weight* w, int* kind, int* group_size, int* rows, int* cols,
                       size_t* device_bytes, int* fp16_scales) {
  LUMINA_CHECK_ARG(w, "weight_info: null weight");
  if (kind) *kind = w->bits;
  if (group_size) *group_size = w->group;
  if (rows) *rows = w->rows;
  if (cols) *cols = w->cols;
  if (device_bytes) *device_bytes = w->bytes;
  if (fp16_scales) *fp16_scales = w->fp16_scales;
  return LUMINA_OK;
}

int lumina_weight_unpack(const lumina_weight* w, uint8_t* codes_dev, void* stream) {
  LUMINA_CHECK_ARG(w && codes_dev, "weight_unpack: null pointer");
  DeviceGuard g(w->device);
  unpack_kernel<<<4 * sm_count(), 256, 0, (cudaStream_t)stream>>>(*w, codes_dev);
  LUMINA_LAUNCH_CHECK();
  return LUMINA_OK;
}

int lumina_weight_dequant(const lumina_weight* w, float* out_dev, void* stream) {
  LUMINA_CHECK_ARG(w && out_dev, "weight_dequant: null pointer");
  DeviceGuard g(w->device);
  int rc = ensure_levels();
  if (rc) return rc;
  dequant_kernel<<<4 * sm_count(), 256, 0, (cudaStream_t)stream>>>(*w, out_dev);
  LUMINA_LAUNCH_CHECK();
  return LUMINA_OK;
}

int lumina_gemv(const lumina_weight* w, const float* x_dev, int batch, int ldx, float* y_dev, int ldy,
                void* stream) {
  LUMINA_CHECK_ARG(w && x_dev && y_dev, "gemv: null pointer");
  LUMINA_CHECK_ARG(batch >= 1 && batch <= 16, "gemv: batch %d not in 1..16", batch);
  LUMINA_CHECK_ARG(ldx >= w->cols && ldy >= w->rows, "gemv: ldx %d / ldy %d smaller than (%d, %d)", ldx,
                   ldy, w->cols, w->rows);
  DeviceGuard g(w->device);
  cudaStream_t s = (cudaStream_t)stream;
  if (w->mma) {
    if (batch <= 4) {
      const int rc = gemv_tc_launch(w, x_dev, ldx, batch, nullptr, 0.f, y_dev, ldy, EPI_STORE, nullptr, 0, s, nullptr);
      if (rc != LUMINA_E_UNSUPPORTED) return rc;
    } else {
      // 5..16 rows: the batched tensor-pipe GEMV (gemv_tcb.cu)
      void* frag = nullptr;
      const size_t fb = gemv_tcb_frag_bytes(batch, w->cols);
      int rc = tcb_frag_scratch(w->device, fb, &frag);
      if (rc) return rc;
      rc = gemv_tcb_launch(w, x_dev, ldx, batch, nullptr, 0.f, frag, fb, y_dev, ldy, EPI_STORE, nullptr, 0, 0, 0, s);
      if (rc != LUMINA_E_UNSUPPORTED) return rc;
    }
    return gemv_mma_launch(w, x_dev, ldx, batch, nullptr, 0.f, y_dev, ldy, EPI_STORE, nullptr, 0, s);
  }
  if (batch <= 4) {
    const int rc = gemv_fused_launch(w, x_dev, ldx, batch, nullptr, 0.f, y_dev, ldy, EPI_STORE, nullptr, 0, s);
    if (rc != LUMINA_E_UNSUPPORTED) return rc;
  }
  const int nblk_pad = w->n_chunks * blocks_per_chunk(w->bits);
  ActQ q;
  int rc = scratch_actq(w->device, batch, nblk_pad, &q);
  if (rc) return rc;
  rc = act_quant(x_dev, ldx, batch, w->cols, nullptr, 0.f, w->bits, q, s);
  if (rc) return rc;
  return gemv_launch(w, q, batch, y_dev, ldy, EPI_STORE, nullptr, 0, s);
}

int lumina_fault_status(int device, int* word, int clear) {
  LUMINA_CHECK_ARG(word, "fault_status: null output");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
    cudaGetLastError();
    set_error("fault_status: device %d not available", device);
    return LUMINA_E_ARG;
  }
  DeviceGuard g(device);
  int* p = fault_flag_ptr();
  if (!p) {
    set_error("fault_status: fault word unavailable on device %d", device);
    return LUMINA_E_CUDA;
  }
  LUMINA_CUDA_TRY(cudaDeviceSynchronize());
  LUMINA_CUDA_TRY(cudaMemcpy(word, p, sizeof(int), cudaMemcpyDeviceToHost));
  if (clear && *word) LUMINA_CUDA_TRY(cudaMemset(p, 0, sizeof(int)));
  return LUMINA_OK;
}

int lumina_debug_wait_limit(long long spins) {
  g_wait_spins.store(spins < 0 ? WAIT_SPIN_DEFAULT : spins, std::memory_order_relaxed);
  return LUMINA_OK;
}

int lumina_gemv_host(const lumina_weight* w, const float* x_host, int batch, float* y_host) {
  LUMINA_CHECK_ARG(w && x_host && y_host, "gemv_host: null pointer");
  LUMINA_CHECK_ARG(batch >= 1 && batch <= 16, "gemv_host: batch %d not in 1..16", batch);
  DeviceGuard g(w->device);
  float *xd = nullptr, *yd = nullptr;
  const size_t xb = (size_t)batch * w->cols * 4, yb = (size_t)batch * w->rows * 4;
  if (cudaMalloc(&xd, xb) != cudaSuccess || cudaMalloc(&yd, yb) != cudaSuccess) {
    cudaGetLastError();
    if (xd) cudaFree(xd);
    set_error("gemv_host: cudaMalloc failed");
    return LUMINA_E_OOM;
  }
  int rc = LUMINA_OK;
  if (cudaMemcpy(xd, x_host, xb, cudaMemcpyHostToDevice) != cudaSuccess) {
    set_error("gemv_host: H2D copy failed");
    rc = LUMINA_E_CUDA;
  }
  if (!rc) rc = clear_fault_async(nullptr);
  if (!rc) rc = lumina_gemv(w, xd, batch, w->cols, yd, w->rows, nullptr);
  if (!rc && cudaMemcpy(y_host, yd, yb, cudaMemcpyDeviceToHost) != cudaSuccess) {
    set_error("gemv_host: D2H copy failed: %s", cudaGetErrorString(cudaGetLastError()));
    rc = LUMINA_E_CUDA;
  }
  int word = 0;
  if (!rc) rc = read_fault_flag(&word);
  if (!rc && word) {
    cudaMemset(fault_flag_ptr(), 0, sizeof(int));
    rc = fault_error("gemv_host", word);
  }
  cudaFree(xd);
  cudaFree(yd);
  return rc;
}

}  // extern "C"
