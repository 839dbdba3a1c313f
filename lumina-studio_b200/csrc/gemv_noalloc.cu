// lumina_gemv_noalloc: the packed dequant GEMV for callers that cannot
// allocate device memory.
//
// lumina_gemv quantizes the activation rows into a per-device scratch buffer
// that the library grows with cudaMalloc on first use (and frees and
// re-allocates when a larger one is needed). Some callers cannot allow that:
// a host runtime that owns every device allocation through its own pool, a
// caller that must not take the device-wide synchronisation a cudaFree
// implies, or one that has budgeted all device memory up front. This entry
// point runs the same two kernels as lumina_gemv's batched path
// (act_quant_kernel then gemv_kernel) with the activation scratch in a
// fixed array that is part of the library's own device image instead.
//
// The array, `g_noalloc_scratch`, is LUMINA_NOALLOC_SCRATCH_BYTES (1 MiB) on
// every GPU that loads the library, held until the process exits. Host code
// cannot use its name as a device address (the name is a host-side stand-in),
// so the first call on each device, with that device current, looks the
// address up with cudaGetSymbolAddress and keeps it; later calls reuse it.
// Every call shares the one array and leaves its contents behind; act_quant
// writes every slot the GEMV then reads, so nothing has to be cleared.
#include <mutex>

#include "weights.cuh"

#ifndef LUMINA_NOALLOC_SCRATCH_BYTES
#define LUMINA_NOALLOC_SCRATCH_BYTES (1u << 20)
#endif

static __device__ __align__(256) unsigned char g_noalloc_scratch[LUMINA_NOALLOC_SCRATCH_BYTES];

namespace {

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};

// device address of g_noalloc_scratch on `device` (which must be current)
int noalloc_scratch(int device, void** out) {
  if (device < 0 || device >= 64) {
    lumina::set_error("gemv_noalloc: bad device %d", device);
    return LUMINA_E_ARG;
  }
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      lumina::set_error("gemv_noalloc: cudaGetSymbolAddress on device %d: %s", device, cudaGetErrorString(e));
      return LUMINA_E_CUDA;
    }
    g_noalloc_ptr[device] = p;
  }
  *out = g_noalloc_ptr[device];
  return LUMINA_OK;
}

}  // namespace

extern "C" int lumina_gemv_noalloc(const lumina_weight* w, const float* x_dev, int batch, int ldx, float* y_dev,
                                   int ldy, void* stream) {
  using namespace lumina;
  LUMINA_CHECK_ARG(w && x_dev && y_dev, "gemv_noalloc: null pointer");
  LUMINA_CHECK_ARG(batch >= 1 && batch <= 16, "gemv_noalloc: batch %d not in 1..16", batch);
  LUMINA_CHECK_ARG(ldx >= w->cols && ldy >= w->rows, "gemv_noalloc: ldx %d / ldy %d smaller than (%d, %d)", ldx,
                   ldy, w->cols, w->rows);
  if (w->mma) {
    set_error("gemv_noalloc: weights in the tensor-core fragment layout are not supported");
    return LUMINA_E_UNSUPPORTED;
  }
  const int nblk_pad = w->n_chunks * blocks_per_chunk(w->bits);
  const size_t need = actq_scratch_bytes(batch, nblk_pad);
  if (need > LUMINA_NOALLOC_SCRATCH_BYTES) {
    set_error("gemv_noalloc: batch %d x %d columns needs %zu bytes of activation scratch, more than the fixed %u",
              batch, w->cols, need, (unsigned)LUMINA_NOALLOC_SCRATCH_BYTES);
    return LUMINA_E_ARG;
  }
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess || (prev != w->device && cudaSetDevice(w->device) != cudaSuccess)) {
    set_error("gemv_noalloc: cannot make device %d current", w->device);
    return LUMINA_E_CUDA;
  }
  void* base = nullptr;
  int rc = noalloc_scratch(w->device, &base);
  if (!rc) {
    ActQ q;
    actq_carve(base, batch, nblk_pad, &q);
    cudaStream_t s = (cudaStream_t)stream;
    rc = act_quant(x_dev, ldx, batch, w->cols, nullptr, 0.f, w->bits, q, s);
    if (!rc) rc = gemv_launch(w, q, batch, y_dev, ldy, EPI_STORE, nullptr, 0, s);
  }
  if (prev >= 0 && prev != w->device) cudaSetDevice(prev);
  return rc;
}
