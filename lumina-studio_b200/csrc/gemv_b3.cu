// Packed GEMV kernels for 3-bit codes (one translation unit per bit width).
#include "gemv_impl.cuh"

namespace lumina {
template int gemv_bits<3>(const GemvArgs&, int, int, int, cudaStream_t);
template int gemv_fused_bits<3>(FusedArgs&, const lumina_weight*, int, int, bool, cudaStream_t);
}  // namespace lumina
