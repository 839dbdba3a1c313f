// Device layout of packed Lumina weights and of quantized activations.
//
// Weights: row-major, each row padded to a whole number of 16-byte "chunks"
// (48-byte chunks for int3). One 32-column "block" of a row is BITS 32-bit
// words:
//   int4   4 words, byte j of a word = columns 2j (low nibble), 2j+1 (high)
//          -- the file's nibble layout (adapters/lumina.py:20-27) unchanged
//   int2   2 words, byte j = columns 4j..4j+3 in bits 0-1..6-7
//          -- the file's 2-bit layout (adapters/lumina.py:30-40) unchanged
//   binary 1 word, bit t of byte j = column 8j+t, 1 = +1
//          -- the file's sign bytes (ptq_ladder.py:37-47) unchanged
//   int3   3 words: two 2-bit planes of the low code bits in the int2 layout
//          (columns 0-15, 16-31) and one plane of the high bits where bit t
//          of byte j is column 4j+t and bit 4+t is column 16+4j+t
//          -- re-packed from the file's byte-per-code layout (3 bits/code)
// Scales: (rows, n_groups) fp16 when every F32 scale is exactly an fp16
// value (then bit-identical), else fp32.
//
// Activations (int16, per 32-column block, in the order the dp2a code paths
// consume): P8 for int4, P16 for int2/int3, P32 for binary.
#pragma once
#include "common.cuh"

struct lumina_weight {
  int device;
  int bits;         // 1, 2, 3, 4
  int group;        // columns per scale (multiple of 32)
  int rows, cols;
  int nblk;         // ceil(cols / 32)
  int n_chunks;     // ceil(nblk / blocks_per_chunk)
  int row_bytes;    // n_chunks * chunk_bytes
  int n_groups;     // ceil(cols / group)
  int fp16_scales;  // 1: half scales, 0: float scales
  uint8_t* codes;   // rows * row_bytes
  void* scales;     // rows * n_groups
  size_t bytes;     // device bytes held
};

namespace lumina {

template <int BITS>
struct Layout {
  static constexpr int CHUNK_WORDS = (BITS == 3) ? 12 : 4;
  static constexpr int CB = CHUNK_WORDS / BITS;  // 32-column blocks per chunk
  static constexpr int CHUNK_BYTES = CHUNK_WORDS * 4;
  static constexpr int L = (1 << BITS) - 1;      // levels - 1
};

__host__ __device__ inline int chunk_bytes(int bits) { return bits == 3 ? 48 : 16; }
__host__ __device__ inline int blocks_per_chunk(int bits) { return bits == 3 ? 4 : 4 / bits; }
inline int perm_kind(int bits) { return bits == 4 ? 8 : (bits == 1 ? 32 : 16); }

// Quantized activation scratch for one GEMV input.
struct ActQ {
  int16_t* xq;   // [batch][nblk_pad][32], permuted
  float* sx;     // [batch][nblk_pad]: amax / 32767
  int* xsum;     // [batch][nblk_pad]: L * sum(xq) of the block
  int nblk_pad;
};

// Activation quantization (optionally fused with RMSNorm). `x` rows have
// stride ldx; `norm_w` may be null.
int act_quant(const float* x, int ldx, int batch, int K, const float* norm_w, float eps,
              int bits, const ActQ& q, cudaStream_t s);

enum { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2 };

struct GemvArgs {
  const uint8_t* codes;
  const void* scales;
  int rows, row_bytes, n_chunks, n_groups, group;
  const int16_t* xq;
  const float* sx;
  const int* xsum;
  int nblk_pad;
  float* y;
  int ldy;
  const float* resid;
  int ldr;
};

int gemv_launch(const lumina_weight* w, const ActQ& q, int batch, float* y, int ldy, int epi,
                const float* resid, int ldr, cudaStream_t s);

// Per-device activation scratch owned by the library (grown on demand).
int scratch_actq(int device, int batch, int nblk_pad, ActQ* out);

}  // namespace lumina
