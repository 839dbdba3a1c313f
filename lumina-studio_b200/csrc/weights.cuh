// Device layout of packed Lumina weights and of quantized activations.
//
// Codes of one row are cut into 16-byte "chunks" (48-byte for int3). A
// 32-column "block" of codes is BITS 32-bit words:
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
// Rows are row-major, each padded to a whole number of chunks, and the row
// count is padded to a multiple of 4 with zero rows. Scales are row-major
// too, each row padded to a multiple of 16 bytes so that the scales of R
// consecutive rows are one contiguous, bulk-copyable span. Scales are fp16
// when every F32 scale is exactly an fp16 value (then bit-identical), else
// fp32.
//
// Activations (int16, per 32-column block, in the order the dp2a code paths
// consume): P8 for int4, P16 for int2/int3, P32 for binary.
#pragma once
#include "common.cuh"

constexpr int ROW_PAD = 4;

struct lumina_weight {
  int device;
  int bits;          // 1, 2, 3, 4
  int group;         // columns per scale (a multiple of 32)
  int rows, cols;
  int rows_pad;      // rows rounded up to ROW_PAD
  int nblk;          // ceil(cols / 32)
  int n_chunks;      // chunks per row
  int row_bytes;     // n_chunks * chunk bytes
  int n_groups;      // ceil(cols / group)
  int spr;           // scale bytes per row (16-byte multiple)
  int fp16_scales;   // 1: half scales, 0: float scales
  int mma;           // 1: int4 in the tensor-core fragment layout (gemv_mma.cu):
                     //    rows_pad % 32 == 0, n_chunks = 32-column blocks
                     //    rounded up to pairs, codes [tile16][pair][lane][16 B],
                     //    scales [tile16][group][g][2]
  uint8_t* codes;    // rows_pad * row_bytes
  uint8_t* scales;   // rows_pad * spr
  size_t bytes;      // device bytes held
};

namespace lumina {

// device bytes of the codes and of the scales of a weight
inline size_t weight_code_bytes(const lumina_weight& w) { return (size_t)w.rows_pad * w.row_bytes; }
inline size_t weight_scale_bytes(const lumina_weight& w) {
  return w.mma ? (size_t)w.rows_pad * w.n_groups * (w.fp16_scales ? 2 : 4) : (size_t)w.rows_pad * w.spr;
}
// an L2 prefetch of a whole weight (codes and scales)
inline L2Prefetch prefetch_of(const lumina_weight* w) {
  L2Prefetch pf;
  if (!w) return pf;
  pf.p[0] = w->codes;
  pf.n[0] = weight_code_bytes(*w) & ~size_t(15);
  pf.p[1] = w->scales;
  pf.n[1] = weight_scale_bytes(*w) & ~size_t(15);
  return pf;
}

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

// code of (row, col) in the tensor-core fragment layout
__host__ __device__ inline size_t mma_code_byte(const lumina_weight& w, int row, int col, int* nibble) {
  const int T = row >> 4, rr = row & 15, g = rr & 7;
  const int b = col >> 5, cc = col & 31;
  const int lane = g * 4 + ((cc & 15) >> 2);
  const int j = (b & 1) * 2 + (cc >> 4);
  *nibble = rr >> 3;
  return (((size_t)T * (w.n_chunks / 2) + (b >> 1)) * 32 + lane) * 16 + j * 4 + (cc & 3);
}
__host__ __device__ inline size_t mma_scale_offset(const lumina_weight& w, int row, int grp) {
  const int es = w.fp16_scales ? 2 : 4;
  return ((((size_t)(row >> 4) * w.n_groups + grp) * 8 + (row & 7)) * 2 + ((row & 15) >> 3)) * es;
}

// byte offset of chunk `c` of row `row` (row-major layout)
__host__ __device__ inline size_t code_offset(const lumina_weight& w, int row, int c) {
  return (size_t)row * w.row_bytes + (size_t)c * chunk_bytes(w.bits);
}

// byte offset of the scale of (row, group g)
__host__ __device__ inline size_t scale_offset(const lumina_weight& w, int row, int g) {
  return (size_t)row * w.spr + (size_t)g * (w.fp16_scales ? 2 : 4);
}

// Quantized activation scratch for one GEMV input (global memory layout).
struct ActQ {
  int16_t* xq;   // [batch][nblk_pad][32], permuted
  float* sx;     // [batch][nblk_pad]: amax / 32767
  int* xsum;     // [batch][nblk_pad]: L * sum(xq) of the block
  int nblk_pad;
};

// Activation quantization (optionally fused with RMSNorm). `x` rows have
// stride ldx; `norm_w` may be null.
int act_quant(const float* x, int ldx, int batch, int K, const float* norm_w, float eps, int bits,
              const ActQ& q, cudaStream_t s);

enum { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_ROPE_KV = 3 };

// RoPE + paged KV append for the fused q/k/v projection (EPI_ROPE_KV). The
// q and k rows of the weight are permuted so that rotation pairs (j,
// j + hd/2) of a head are adjacent rows (2j', 2j'+1).
struct RopeKV {
  int nh, nkv, hd;
  const float* cos_t;
  const float* sin_t;
  const int* row_pos;   // per batch row
  const int* t_prev;    // device: KV length before this forward
  const int* block_table;
  int bs;
  void* kcache;         // this layer's pool
  void* vcache;
  int kv_fp16;
  float* q_out;         // (batch, nh*hd) rotated queries
  int row_base;         // KV slot of batch row b is *t_prev + row_base + b
};

struct GemvArgs {
  lumina_weight w;
  const int16_t* xq;
  const float* sx;
  const int* xsum;
  int nblk_pad;
  float* y;
  int ldy;
  const float* resid;
  int ldr;
  RopeKV rk;
};

// Packed GEMV reading pre-quantized activations from global memory (any
// batch; the path for prefill chunks).
int gemv_launch(const lumina_weight* w, const ActQ& q, int batch, float* y, int ldy, int epi,
                const float* resid, int ldr, cudaStream_t s, const RopeKV* rk = nullptr);

// Decode GEMV: 128-bit code loads software-pipelined in registers, scale
// rows bulk-copied (TMA) into shared memory, activations quantized (and RMS-
// normalized when norm_w is given) inside each CTA. batch 1, 2 or 4. Returns
// LUMINA_E_UNSUPPORTED when the shape does not fit (callers then use
// act_quant + gemv_launch).
int gemv_fused_launch(const lumina_weight* w, const float* x, int ldx, int batch, const float* norm_w, float eps,
                      float* y, int ldy, int epi, const float* resid, int ldr, cudaStream_t s,
                      const RopeKV* rk = nullptr);

// int4 GEMV on the tensor pipe (weights in the fragment layout), any batch
// in tiles of 8. LUMINA_E_UNSUPPORTED when the weight is not in that layout
// or the shape does not fit.
int gemv_mma_launch(const lumina_weight* w, const float* x, int ldx, int batch, const float* norm_w, float eps,
                    float* y, int ldy, int epi, const float* resid, int ldr, cudaStream_t s,
                    const RopeKV* rk = nullptr);

// The tensor-parallel sum of a row-parallel projection fused into the decode
// GEMVs on both sides of it (no exchange kernel in between). The producer
// (EPI_STORE) writes its rows into every rank's receive slot for this rank
// (push[r], peer memory over NVLink), and its last CTA (ticket) advances
// this rank's epoch of the exchange and release-stores it into every rank's
// flag for this rank (flags[r]). The consumer (a NORM prologue) reads the
// epoch its own producer set, waits until in_flags[r] holds it for every
// rank r (bounded by timeout_ns), reads x + sum over r of add[r] (rank
// order: every rank computes the same bits), and CTA 0 stores that sum in
// xout, the residual the next exchange builds on.
constexpr int TCTP_MAX = 8;
struct TcTp {
  int tp = 0;  // ranks; 0: not part of an exchange
  int ld = 0;  // floats per row in the slots
  float* push[TCTP_MAX] = {};
  unsigned* flags[TCTP_MAX] = {};
  int* ticket = nullptr;
  const float* add[TCTP_MAX] = {};
  const unsigned* in_flags = nullptr;
  float* xout = nullptr;
  unsigned* epoch = nullptr;
  unsigned long long timeout_ns = 0;
};

// int4 decode GEMV on the tensor pipe (gemv_tc.cu), batch 1, 2 or 4 (3 runs
// as 4), weights in the fragment layout with group = 64 * 2^k.
// LUMINA_E_UNSUPPORTED when the shape does not fit.
// `pf` (may be null): the next kernel's bytes to pull into L2 meanwhile.
// `tp` (may be null): this GEMV's side of a fused tensor-parallel exchange.
int gemv_tc_launch(const lumina_weight* w, const float* x, int ldx, int batch, const float* norm_w, float eps,
                   float* y, int ldy, int epi, const float* resid, int ldr, cudaStream_t s, const RopeKV* rk,
                   const L2Prefetch* pf = nullptr, const TcTp* tp = nullptr);

// Workspace of a kernel whose grid splits its reduction (K of a projection,
// the keys of an attention row block) over several CTAs: partial results go
// to `ws`, and the CTA that takes the last ticket of its tile's counter
// combines them in split order (deterministic, no CTA waits on another).
// Counters start at zero and the combining CTA resets its own, so kernels of
// one stream can share the workspace; kernels on different streams cannot.
struct SplitWork {
  float* ws = nullptr;
  size_t ws_elems = 0;
  int* cnt = nullptr;
  int cnt_n = 0;
};
// per-device workspace for the library's own entry points (lumina_gemm_rows)
int split_scratch(int device, SplitWork* out);
constexpr size_t SPLIT_WS_ELEMS = (size_t)8 << 20;  // 32 MiB of fp32 partials
constexpr int SPLIT_COUNTERS = 8192;

// Multi-row int4 projection on tcgen05 (gemm_tc05.cu): x (M rows, stride
// ldx, fp32) -> fp16 hi and lo planes in x16 (gemm_tc05_x16_elems(M, cols)
// halves; RMSNorm fused when norm_w is given) -> y (M rows, stride ldy).
// Epilogues: G5_STORE (rows < qk_rows of a fused q/k/v weight are stored at
// their un-permuted index, head size hd), G5_RESID (y = resid + W x),
// G5_SWIGLU (interleaved gate/up rows -> silu(gate) * up at row / 2). With
// `sw`, a grid of fewer tiles than SMs splits K over CTAs.
// LUMINA_E_UNSUPPORTED when the weight is not int4 in the fragment layout.
enum { G5_STORE = 0, G5_RESID = 1, G5_SWIGLU = 2 };
size_t gemm_tc05_x16_elems(int rows, int cols);
int gemm_tc05_launch(const lumina_weight* w, const float* x, int ldx, int M, const float* norm_w, float eps,
                     __half* x16, float* y, int ldy, int epi, const float* resid, int ldr, int qk_rows, int hd,
                     cudaStream_t s, const SplitWork* sw = nullptr);
// The same contraction with a dense fp16 weight W (rows x K, row-major, K a
// multiple of 8; the LM head): y[m, r] = sum_k x[m, k] W[r, k], stored.
int dense_tc05_launch(const __half* W, int rows, int K, const float* x, int ldx, int M, __half* x16, float* y,
                      int ldy, cudaStream_t s, const SplitWork* sw = nullptr);

// int4 GEMV on the tensor pipe for 1..32 activation rows (gemv_tcb.cu),
// weights in the fragment layout: x (M rows, stride ldx; RMSNorm fused when
// norm_w is given) -> int16 B fragments in `frag` (gemv_tcb_frag_bytes(M,
// cols) bytes, 16-byte aligned) -> y. Epilogues EPI_STORE (rows < qk_rows of
// a fused q/k/v weight are stored at their un-permuted index, head size hd),
// EPI_RESID, EPI_SWIGLU, EPI_ROPE_KV (with `rk`, as the decode GEMV). K is split over the CTAs of a thread-block
// cluster (partials combined over distributed shared memory, in slice
// order) when the fragments of a whole row do not fit a CTA's shared memory
// or the grid would leave SMs idle. LUMINA_E_UNSUPPORTED when the weight or
// the shape does not fit.
size_t gemv_tcb_frag_bytes(int M, int cols);
int gemv_tcb_launch(const lumina_weight* w, const float* x, int ldx, int M, const float* norm_w, float eps,
                    void* frag, size_t frag_bytes, float* y, int ldy, int epi, const float* resid, int ldr,
                    int qk_rows, int hd, cudaStream_t s, const RopeKV* rk = nullptr);
// per-device fragment scratch for the library's own entry points
int tcb_frag_scratch(int device, size_t bytes, void** out);

// Per-device activation scratch owned by the library (grown on demand).
int scratch_actq(int device, int batch, int nblk_pad, ActQ* out);
// Bytes of, and carving of, one activation scratch region at `base`.
size_t actq_scratch_bytes(int batch, int nblk_pad);
void actq_carve(void* base, int batch, int nblk_pad, ActQ* out);

// Device-side error word: bounded waits that give up set a bit here.
int read_fault_flag(int* out);
int* fault_flag_ptr();
// stream-ordered clear of the current device's fault word
int clear_fault_async(cudaStream_t s);
// LUMINA_E_CUDA with the text of a set fault word
int fault_error(const char* what, int word);

}  // namespace lumina
