// Decode model internals shared by model.cu and model_kernels.cu.
#pragma once
#include <array>
#include <vector>

#include "weights.cuh"

namespace lumina {

// Per-forward values the kernels read from device memory, so that one
// captured CUDA graph serves every decode position.
struct DevParams {
  int n;         // rows in this forward
  int t_prev;    // KV length before the append
  int t_tot;     // t_prev + n
  int n_splits;  // unused (1)
  int bias_ld;   // columns of the bias matrix (= t_tot)
  int pad[3];
};

template <typename KT>
__device__ __forceinline__ KT to_kv(float v);
template <>
__device__ __forceinline__ float to_kv<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half to_kv<__half>(float v) { return __float2half_rn(v); }

__device__ __forceinline__ float from_kv(float v) { return v; }
__device__ __forceinline__ float from_kv(__half v) { return __half2float(v); }

// DL consecutive KV elements -> fp32 (16-byte loads).
template <typename KT, int DL>
__device__ __forceinline__ void load_kv(const KT* p, float* out) {
  if constexpr (sizeof(KT) == 2) {
    static_assert(DL % 8 == 0, "fp16 KV slice must be a multiple of 8");
#pragma unroll
    for (int q = 0; q < DL / 8; ++q) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(p) + q);
      const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(h[e]);
        out[q * 8 + 2 * e] = f.x;
        out[q * 8 + 2 * e + 1] = f.y;
      }
    }
  } else {
    static_assert(DL % 4 == 0, "fp32 KV slice must be a multiple of 4");
#pragma unroll
    for (int q = 0; q < DL / 4; ++q) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(p) + q);
      out[4 * q] = v.x;
      out[4 * q + 1] = v.y;
      out[4 * q + 2] = v.z;
      out[4 * q + 3] = v.w;
    }
  }
}

int launch_embed(const __half* emb, int d, int vocab, const int* tokens, const DevParams* P, float* x, int max_n,
                 unsigned long long* argmax_key, cudaStream_t s);
int launch_rope_append(bool fp16, const float* qkv, int nh, int nkv, int hd, const float* cos_t, const float* sin_t,
                       const int* row_pos, const DevParams* P, const int* bt, int bs, void* kc, void* vc,
                       float* q_out, int max_n, cudaStream_t s);
// attention of several query rows (prefill, tree verification) on the tensor
// pipe: one CTA per (head, 64 rows), K/V tiles of 64 keys (attn_rows.cu);
// when heads x row blocks leave SMs idle, the keys (t_tot of them, the host's
// copy of P->t_tot) split over CTAs whose partial softmax states `sw` holds
int launch_attention_rows(bool fp16, int hd, const float* q, int nh, int nkv, const void* kc, const void* vc,
                          const int* bt, int bs, const int* row_pos, const float* bias, const DevParams* P, float* out,
                          int max_n, int t_tot, const SplitWork* sw, cudaStream_t s);
// single-query decode attention (one new row, no bias): one cluster of
// ATTNC_CLUSTER CTAs per head, keys streamed in chunks of ATTNC_CHUNK
constexpr int ATTNC_CLUSTER = 8;
constexpr int ATTNC_CHUNK = 64;
int launch_attention_cluster(bool fp16, int hd, const float* q, int nh, int nkv, const void* kc, const void* vc,
                             const int* bt, int bs, const DevParams* P, float* out, cudaStream_t s,
                             const L2Prefetch* pf = nullptr);

// Virtual-MoE MLP (moe.cu): router scores, gate/up + SwiGLU of the picked
// experts, transposed down projection + residual, in place on x.
constexpr int MOE_MAX_E = 64;      // experts per layer
constexpr int MOE_MAX_K = 8;       // top-k
constexpr int MOE_ROWS = 4;        // batch rows per pass of the expert kernels
constexpr int MOE_PPC = 8;         // (gate, up) neuron pairs per CTA: one per warp
constexpr int MOE_SPLITS_MAX = 8;  // neuron ranges of the down projection
inline int moe_splits(int n) { return n <= 32 ? MOE_SPLITS_MAX : 4; }
// rows of down partials a forward of up to max_rows rows needs
inline size_t moe_part_rows(int max_rows) {
  const int a = max_rows < 32 ? max_rows : 32;
  const size_t p1 = (size_t)moe_splits(a) * a, p2 = (size_t)moe_splits(max_rows) * max_rows;
  return p1 > p2 ? p1 : p2;
}
struct MoeLayerArgs {
  const lumina_weight* gate_up;  // (E*2Ie, d) int4, row-major chunk layout
  const lumina_weight* down;     // (E*Ie, d)
  const float* router_w;         // (E, d) fp32 (fp16-rounded values)
  const float* router_b;         // (E) or null
  const float* norm_w;           // post-attention RMSNorm weight
  float eps;
  int E, Ie, K, d;
  // expert parallelism: this rank holds experts [e_lo, e_lo + e_n) (rows of
  // gate_up / down, in order); the router covers all E
  int e_lo = 0, e_n = 0;
  float* out = nullptr;  // null: x += MLP(x); else out = this rank's share of MLP(x)
};
struct MoeScratch {
  float* h;                 // (rows, d) normalized rows
  float* score;             // (rows, MOE_MAX_E) router scores
  float* act;               // (rows, K, Ie) silu(g) * u
  float* part;              // (moe_part_rows(max_rows), d) down partials
  unsigned int* counters;   // d / 64, zero between launches
};
int moe_check(const MoeLayerArgs& a);
int moe_prepare(int d);
int launch_moe(const MoeLayerArgs& a, int n, const MoeScratch& sc, float* x, cudaStream_t s);

// Tensor-parallel exchange over peer memory (peer.cu).
constexpr int PEER_MAX = 8;        // ranks
constexpr int PEER_CTAS = 32;      // CTAs of every exchange (each owns one flag slot per rank)
constexpr int PEER_THREADS = 256;
constexpr size_t PEER_FLAG_BYTES = 4096;  // PEER_CTAS x PEER_MAX u32, padded
enum { PEER_SUM = 0, PEER_GATHER = 1 };
struct PeerArgs {
  const float* slot[PEER_MAX];  // this exchange's slot on every rank (rank order)
  unsigned* flags[PEER_MAX];    // every rank's flag array
  unsigned* epoch;              // this rank's per-CTA exchange counters
  int tp, rank;
  size_t n;                     // floats per rank's contribution
  float* out;                   // PEER_SUM: x += sum (n floats); PEER_GATHER: tp * n floats
  int* fault;
  unsigned long long timeout_ns;
};
int launch_peer_exchange(const PeerArgs& a, int mode, cudaStream_t s);

int launch_dense_gemv(const __half* W, int N, int K, const float* x, int ldx, int batch, float* y, int ldy,
                      const float* resid, int ldr, cudaStream_t s, unsigned long long* amax = nullptr,
                      const L2Prefetch* pf = nullptr);
int launch_gather_rows(const lumina_weight& out, const lumina_weight& s0, const lumina_weight& s1,
                       const lumina_weight& s2, const int* sel, const int* srow, cudaStream_t s);
int launch_swiglu(const float* g, const float* u, float* o, int n, int ffn, int ld, cudaStream_t s);
int launch_argmax(const float* v, int n, int* out, cudaStream_t s);
int launch_kv_read(bool fp16, const void* kc, const void* vc, const int* bt, int bs, int nh, int nkv, int hd,
                   int start, int n, float* ko, float* vo, cudaStream_t s);
int launch_kv_gather(bool fp16, void* kc, void* vc, const int* bt, int bs, int nkv, int hd, int base, const int* src,
                     int n, void* tmp, cudaStream_t s);

}  // namespace lumina
