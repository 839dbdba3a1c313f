/* liblumina_cuda — C ABI of the B200 (sm_100a) Lumina decode path.
 *
 * The reference binds exactly one native library on this path: the TOPS
 * kernels (src/lumina_framework/kernels/tops_int8.c) through ctypes
 * (src/lumina_framework/tops.py:89-112). This header is the replacement
 * surface: plain pointers and sizes, an int status on every entry (0 = ok,
 * else a LUMINA_E_* code with text from lumina_last_error()), no C++ or
 * framework types.
 *
 * Pointer conventions: arguments suffixed _dev are device pointers that the
 * caller owns; _host arguments are host pointers; every other buffer is owned
 * by the library (weights, KV pages, activations, scratch). `stream` is a
 * cudaStream_t passed as void* (NULL = the legacy default stream).
 */
#ifndef LUMINA_CUDA_H
#define LUMINA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LUMINA_CUDA_VERSION 1

enum {
  LUMINA_OK = 0,
  LUMINA_E_ARG = 1,          /* bad argument (shape, size, pointer, range)   */
  LUMINA_E_CUDA = 2,         /* CUDA runtime error                           */
  LUMINA_E_UNSUPPORTED = 3,  /* valid input this build does not handle       */
  LUMINA_E_OOM = 4,          /* device allocation failed                     */
  LUMINA_E_STATE = 5,        /* call out of order (e.g. model not finalized) */
  LUMINA_E_NCCL = 6,         /* collective error (unused: no collective library) */
  LUMINA_E_SELFTEST = 7      /* numeric self-test mismatch                   */
};

/* Lumina code kinds = bits per code (adapters/lumina.py:135-150). */
enum { LUMINA_KIND_BINARY = 1, LUMINA_KIND_INT2 = 2, LUMINA_KIND_INT3 = 3, LUMINA_KIND_INT4 = 4 };
/* The file's "packed" flag (adapters/lumina.py:50-76, lumina_convert.py:136-147). */
enum { LUMINA_PACK_NONE = 0, LUMINA_PACK_NIBBLE = 1, LUMINA_PACK_2BIT = 2 };

/* ---- library --------------------------------------------------------- */

/* Replaces tops_version() (tops_int8.c:32), checked by tops._bind (tops.py:95-97). */
int lumina_cuda_version(void);
/* Text of the last error on this thread ("" if none). */
const char* lumina_last_error(void);
/* Number of visible CUDA devices. */
int lumina_device_count(int* n);
/* Numeric self-test on `device` (packed GEMV of every kind vs an exact
 * integer model, int8 GEMV vs the tops KAT shape). Replaces tops._self_test
 * (tops.py:152-238), which gates trust before first use. */
int lumina_selftest(int device);

/* ---- packed Lumina weights (dequant GEMV, hot path) -------------------- */

typedef struct lumina_weight lumina_weight;

/* Upload one `.lumina` tensor record exactly as stored in the file: `codes`
 * is the codes blob (nibble / 2-bit / byte-per-code / packed sign bytes as
 * the record's `packed` flag and kind say), `scales` the F32 scales blob
 * (rows x ceil(cols/group)). The codes are re-tiled on the device for the
 * GEMV and are never expanded to floating point. Replaces the per-tensor
 * unpack + dequant of LuminaAdapter.load (adapters/lumina.py:122-151).
 * For kind BINARY `cols` must be the logical width (the reference loader
 * requires it to be ceil(cols/group)*group, lumina.py:143-148).
 * Device layout: row-major packed codes; with LUMINA_INT4_LAYOUT=mma in the
 * environment int4 codes, and with LUMINA_NARROW_LAYOUT=mma int3 / int2 /
 * binary codes (one per nibble: 4 bits of device memory per code), go to
 * the tensor-core fragment layout that the tensor-pipe GEMVs read (group a
 * multiple of 64: 64, 128 or 256). A model takes narrow codes row-major
 * only. */
int lumina_weight_upload(int device, int kind, int group_size, int pack,
                         const uint8_t* codes_host, size_t codes_len,
                         const float* scales_host, size_t n_scales,
                         int rows, int cols, lumina_weight** out);
int lumina_weight_free(lumina_weight* w);
int lumina_weight_info(const lumina_weight* w, int* kind, int* group_size, int* rows,
                       int* cols, size_t* device_bytes, int* fp16_scales);

/* Bit-exact unpack gate: codes as one byte each, (rows, cols) row-major
 * (adapters/lumina.py:50-76; binary: the 0/1 sign bit, ptq_ladder.py:50-55). */
int lumina_weight_unpack(const lumina_weight* w, uint8_t* codes_dev, void* stream);
/* Bit-exact dequant gate: (float)((double)scale * linspace(-1,1,2^b)[code]),
 * (rows, cols) fp32 (adapters/lumina.py:135-150). */
int lumina_weight_dequant(const lumina_weight* w, float* out_dev, void* stream);

/* y[b, n] = sum_k x[b, k] * W[n, k] for b < batch (1..16): the fused dequant
 * GEMV that replaces `h @ W(name)` in ChatModel._layer (chat.py:239-243,282,
 * 300-303; W = dequantized Lumina weight). x rows have stride ldx floats, y
 * rows stride ldy floats. Uses the library's per-device activation scratch
 * for batches the fused kernels do not take, and for 5..16 rows over the
 * fragment layout (calls that overlap on the GPU on one device race on it). */
int lumina_gemv(const lumina_weight* w, const float* x_dev, int batch, int ldx,
                float* y_dev, int ldy, void* stream);
/* y[m, n] = sum_k x[m, k] * W[n, k] for `rows` hidden rows at once (any
 * count): the projection of a prompt prefill or a tree verification, where
 * ChatModel._layer runs h @ W with sq > 1 (chat.py:239-243). Built for int4
 * weights in the tensor-core fragment layout (LUMINA_E_UNSUPPORTED
 * otherwise): the codes are turned into the reference's fp16 weights in
 * shared memory (chat.py:140 rounds the dequantized weights to fp16), x is
 * rounded to fp16, and tcgen05 tensor cores accumulate in fp32. Uses a
 * per-device fp16 activation scratch the library grows on demand (calls that
 * overlap on the GPU on one device race on it). Asynchronous on `stream`. */
int lumina_gemm_rows(const lumina_weight* w, const float* x_dev, int rows, int ldx,
                     float* y_dev, int ldy, void* stream);
/* Same contraction with host buffers; copies in, runs, copies out, syncs. */
int lumina_gemv_host(const lumina_weight* w, const float* x_host, int batch, float* y_host);

/* lumina_gemv for callers that cannot allocate device memory (a runtime that
 * owns every allocation through its own pool, or one that must not trigger
 * the device-wide synchronisation of a cudaFree). It has no counterpart in
 * the reference. Same arguments and the same arithmetic as lumina_gemv (the
 * batched path: activation quantization, then the packed GEMV); it makes no
 * cudaMalloc or cudaFree call of any kind. Its activation scratch is a fixed
 * 1 MiB array in the library's device image (LUMINA_NOALLOC_SCRATCH_BYTES),
 * held on every GPU that loads the library until the process exits; calls
 * whose batch x padded columns need more (batch * ceil(cols/32) * 72 bytes,
 * roughly) fail with LUMINA_E_ARG. The first call on each device looks up
 * the array's device address and keeps it, so make that first call outside
 * any stream capture. All calls share the one array: two calls that overlap
 * on the GPU (different streams, no ordering between them) race on it and
 * produce wrong results. Weights in the tensor-core fragment layout are not
 * supported (LUMINA_E_UNSUPPORTED). */
int lumina_gemv_noalloc(const lumina_weight* w, const float* x_dev, int batch, int ldx,
                        float* y_dev, int ldy, void* stream);

/* Timeouts. Kernels that wait on their own asynchronous transfers or on
 * peers (the decode GEMVs, the tcgen05 multi-row projection, the
 * tensor-parallel exchange) bound every wait; one that gives up ORs a bit
 * into a per-device fault word (1: gemv_fused, 2: gemv_tc, 4: peer exchange,
 * 8: gemm_tc05) and returns, leaving its outputs unwritten. Every
 * synchronous entry (lumina_gemv_host, lumina_forward, lumina_layer_forward,
 * lumina_decode_step, lumina_decode_greedy, lumina_profile_gemv) clears the
 * word as it starts and returns LUMINA_E_CUDA ("a device wait timed out")
 * when it is set at the end. lumina_gemv, lumina_gemm_rows and
 * lumina_gemv_noalloc are asynchronous: after synchronizing their stream, the caller reads (and with
 * `clear`, resets) the word here. The tops-style reference reported no
 * errors at all (tops_int8.c: void returns); the dict convention of
 * tops.py:296-314 carries this one to Python callers. */
int lumina_fault_status(int device, int* word_host, int clear);
/* Testing aid: the polls a kernel makes on a pending transfer before it gives
 * up (default 2^24, about a second); 0 makes every such wait give up without
 * polling, so that tests can check that a timeout surfaces as an error and
 * that the next call succeeds. A negative value restores the default.
 * Applies to kernels launched after the call; a CUDA graph keeps the value
 * its capture saw. The transfers themselves always complete: a kernel whose
 * wait gave up still waits, with the default limit, for its copies in
 * flight before it exits. */
int lumina_debug_wait_limit(long long spins);

/* ---- int8 fused GEMV family (TOPS semantics, MoE-runtime path) -------- */
/* Host-pointer entries with the exact argument meaning of the TOPS C ABI
 * (caller owns every buffer, row-major (N, K) weights). */

/* out[n] = ws[n] * sum_b xs[b] * dot32(xq_b, wq[n]_b); replaces tops_gemv_int8
 * (tops_int8.c:41-66) and tops_gemv_int8_mt (:197-222) behind
 * fused.fused_gemv_int8 (fused.py:186-214). */
int lumina_gemv_int8(const int8_t* xq, const float* xs, const int8_t* wq, const float* ws,
                     float* out, int N, int K);
/* Q4_0: wq packed (N, K/2), byte j = weights 2j (low) and 2j+1 (high), value =
 * code - 8, ws (N, K/32); replaces tops_gemv_q4_0 (tops_int8.c:73-106). */
int lumina_gemv_q4_0(const int8_t* xq, const float* xs, const uint8_t* wq, const float* ws,
                     float* out, int N, int K);
/* fp16 x and W, fp32 out; replaces tops_gemv_fp16 (tops_int8.c:225-243). */
int lumina_gemv_fp16(const void* x_fp16, const void* w_fp16, float* out, int N, int K);
/* out[m, n] per row m as gemv_int8; replaces tops_gemm_int8 (tops_int8.c:300-326). */
int lumina_gemm_int8(const int8_t* xq, const float* xs, const int8_t* wq, const float* ws,
                     float* out, int M, int N, int K);

/* ---- decode model: weights + paged KV + layer / step forward ---------- */

typedef struct lumina_model lumina_model;

typedef struct {
  int n_layer, d_model, n_heads, n_kv, head_dim, ffn, vocab;
  float eps;        /* RMSNorm eps (chat.py:63-66: 1e-6)                     */
  float theta;      /* RoPE base (chat.py:119; pass explicitly)              */
  int kv_fp16;      /* 0: fp32 KV pages, 1: fp16 KV pages                    */
  int block_size;   /* KV page size in tokens (16)                           */
  int max_seq;      /* KV capacity in tokens                                 */
  int max_rows;     /* largest row count of one forward (prefill chunk)      */
  int tp_rank, tp_size;  /* tensor-parallel shard of this process (0, 1)    */
} lumina_model_config;

/* Create a model shell on `device` and register its weights. Names are the
 * HF-Llama tensor names the reference reads (chat.py:240-303). Packed
 * weights transfer ownership to the model. Raw fp32 tensors (embed, head,
 * norms — kept raw by lumina_convert.py:48-79) are rounded to fp16 exactly
 * as ChatModel.from_tensors does (chat.py:138-143). */
int lumina_model_create(int device, const lumina_model_config* cfg, lumina_model** out);
int lumina_model_set_weight(lumina_model* m, const char* name, lumina_weight* w);
int lumina_model_set_tensor(lumina_model* m, const char* name, const float* host,
                            int rows, int cols);
/* Mark `layer` as a virtual-MoE layer (replaces the per-layer entry of the
 * .lumina header's "virtual_moe" map that ChatModel reads, chat.py:157-183,
 * and its routed branch, chat.py:285-299 -> qwen_next.py:31-78 with unit
 * weights). The layer then takes, instead of gate/up/down_proj:
 *   "model.layers.L.mlp.experts.gate_up_proj"  packed int4 (experts*2*ie, d)
 *   "model.layers.L.mlp.experts.down_proj"     packed int4 (experts*ie, d)
 *   "model.layers.L.mlp.gate.weight"           raw router (experts, d)
 *   "model.layers.L.mlp.gate_bias"             raw router bias (experts), optional
 * int4 with groups of 64k, d % 64 == 0, experts <= 64, top_k <= 8. Under
 * tensor parallelism (tp_size > 1) the experts are sharded: rank r passes
 * the rows of experts [r E/tp, (r+1) E/tp) (E divisible by tp) and the full
 * router; each rank computes its experts' share of the routed MLP and the
 * shares are summed over peer memory like a row-parallel down_proj. */
int lumina_model_set_moe(lumina_model* m, int layer, int experts, int ie, int top_k);
/* Check every tensor is present, allocate KV pages and buffers, build the
 * fused projection layouts. */
int lumina_model_finalize(lumina_model* m);
int lumina_model_free(lumina_model* m);

/* Tensor parallelism (tp_size > 1 in the config): each rank's sums after
 * o_proj / down_proj and its vocab shard of the logits are exchanged over
 * peer memory (NVLink) by one kernel per exchange, with no collective
 * library. The reference has no multi-GPU path; this pair joins the ranks.
 * After lumina_model_finalize every rank calls lumina_model_peer_handle (the
 * 64-byte CUDA IPC handle of its exchange region), the handles travel to
 * every rank in rank order (tp_size x 64 bytes), and each rank calls
 * lumina_model_init_peers before its first forward. Every rank must then run
 * the same forwards in the same order; a wait for a peer is bounded (about
 * 10 s) and reports a timeout through the fault word. */
int lumina_model_peer_handle(lumina_model* m, uint8_t* handle64_host);
int lumina_model_init_peers(lumina_model* m, const uint8_t* handles_host);

/* KV contract of chat.py (cache[lyr] = (k, v), rows (T, n_heads, hd)). */
/* Rows held by `layer` (layer = -1: every layer, which must agree; layers
 * differ only while a caller runs a forward layer by layer). */
int lumina_kv_length(const lumina_model* m, int layer, int* len);
/* k[:n], v[:n] on every layer: prefix truncation (chat.py:438-447), spec
 * rollback (chat.py:636-638). Pages are kept; only the length shrinks. */
int lumina_kv_truncate(lumina_model* m, int len);
/* Copy rows [start, start+n) of layer `layer` to host as fp32
 * (n, n_heads, head_dim), GQA-expanded like chat.py:257-263. */
int lumina_kv_read(const lumina_model* m, int layer, int start, int n,
                   float* k_host, float* v_host);
/* EAGLE commit (eagle.py:340-350): rows base+src[i] -> base+i for i < n on
 * every layer, then length = base + n. */
int lumina_kv_commit_rows(lumina_model* m, int base, const int* src_host, int n);

/* Single-query attention of q (host fp32, (n_heads, head_dim) of this shard)
 * over rows [0, len) of layer `layer`: softmax(q K^T / sqrt(hd)) V per head
 * with every cached key visible and no bias — the decode row of chat.py:
 * 264-281 (sq = 1), on the kernel the decode step runs. out_host receives
 * (n_heads, head_dim) fp32. Synchronous. */
int lumina_kv_attend(lumina_model* m, int layer, const float* q_host, float* out_host);

/* One decoder layer over n rows of hidden state (device fp32, (n, d_model),
 * updated in place): the drop-in for ChatModel._layer(x, lyr, cache, pos0,
 * attn_bias, pos_override) (chat.py:232-304). Appends n KV rows at the
 * current length. pos_override_host (n ints) and bias_host ((n, len+n) fp32,
 * 0 / -inf; a positive entry admits its key whatever the key's position, as
 * for lumina_forward) may be NULL. */
int lumina_layer_forward(lumina_model* m, int layer, float* x_dev, int n, int pos0,
                         const int* pos_override_host, const float* bias_host,
                         void* stream);
/* Embed `tokens`, run every layer at positions pos0.. (appending KV) and
 * write the head logits of the last row (or of every row if all_rows) to
 * logits_host — the body of generate's prefill / decode loop (chat.py:
 * 379-402) with the head GEMV of :388 (no final norm). With
 * pos_override_host (n positions) and bias_host ((n, len+n) additive, 0 /
 * -inf) it is the tree-verification forward of eagle.verify_tree
 * (eagle.py:259-291); both may be NULL. A key is visible to a row when its
 * position (a cached key's: its row index) is not past the row's, as in
 * chat.py:264-274; a positive bias entry, which the reference never
 * passes, admits the key whatever its position (several sequences sharing
 * one cache: engine.generate_shared_prefix). */
int lumina_forward(lumina_model* m, const int* tokens_host, int n, int pos0,
                   const int* pos_override_host, const float* bias_host,
                   float* logits_host, int all_rows);
/* One greedy decode step at the current KV length as a replayed CUDA graph:
 * embed `token`, all layers, head; logits to logits_host (may be NULL),
 * argmax (first max, as np.argmax in chat.py:339) to *argmax_host. */
int lumina_decode_step(lumina_model* m, int token, float* logits_host, int* argmax_host);

/* n greedy decode steps with the argmax of each step fed to the next on
 * the device (no host round trip per token): the same per-token work as n
 * calls of lumina_decode_step with argmax sampling (chat.py:339, temperature
 * 0), generated tokens to tokens_host. The first step embeds `token`.
 * Optional outputs (may be NULL): device_ms = CUDA-event time of the n
 * steps on the model's stream; kernels_per_step = kernel launches in one
 * step's graph. */
int lumina_decode_greedy(lumina_model* m, int token, int n, int* tokens_host, float* device_ms,
                         int* kernels_per_step);

/* Measurement: replay the packed-weight GEMVs of one decode token (every
 * layer's q/k/v, o, gate/up and down in decode order, on this model's
 * weights and buffers) `iters` times as one CUDA graph, timed with CUDA
 * events on the model's stream. Returns the mean duration of one GEMV
 * launch (ms), the launches per token, and the algorithmic bytes of those
 * launches per token (packed codes + scales read, fp32 activations read,
 * fp32 outputs written). */
int lumina_profile_gemv(lumina_model* m, int iters, float* ms_per_launch, int* launches_per_token,
                        double* bytes_per_token);

/* Measurement: replay the decode row's attention (attnc_kernel) of every
 * layer at the current KV length `iters` times as one CUDA graph, timed with
 * CUDA events on the model's stream: the mean duration of one launch (ms)
 * and its algorithmic bytes (the K and V rows of every cached key of this
 * shard's heads, q in, the output out). Leaves the KV rows unchanged. */
int lumina_profile_attention(lumina_model* m, int iters, float* ms_per_launch, double* bytes_per_launch);

#ifdef __cplusplus
}
#endif

#endif /* LUMINA_CUDA_H */
