// Decode model: weight registry, paged KV, the dense decoder layer of
// chat.py:_layer (232-304) on the device, whole forwards and a graph-replayed
// greedy decode step. Optional tensor parallelism (column-parallel
// q/k/v/gate/up/head, row-parallel o/down) whose sums and logits gather run
// over peer memory (peer.cu).

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "model.cuh"

using namespace lumina;

namespace {

struct Layer {
  lumina_weight *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr;
  lumina_weight *gate = nullptr, *up = nullptr, *down = nullptr;
  lumina_weight *qkv = nullptr, *gu = nullptr;  // fused layouts built at finalize
  float *in_norm = nullptr, *post_norm = nullptr;
  // virtual-MoE MLP (moe_e > 0): flat experts + router (chat.py:285-299)
  lumina_weight *moe_gu = nullptr, *moe_down = nullptr;
  float *router_w = nullptr, *router_b = nullptr;
  int moe_e = 0, moe_ie = 0, moe_k = 0;
  int moe_e_lo = 0, moe_e_n = 0;  // this rank's experts (expert parallelism under TP)
  int router_rows = 0, router_blen = 0;  // as set, checked against moe_e at finalize
};

size_t al256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace

struct lumina_model {
  int device = 0;
  lumina_model_config c{};
  int nh = 0, nkv = 0, hd = 0, ffn = 0, vocab = 0, d = 0;  // local (this shard) sizes
  std::vector<Layer> L;
  std::vector<float> in_norm_h, post_norm_h;
  __half* embed = nullptr;
  int embed_rows = 0;
  __half* head = nullptr;
  int head_rows = 0;
  float *rope_cos = nullptr, *rope_sin = nullptr;
  std::vector<float> rope_cos_h, rope_sin_h;

  // paged KV
  void *kpool = nullptr, *vpool = nullptr;
  size_t layer_elems = 0;  // elements of one layer's K (or V) pool
  int n_blocks = 0;
  std::vector<int> bt_host;
  std::vector<int> free_blocks;
  int* bt_dev = nullptr;
  std::vector<int> layer_len;

  // activations
  float *x = nullptr, *qkv_buf = nullptr, *q_buf = nullptr, *attn = nullptr, *ffn_buf = nullptr;
  float *g_buf = nullptr, *u_buf = nullptr, *part = nullptr, *logits = nullptr;
  __half* x16 = nullptr;  // fp16 activation rows of the tcgen05 projections
  size_t x16_bytes = 0;   // (also the int16 fragments of the batched tensor-pipe GEMV)
  SplitWork split;        // partials of split-K projections and split-key attention
  ActQ aq{};
  void* kv_tmp = nullptr;
  float* bias_dev = nullptr;
  int bias_rows = 64;
  DevParams* P_dev = nullptr;
  DevParams* P_host = nullptr;  // pinned
  int *rowpos_dev = nullptr, *rowpos_host = nullptr, *tokens_dev = nullptr, *tokens_host = nullptr;
  int *argmax_dev = nullptr, *argmax_host = nullptr, *src_dev = nullptr;
  unsigned long long* amax_key_dev = nullptr;   // fused head argmax (value, index) key
  unsigned long long* amax_key_host = nullptr;  // pinned
  int* fault_host = nullptr;                     // pinned copy of the device fault word
  float* logits_host = nullptr;  // pinned
  cudaStream_t stream = nullptr;
  cudaGraphExec_t step_graph = nullptr;
  cudaGraphExec_t chain_graph = nullptr;  // greedy steps with on-device token feedback
  int* chain_tokens = nullptr;            // [max_seq] generated tokens
  int* chain_count = nullptr;
  int chain_kernels = 0;                  // kernel nodes in chain_graph
  MoeScratch moe{};                       // virtual-MoE scratch (null without MoE layers)
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  int graph_splits = 0;
  bool finalized = false;
  // tensor parallelism: this rank's exchange region [flags][slot 0..2] and
  // every rank's region as mapped here (this rank's own at [tp_rank])
  char* exch = nullptr;
  size_t exch_slot = 0;  // floats per slot
  char* peer_exch[PEER_MAX] = {};
  unsigned* peer_epoch = nullptr;  // PEER_CTAS exchange counters
  bool peers_ready = false;
  // the decode step's exchanges fused into its GEMVs (TcTp): per kind (0:
  // o_proj, 1: down_proj) every rank owns receive slots [kind][source rank]
  // of TP_PUSH_ROWS rows behind the three exchange slots and flags
  // [kind][source rank] at TP_PUSH_FLAGS in the flag page; the residual
  // alternates between xa (after the attention sum) and xb (after the MLP
  // sum) because a consumer's CTAs read one while CTA 0 writes the other
  bool tp_fusable = false;   // every layer's projections run on gemv_tc
  bool tp_fuse_now = false;  // set while the decode graphs are captured
  unsigned* tp_epoch = nullptr;  // [2] exchanges published, per kind
  int* tp_ticket = nullptr;      // [2] producer CTA tickets
  float *xa = nullptr, *xb = nullptr;
  std::vector<void*> allocs;
};

namespace {

struct Guard {
  int prev = -1;
  explicit Guard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~Guard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

int dalloc(lumina_model* m, void** p, size_t bytes) {
  if (cudaMalloc(p, std::max<size_t>(bytes, 256)) != cudaSuccess) {
    cudaGetLastError();
    set_error("model: cudaMalloc(%zu) failed", bytes);
    return LUMINA_E_OOM;
  }
  m->allocs.push_back(*p);
  return LUMINA_OK;
}

int parse_layer_name(const char* name, int* layer, std::string* what) {
  int l = -1, n = 0;
  if (sscanf(name, "model.layers.%d.%n", &l, &n) == 1 && n > 0) {
    *layer = l;
    *what = std::string(name + n);
    return 1;
  }
  return 0;
}

// fused [a; b; c] rows (same kind / group / width / scale type)
bool compatible(const lumina_weight* a, const lumina_weight* b) {
  return a && b && a->bits == b->bits && a->group == b->group && a->cols == b->cols &&
         a->fp16_scales == b->fp16_scales && a->row_bytes == b->row_bytes && a->spr == b->spr &&
         a->mma == b->mma;
}

// A new tiled weight with the geometry of `a` and `rows` rows (zeroed); with
// `to_mma` (int4, group % 64 == 0) in the tensor-core fragment layout.
lumina_weight* alloc_like(const lumina_weight* a, int rows, int* rc, bool to_mma = false) {
  lumina_weight* w = new lumina_weight(*a);
  w->rows = rows;
  w->rows_pad = (rows + ROW_PAD - 1) / ROW_PAD * ROW_PAD;
  if (to_mma && !a->mma) {
    w->mma = 1;
    w->n_chunks = (a->nblk + 1) / 2 * 2;  // 32-column blocks, whole pairs
    w->row_bytes = w->n_chunks * 16;
  }
  if (w->mma) w->rows_pad = (rows + 31) / 32 * 32;
  const size_t cb = (size_t)w->rows_pad * w->row_bytes;
  const size_t sb = w->mma ? (size_t)w->rows_pad * a->n_groups * (a->fp16_scales ? 2 : 4)
                           : (size_t)w->rows_pad * a->spr;
  w->codes = nullptr;
  w->scales = nullptr;
  if (cudaMalloc(&w->codes, cb) != cudaSuccess || cudaMalloc(&w->scales, sb) != cudaSuccess ||
      cudaMemset(w->codes, 0, cb) != cudaSuccess || cudaMemset(w->scales, 0, sb) != cudaSuccess) {
    cudaGetLastError();
    if (w->codes) cudaFree(w->codes);
    if (w->scales) cudaFree(w->scales);
    delete w;
    set_error("model: fused weight allocation failed");
    *rc = LUMINA_E_OOM;
    return nullptr;
  }
  w->bytes = cb + sb;
  *rc = LUMINA_OK;
  return w;
}

// out row r <- row srow[r] of source sel[r] (up to three sources)
lumina_weight* gather_rows(const std::vector<const lumina_weight*>& srcs, const std::vector<int>& sel,
                           const std::vector<int>& srow, int* rc, bool to_mma = false) {
  lumina_weight* w = alloc_like(srcs[0], (int)sel.size(), rc, to_mma);
  if (!w) return nullptr;
  int* d = nullptr;
  if (cudaMalloc(&d, sel.size() * 8) != cudaSuccess) {
    cudaGetLastError();
    lumina_weight_free(w);
    set_error("model: gather index allocation failed");
    *rc = LUMINA_E_OOM;
    return nullptr;
  }
  cudaMemcpy(d, sel.data(), sel.size() * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(d + sel.size(), srow.data(), sel.size() * 4, cudaMemcpyHostToDevice);
  const lumina_weight& s0 = *srcs[0];
  const lumina_weight& s1 = *srcs[std::min<size_t>(1, srcs.size() - 1)];
  const lumina_weight& s2 = *srcs[std::min<size_t>(2, srcs.size() - 1)];
  *rc = launch_gather_rows(*w, s0, s1, s2, d, d + sel.size(), nullptr);
  const cudaError_t e = cudaDeviceSynchronize();
  cudaFree(d);
  if (!*rc && e != cudaSuccess) {
    set_error("model: gather failed: %s", cudaGetErrorString(e));
    *rc = LUMINA_E_CUDA;
  }
  if (*rc) {
    lumina_weight_free(w);
    return nullptr;
  }
  return w;
}

// fused q/k/v with each head's rotation pairs (j, j + hd/2) as adjacent rows
lumina_weight* build_qkv(const lumina_weight* q, const lumina_weight* k, const lumina_weight* v, int hd, int* rc,
                         bool to_mma) {
  std::vector<int> sel, srow;
  const lumina_weight* parts[2] = {q, k};
  for (int pi = 0; pi < 2; ++pi)
    for (int h = 0; h < parts[pi]->rows / hd; ++h)
      for (int p = 0; p < hd / 2; ++p)
        for (int e = 0; e < 2; ++e) {
          sel.push_back(pi);
          srow.push_back(h * hd + p + e * (hd / 2));
        }
  for (int r = 0; r < v->rows; ++r) {
    sel.push_back(2);
    srow.push_back(r);
  }
  return gather_rows({q, k, v}, sel, srow, rc, to_mma);
}

// gate/up interleaved: row 2i = gate_i, 2i+1 = up_i (SwiGLU epilogue)
lumina_weight* build_gu(const lumina_weight* g, const lumina_weight* u, int* rc, bool to_mma) {
  std::vector<int> sel, srow;
  for (int i = 0; i < g->rows; ++i)
    for (int e = 0; e < 2; ++e) {
      sel.push_back(e);
      srow.push_back(i);
    }
  return gather_rows({g, u}, sel, srow, rc, to_mma);
}

// the same rows in the tensor-core fragment layout
lumina_weight* to_fragment_layout(const lumina_weight* a, int* rc) {
  std::vector<int> sel(a->rows, 0), srow(a->rows);
  for (int r = 0; r < a->rows; ++r) srow[r] = r;
  return gather_rows({a}, sel, srow, rc, true);
}

// int4 with groups of 64k runs on the tensor-pipe decode GEMV unless
// LUMINA_GEMV=dp2a keeps the CUDA-core layout
bool wants_tc(const lumina_weight* w) {
  const char* e = getenv("LUMINA_GEMV");
  if (e && strcmp(e, "dp2a") == 0) return false;
  return w->bits == 4 && w->group % 64 == 0;
}

// rope tables: cos/sin(float32(p) * freq_i) with freq_i =
// 1 / theta^(float32(2i) / hd) (chat.py:69-85), computed in double and rounded
// once; callers wanting numpy's float32 cos/sin bit for bit pass their own
// tables as the "rope.cos" / "rope.sin" tensors.
void default_rope(lumina_model* m) {
  const int half = m->hd / 2, npos = m->c.max_seq + 1;
  m->rope_cos_h.assign((size_t)npos * half, 0.f);
  m->rope_sin_h.assign((size_t)npos * half, 0.f);
  for (int i = 0; i < half; ++i) {
    const float e = (float)(2 * i) / (float)m->hd;
    const float freq = 1.0f / powf(m->c.theta, e);
    for (int p = 0; p < npos; ++p) {
      const float a = (float)p * freq;
      m->rope_cos_h[(size_t)p * half + i] = (float)cos((double)a);
      m->rope_sin_h[(size_t)p * half + i] = (float)sin((double)a);
    }
  }
}

int ensure_blocks(lumina_model* m, int len) {
  const int need = (len + m->c.block_size - 1) / m->c.block_size;
  if (need > m->n_blocks) {
    set_error("KV capacity exceeded: %d tokens > max_seq %d", len, m->n_blocks * m->c.block_size);
    return LUMINA_E_OOM;
  }
  bool changed = false;
  const int first = (int)m->bt_host.size();
  while ((int)m->bt_host.size() < need) {
    m->bt_host.push_back(m->free_blocks.back());
    m->free_blocks.pop_back();
    changed = true;
  }
  if (changed) {
    const cudaError_t e = cudaMemcpyAsync(m->bt_dev + first, m->bt_host.data() + first,
                                          (m->bt_host.size() - first) * sizeof(int), cudaMemcpyHostToDevice, m->stream);
    if (e != cudaSuccess) {
      set_error("block table upload: %s", cudaGetErrorString(e));
      return LUMINA_E_CUDA;
    }
    // the pageable source must stay valid until the copy ran
    cudaStreamSynchronize(m->stream);
  }
  return LUMINA_OK;
}

void release_blocks(lumina_model* m, int len) {
  const int keep = (len + m->c.block_size - 1) / m->c.block_size;
  while ((int)m->bt_host.size() > keep) {
    m->free_blocks.push_back(m->bt_host.back());
    m->bt_host.pop_back();
  }
}


size_t kv_es(const lumina_model* m) { return m->c.kv_fp16 ? 2 : 4; }

char* layer_k(lumina_model* m, int l) { return (char*)m->kpool + (size_t)l * m->layer_elems * kv_es(m); }
char* layer_v(lumina_model* m, int l) { return (char*)m->vpool + (size_t)l * m->layer_elems * kv_es(m); }

// slot `slot` of this rank's exchange region
float* exch_slot_ptr(lumina_model* m, int slot) {
  return reinterpret_cast<float*>(m->exch + PEER_FLAG_BYTES) + (size_t)slot * m->exch_slot;
}

constexpr int TP_PUSH_ROWS = 4;        // decode rows of a fused exchange (gemv_tc batch)
constexpr size_t TP_PUSH_FLAGS = 2048;  // byte offset of the push flags in the flag page
static_assert(TCTP_MAX == PEER_MAX, "one receive slot per rank");
static_assert(PEER_CTAS * PEER_MAX * 4 <= TP_PUSH_FLAGS && TP_PUSH_FLAGS + 2 * PEER_MAX * 4 <= PEER_FLAG_BYTES,
              "flag page layout");

// receive slot (kind, source rank src) in rank r's region, and its flag
float* tp_push_slot(const lumina_model* m, int r, int kind, int src) {
  float* base = reinterpret_cast<float*>(m->peer_exch[r] + PEER_FLAG_BYTES) + 3 * m->exch_slot;
  return base + ((size_t)kind * PEER_MAX + src) * TP_PUSH_ROWS * m->d;
}
unsigned* tp_push_flag(const lumina_model* m, int r, int kind, int src) {
  return reinterpret_cast<unsigned*>(m->peer_exch[r] + TP_PUSH_FLAGS) + kind * PEER_MAX + src;
}
unsigned long long tp_timeout_ns() { return wait_spin_limit() == 0 ? 0ull : 10000000000ull; }

// this rank's producing side of exchange `kind`: rows to every rank's slot
TcTp tp_producer(const lumina_model* m, int kind) {
  TcTp t;
  t.tp = m->c.tp_size;
  t.ld = m->d;
  for (int r = 0; r < t.tp; ++r) {
    t.push[r] = tp_push_slot(m, r, kind, m->c.tp_rank);
    t.flags[r] = tp_push_flag(m, r, kind, m->c.tp_rank);
  }
  t.ticket = m->tp_ticket + kind;
  t.epoch = m->tp_epoch + kind;
  t.timeout_ns = tp_timeout_ns();
  return t;
}
// the consuming side: x + every rank's rows, the sum kept in xout
TcTp tp_consumer(const lumina_model* m, int kind, float* xout) {
  TcTp t;
  t.tp = m->c.tp_size;
  t.ld = m->d;
  for (int r = 0; r < t.tp; ++r) t.add[r] = tp_push_slot(m, m->c.tp_rank, kind, r);
  t.in_flags = tp_push_flag(m, m->c.tp_rank, kind, 0);
  t.xout = xout;
  t.epoch = m->tp_epoch + kind;
  t.timeout_ns = tp_timeout_ns();
  return t;
}

// Exchange slot `slot` (n floats, written by the previous kernel) with every
// rank: PEER_SUM adds the ranks' sum into out, PEER_GATHER writes the ranks'
// slots side by side to out.
int peer_exchange(lumina_model* m, int slot, int mode, size_t n, float* out) {
  PeerArgs a{};
  const int tp = m->c.tp_size;
  for (int r = 0; r < tp; ++r) {
    a.slot[r] = reinterpret_cast<const float*>(m->peer_exch[r] + PEER_FLAG_BYTES) + (size_t)slot * m->exch_slot;
    a.flags[r] = reinterpret_cast<unsigned*>(m->peer_exch[r]);
  }
  a.epoch = m->peer_epoch;
  a.tp = tp;
  a.rank = m->c.tp_rank;
  a.n = n;
  a.out = out;
  a.fault = fault_flag_ptr();
  // peers run the same calls within moments of each other; 10 s is a hang
  // guard, not a latency figure (a wait limit of 0 gives up at once)
  a.timeout_ns = wait_spin_limit() == 0 ? 0ull : 10000000000ull;
  if (!a.fault) {
    set_error("peer exchange: fault word unavailable");
    return LUMINA_E_CUDA;
  }
  return launch_peer_exchange(a, mode, m->stream);
}

#define TRY(expr)            \
  do {                       \
    int _rc = (expr);        \
    if (_rc) return _rc;     \
  } while (0)

// y = W x (+ epilogue): the fused decode GEMV for 1, 2 or 4 rows, else (or
// when the shape does not fit it) act_quant + the global-activation GEMV.
// rows from which a projection runs as a tcgen05 GEMM instead of the
// batched tensor-pipe GEMV
constexpr int TC05_MIN_ROWS = 8;
// rows up to which a projection runs on the batched tensor-pipe GEMV
// (gemv_tcb.cu) before the tcgen05 GEMM
constexpr int TCB_MAX_ROWS = 32;

// `exact_rows`: keep several-row projections on the int16-activation path
// (about 5e-5 relative) instead of the fp16-activation tcgen05 GEMM (about
// 3e-4): the projections that feed a virtual-MoE router, whose top-k choice
// flips at score gaps of 1e-4 .. 1e-3.
int gemv_any(lumina_model* m, const lumina_weight* w, const float* x, int ldx, int n, const float* norm, float* y,
             int ldy, int epi, const float* resid, int ldr, const RopeKV* rk, const L2Prefetch* pf = nullptr,
             bool exact_rows = false, const TcTp* tpx = nullptr) {
  if (tpx) {
    // a fused exchange has no other kernel to fall back to
    const int rc = w->mma && n <= 4
                       ? gemv_tc_launch(w, x, ldx, n, norm, m->c.eps, y, ldy, epi, resid, ldr, m->stream, rk, pf, tpx)
                       : LUMINA_E_UNSUPPORTED;
    if (rc == LUMINA_E_UNSUPPORTED) set_error("fused exchange: projection not on the tensor-pipe GEMV");
    return rc;
  }
  if (w->mma) {
    if (n <= 4) {
      const int rc = gemv_tc_launch(w, x, ldx, n, norm, m->c.eps, y, ldy, epi, resid, ldr, m->stream, rk, pf);
      if (rc != LUMINA_E_UNSUPPORTED) return rc;
    }
    if (n <= TCB_MAX_ROWS && m->x16) {
      // 5..32 rows (decode batches, tree verification): the batched
      // tensor-pipe GEMV, int16 activations like the decode GEMV, RoPE + KV
      // append fused into its epilogue for the q/k/v rows
      const int rc = gemv_tcb_launch(w, x, ldx, n, norm, m->c.eps, m->x16, m->x16_bytes, y, ldy, epi, resid, ldr, 0, 0,
                                     m->stream, rk);
      if (rc != LUMINA_E_UNSUPPORTED) return rc;
    }
    if (n >= TC05_MIN_ROWS && m->x16 && !exact_rows) {
      // several rows (prefill, tree verification): tcgen05 GEMM; the fused
      // q/k/v rows go to qkv_buf in their original order for the RoPE + KV
      // append kernel
      const bool qkv = epi == EPI_ROPE_KV;
      const int g5 = epi == EPI_RESID ? G5_RESID : epi == EPI_SWIGLU ? G5_SWIGLU : G5_STORE;
      const int width = rk ? (rk->nh + 2 * rk->nkv) * rk->hd : 0;
      int rc = gemm_tc05_launch(w, x, ldx, n, norm, m->c.eps, m->x16, qkv ? m->qkv_buf : y, qkv ? width : ldy, g5,
                                resid, ldr, qkv ? (rk->nh + rk->nkv) * rk->hd : 0, rk ? rk->hd : 0, m->stream,
                                &m->split);
      if (rc == LUMINA_OK && qkv)
        rc = launch_rope_append(rk->kv_fp16, m->qkv_buf, rk->nh, rk->nkv, rk->hd, rk->cos_t, rk->sin_t, rk->row_pos,
                                m->P_dev, rk->block_table, rk->bs, rk->kcache, rk->vcache, rk->q_out, n, m->stream);
      if (rc != LUMINA_E_UNSUPPORTED) return rc;
    }
    const int rc = gemv_mma_launch(w, x, ldx, n, norm, m->c.eps, y, ldy, epi, resid, ldr, m->stream, rk);
    if (rc != LUMINA_E_UNSUPPORTED) return rc;
  }
  if (n == 1 || n == 2 || n == 4) {
    const int rc = gemv_fused_launch(w, x, ldx, n, norm, m->c.eps, y, ldy, epi, resid, ldr, m->stream, rk);
    if (rc != LUMINA_E_UNSUPPORTED) return rc;
  }
  TRY(act_quant(x, ldx, n, w->cols, norm, m->c.eps, w->bits, m->aq, m->stream));
  return gemv_launch(w, m->aq, n, y, ldy, epi, resid, ldr, m->stream, rk);
}

// the first bytes of the LM head (the kernel after the last layer)
L2Prefetch head_prefetch(const lumina_model* m) {
  L2Prefetch pf;
  pf.p[0] = m->head;
  pf.n[0] = std::min<size_t>((size_t)m->head_rows * m->d * 2, (size_t)48 << 20) & ~size_t(15);
  return pf;
}

// the packed weight the first GEMV of layer l streams
const lumina_weight* qkv_weight(const lumina_model* m, int l) {
  const Layer& Ly = m->L[l];
  return Ly.qkv ? Ly.qkv : Ly.q;
}

// One decoder layer over n rows of m->x (device params already uploaded).
// Each kernel of the layer pulls its successor's HBM bytes into L2 while it
// runs (L2Prefetch): q/k/v the layer's cached KV rows, attention o_proj,
// o_proj the MLP's gate/up, gate/up the down projection, down the next
// layer's q/k/v (after the last layer, the first bytes of the head).
int run_layer(lumina_model* m, int l, int n, const float* bias) {
  Layer& Ly = m->L[l];
  const int d = m->d, nh = m->nh, nkv = m->nkv, hd = m->hd;
  const int qw = nh * hd, kw = nkv * hd, width = qw + 2 * kw;
  cudaStream_t s = m->stream;
  const bool tp = m->c.tp_size > 1;
  // decode rows with the exchanges fused into the GEMVs: the layer's input
  // residual is x (layer 0) or xa plus every rank's down_proj rows of the
  // layer before, and the attention sum builds on that in xb
  const bool fused = tp && m->tp_fuse_now && n <= TP_PUSH_ROWS;
  const bool last = l + 1 == m->c.n_layer;
  const float* x_in = fused && l > 0 ? m->xa : m->x;  // the residual before this layer's sums
  const float* x_mid = fused ? (l > 0 ? m->xb : m->x) : m->x;  // the residual gate/up adds the o_proj sum to
  TcTp tp_qkv, tp_o, tp_gu, tp_down;
  if (fused) {
    if (l > 0) tp_qkv = tp_consumer(m, 1, m->xb);
    tp_o = tp_producer(m, 0);
    tp_gu = tp_consumer(m, 0, m->xa);
    if (!last) tp_down = tp_producer(m, 1);
  }
  L2Prefetch pf_kv;
  const unsigned kv_block_bytes = (unsigned)((size_t)nkv * m->c.block_size * hd * kv_es(m));
  if (kv_block_bytes % 16 == 0) {
    pf_kv.kc = layer_k(m, l);
    pf_kv.vc = layer_v(m, l);
    pf_kv.bt = m->bt_dev;
    pf_kv.len = &m->P_dev->t_prev;
    pf_kv.bs = m->c.block_size;
    pf_kv.block_bytes = kv_block_bytes;
  }
  const L2Prefetch pf_o = prefetch_of(Ly.o);
  const L2Prefetch pf_mlp = Ly.moe_e ? L2Prefetch{} : prefetch_of(Ly.gu ? Ly.gu : Ly.gate);
  const L2Prefetch pf_down = Ly.moe_e ? L2Prefetch{} : prefetch_of(Ly.down);
  const L2Prefetch pf_next = l + 1 < m->c.n_layer ? prefetch_of(qkv_weight(m, l + 1)) : head_prefetch(m);
  // 1) h = rmsnorm(x) -> q, k, v; RoPE; K/V appended (chat.py:240-263)
  if (Ly.qkv) {
    RopeKV rk{};
    rk.nh = nh;
    rk.nkv = nkv;
    rk.hd = hd;
    rk.cos_t = m->rope_cos;
    rk.sin_t = m->rope_sin;
    rk.row_pos = m->rowpos_dev;
    rk.t_prev = &m->P_dev->t_prev;
    rk.block_table = m->bt_dev;
    rk.bs = m->c.block_size;
    rk.kcache = layer_k(m, l);
    rk.vcache = layer_v(m, l);
    rk.kv_fp16 = m->c.kv_fp16;
    rk.q_out = m->q_buf;
    rk.row_base = 0;
    TRY(gemv_any(m, Ly.qkv, x_in, d, n, Ly.in_norm, nullptr, 0, EPI_ROPE_KV, nullptr, 0, &rk, &pf_kv,
                 Ly.moe_e > 0, fused && l > 0 ? &tp_qkv : nullptr));
  } else {
    if (fused) {
      set_error("fused exchange: the layer has separate q/k/v projections");
      return LUMINA_E_STATE;
    }
    lumina_weight* ws[3] = {Ly.q, Ly.k, Ly.v};
    const int off[3] = {0, qw, qw + kw};
    for (int i = 0; i < 3; ++i)
      TRY(gemv_any(m, ws[i], m->x, d, n, Ly.in_norm, m->qkv_buf + off[i], width, EPI_STORE, nullptr, 0, nullptr));
    TRY(launch_rope_append(m->c.kv_fp16, m->qkv_buf, nh, nkv, hd, m->rope_cos, m->rope_sin, m->rowpos_dev, m->P_dev,
                           m->bt_dev, m->c.block_size, layer_k(m, l), layer_v(m, l), m->q_buf, n, s));
  }
  // 2) attention (chat.py:264-281)
  if (n == 1 && !bias) {
    TRY(launch_attention_cluster(m->c.kv_fp16, hd, m->q_buf, nh, nkv, layer_k(m, l), layer_v(m, l), m->bt_dev,
                                 m->c.block_size, m->P_dev, m->attn, s, &pf_o));
  } else {
    TRY(launch_attention_rows(m->c.kv_fp16, hd, m->q_buf, nh, nkv, layer_k(m, l), layer_v(m, l), m->bt_dev,
                              m->c.block_size, m->rowpos_dev, bias, m->P_dev, m->attn, n, m->P_host->t_tot,
                              &m->split, s));
  }
  // 3) o_proj + residual (chat.py:282-283)
  if (fused) {
    TRY(gemv_any(m, Ly.o, m->attn, qw, n, nullptr, exch_slot_ptr(m, 0), d, EPI_STORE, nullptr, 0, nullptr, &pf_mlp,
                 false, &tp_o));
  } else if (tp) {
    TRY(gemv_any(m, Ly.o, m->attn, qw, n, nullptr, exch_slot_ptr(m, 0), d, EPI_STORE, nullptr, 0, nullptr, &pf_mlp));
    TRY(peer_exchange(m, 0, PEER_SUM, (size_t)n * d, m->x));
  } else {
    TRY(gemv_any(m, Ly.o, m->attn, qw, n, nullptr, m->x, d, EPI_RESID, m->x, d, nullptr, &pf_mlp, Ly.moe_e > 0));
  }
  // 4) rmsnorm -> virtual-MoE MLP (chat.py:284-299), residual in place
  if (Ly.moe_e) {
    MoeLayerArgs ma{Ly.moe_gu, Ly.moe_down, Ly.router_w, Ly.router_b, Ly.post_norm, m->c.eps,
                    Ly.moe_e, Ly.moe_ie, Ly.moe_k, d};
    ma.e_lo = Ly.moe_e_lo;
    ma.e_n = Ly.moe_e_n;
    if (!tp) return launch_moe(ma, n, m->moe, m->x, s);
    // expert parallelism: this rank's experts' share of the MLP, then the
    // ranks' shares summed into the residual like a row-parallel down_proj
    ma.out = exch_slot_ptr(m, 1);
    TRY(launch_moe(ma, n, m->moe, m->x, s));
    return peer_exchange(m, 1, PEER_SUM, (size_t)n * d, m->x);
  }
  // 4) rmsnorm -> SwiGLU MLP (chat.py:284, 300-304)
  if (Ly.gu) {
    TRY(gemv_any(m, Ly.gu, x_mid, d, n, Ly.post_norm, m->ffn_buf, m->ffn, EPI_SWIGLU, nullptr, 0, nullptr,
                 &pf_down, false, fused ? &tp_gu : nullptr));
  } else {
    if (fused) {
      set_error("fused exchange: the layer has separate gate/up projections");
      return LUMINA_E_STATE;
    }
    TRY(gemv_any(m, Ly.gate, m->x, d, n, Ly.post_norm, m->g_buf, m->ffn, EPI_STORE, nullptr, 0, nullptr));
    TRY(gemv_any(m, Ly.up, m->x, d, n, Ly.post_norm, m->u_buf, m->ffn, EPI_STORE, nullptr, 0, nullptr));
    TRY(launch_swiglu(m->g_buf, m->u_buf, m->ffn_buf, n, m->ffn, m->ffn, s));
  }
  if (fused && !last) {
    TRY(gemv_any(m, Ly.down, m->ffn_buf, m->ffn, n, nullptr, exch_slot_ptr(m, 1), d, EPI_STORE, nullptr, 0, nullptr,
                 &pf_next, false, &tp_down));
  } else if (tp) {
    // (a fused step's last layer: the exchange kernel adds the sum into xa,
    // which the head reads)
    TRY(gemv_any(m, Ly.down, m->ffn_buf, m->ffn, n, nullptr, exch_slot_ptr(m, 1), d, EPI_STORE, nullptr, 0, nullptr,
                 &pf_next));
    TRY(peer_exchange(m, 1, PEER_SUM, (size_t)n * d, fused ? m->xa : m->x));
  } else {
    TRY(gemv_any(m, Ly.down, m->ffn_buf, m->ffn, n, nullptr, m->x, d, EPI_RESID, m->x, d, nullptr, &pf_next));
  }
  return LUMINA_OK;
}

// head logits of `rows` rows starting at x row `first` (chat.py:388: no final
// norm). Vocab-parallel under TP: each rank computes its slice, then the peer
// gather assembles [rank0 | rank1 | ...].
int run_head(lumina_model* m, int first, int rows, unsigned long long* amax = nullptr) {
  const int V = m->head_rows;
  // a fused decode step leaves its residual in xa
  const float* xin = m->c.tp_size > 1 && m->tp_fuse_now && rows <= TP_PUSH_ROWS ? m->xa : m->x;
  // the next token's first GEMV (layer 0 q/k/v) into L2 meanwhile
  const L2Prefetch pf = prefetch_of(qkv_weight(m, 0));
  if (m->c.tp_size <= 1) {
    if (rows >= TC05_MIN_ROWS && m->x16 && !amax) {
      // several rows (tree verification, all-row logits): the fp16 head on
      // the tensor pipe, read once for all rows
      const int rc = dense_tc05_launch(m->head, V, m->d, m->x + (size_t)first * m->d, m->d, rows, m->x16, m->logits,
                                       V, m->stream, &m->split);
      if (rc != LUMINA_E_UNSUPPORTED) return rc;
    }
    return launch_dense_gemv(m->head, V, m->d, m->x + (size_t)first * m->d, m->d, rows, m->logits, V, nullptr, 0,
                             m->stream, amax, &pf);
  }
  const int tp = m->c.tp_size;
  for (int r = 0; r < rows; ++r) {
    TRY(launch_dense_gemv(m->head, V, m->d, xin + (size_t)(first + r) * m->d, m->d, 1, exch_slot_ptr(m, 2), V,
                          nullptr, 0, m->stream, nullptr, r == 0 ? &pf : nullptr));
    TRY(peer_exchange(m, 2, PEER_GATHER, (size_t)V, m->logits + (size_t)r * V * tp));
  }
  return LUMINA_OK;
}

int upload_params(lumina_model* m, int n, int t_prev, const int* positions, const int* tokens, int bias_ld) {
  DevParams& P = *m->P_host;
  P.n = n;
  P.t_prev = t_prev;
  P.t_tot = t_prev + n;
  P.n_splits = 1;
  P.bias_ld = bias_ld;
  for (int i = 0; i < n; ++i) m->rowpos_host[i] = positions[i];
  if (tokens)
    for (int i = 0; i < n; ++i) m->tokens_host[i] = tokens[i];
  cudaStream_t s = m->stream;
  LUMINA_CUDA_TRY(cudaMemcpyAsync(m->P_dev, m->P_host, sizeof(DevParams), cudaMemcpyHostToDevice, s));
  LUMINA_CUDA_TRY(cudaMemcpyAsync(m->rowpos_dev, m->rowpos_host, n * sizeof(int), cudaMemcpyHostToDevice, s));
  if (tokens) LUMINA_CUDA_TRY(cudaMemcpyAsync(m->tokens_dev, m->tokens_host, n * sizeof(int), cudaMemcpyHostToDevice, s));
  return LUMINA_OK;
}

int check_ready(const lumina_model* m) {
  if (!m) {
    set_error("null model");
    return LUMINA_E_ARG;
  }
  if (!m->finalized) {
    set_error("model not finalized");
    return LUMINA_E_STATE;
  }
  return LUMINA_OK;
}

// a forward of a tensor-parallel shard needs its peers
int check_peers(const lumina_model* m) {
  if (m->c.tp_size > 1 && !m->peers_ready) {
    set_error("tensor-parallel model: lumina_model_init_peers has not run");
    return LUMINA_E_STATE;
  }
  return LUMINA_OK;
}

int uniform_len(const lumina_model* m, int* len) {
  const int v = m->layer_len.empty() ? 0 : m->layer_len[0];
  for (int x : m->layer_len)
    if (x != v) {
      set_error("KV layers have different lengths (a layer-by-layer forward is in progress)");
      return LUMINA_E_STATE;
    }
  *len = v;
  return LUMINA_OK;
}

// End of a synchronous entry: the fault word joins the copies on the model
// stream, the stream is drained, and a set word (a bounded wait in a GEMV
// gave up during this call) becomes the call's error and is cleared.
int finish_checked(lumina_model* m, const char* what) {
  LUMINA_CUDA_TRY(cudaMemcpyAsync(m->fault_host, fault_flag_ptr(), sizeof(int), cudaMemcpyDeviceToHost, m->stream));
  LUMINA_CUDA_TRY(cudaStreamSynchronize(m->stream));
  if (*m->fault_host) {
    const int word = *m->fault_host;
    *m->fault_host = 0;
    cudaMemset(fault_flag_ptr(), 0, sizeof(int));
    return fault_error(what, word);
  }
  return LUMINA_OK;
}

// Whole forward of n tokens at positions pos0.. (chunked by max_rows); head
// logits of the last row or every row go to m->logits.
int forward_rows(lumina_model* m, const int* tokens, int n, int pos0, const int* pos_override, const float* bias,
                 int all_rows, float* logits_host) {
  int len = 0;
  TRY(uniform_len(m, &len));
  if (bias && n > m->bias_rows) {
    set_error("forward: a bias matrix needs n <= %d rows (got %d)", m->bias_rows, n);
    return LUMINA_E_ARG;
  }
  if (bias && n > m->c.max_rows) {
    set_error("forward: a bias matrix needs one chunk (n <= max_rows %d)", m->c.max_rows);
    return LUMINA_E_ARG;
  }
  for (int t : std::vector<int>(tokens, tokens + n))
    if (t < 0 || t >= m->embed_rows) {
      set_error("token id %d out of range [0, %d)", t, m->embed_rows);
      return LUMINA_E_ARG;
    }
  const int V = m->head_rows * std::max(1, m->c.tp_size);
  std::vector<int> pos(m->c.max_rows);
  TRY(clear_fault_async(m->stream));
  for (int c0 = 0; c0 < n; c0 += m->c.max_rows) {
    const int cn = std::min(m->c.max_rows, n - c0);
    TRY(ensure_blocks(m, len + cn));
    for (int i = 0; i < cn; ++i) pos[i] = pos_override ? pos_override[c0 + i] : pos0 + c0 + i;
    for (int i = 0; i < cn; ++i)
      LUMINA_CHECK_ARG(pos[i] >= 0 && pos[i] <= m->c.max_seq, "forward: position %d beyond the RoPE table", pos[i]);
    TRY(upload_params(m, cn, len, pos.data(), tokens + c0, bias ? len + cn : 0));
    if (bias)
      LUMINA_CUDA_TRY(cudaMemcpyAsync(m->bias_dev, bias, (size_t)cn * (len + cn) * 4, cudaMemcpyHostToDevice,
                                      m->stream));
    TRY(launch_embed(m->embed, m->d, m->embed_rows, m->tokens_dev, m->P_dev, m->x, cn, nullptr, m->stream));
    for (int l = 0; l < m->c.n_layer; ++l) TRY(run_layer(m, l, cn, bias ? m->bias_dev : nullptr));
    len += cn;
    for (auto& v : m->layer_len) v = len;
    if (logits_host && (all_rows || c0 + cn == n)) {
      const int first = all_rows ? 0 : cn - 1, rows = all_rows ? cn : 1;
      for (int r0 = 0; r0 < rows; r0 += m->c.max_rows) {
        TRY(run_head(m, first + r0, std::min(rows - r0, m->c.max_rows)));
        const int rr = std::min(rows - r0, m->c.max_rows);
        float* dst = logits_host + (size_t)((all_rows ? c0 : 0) + r0) * V;
        LUMINA_CUDA_TRY(cudaMemcpyAsync(dst, m->logits, (size_t)rr * V * 4, cudaMemcpyDeviceToHost, m->stream));
      }
    }
  }
  return finish_checked(m, "forward");
}

// while a decode graph is captured, its tensor-parallel exchanges are fused
// into the GEMVs (when every projection allows it)
struct FuseExchanges {
  lumina_model* m;
  explicit FuseExchanges(lumina_model* mm) : m(mm) { m->tp_fuse_now = m->c.tp_size > 1 && m->tp_fusable; }
  ~FuseExchanges() { m->tp_fuse_now = false; }
};

int capture_step(lumina_model* m) {
  cudaStream_t s = m->stream;
  cudaGraph_t g = nullptr;
  FuseExchanges fuse(m);
  LUMINA_CUDA_TRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  int rc = LUMINA_OK;
  const int V = m->head_rows * std::max(1, m->c.tp_size);
  do {
    if (clear_fault_async(s) != LUMINA_OK ||
        cudaMemcpyAsync(m->P_dev, m->P_host, sizeof(DevParams), cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(m->rowpos_dev, m->rowpos_host, sizeof(int), cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(m->tokens_dev, m->tokens_host, sizeof(int), cudaMemcpyHostToDevice, s) != cudaSuccess) {
      set_error("capture: param copy");
      rc = LUMINA_E_CUDA;
      break;
    }
    const bool fused_argmax = m->c.tp_size <= 1;
    if ((rc = launch_embed(m->embed, m->d, m->embed_rows, m->tokens_dev, m->P_dev, m->x, 1,
                           fused_argmax ? m->amax_key_dev : nullptr, s)))
      break;
    for (int l = 0; l < m->c.n_layer && !rc; ++l) rc = run_layer(m, l, 1, nullptr);
    if (rc) break;
    if ((rc = run_head(m, 0, 1, fused_argmax ? m->amax_key_dev : nullptr))) break;
    if (!fused_argmax && (rc = launch_argmax(m->logits, V, m->argmax_dev, s))) break;
    if (cudaMemcpyAsync(m->logits_host, m->logits, (size_t)V * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyAsync(m->argmax_host, m->argmax_dev, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyAsync(m->amax_key_host, m->amax_key_dev, 8, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyAsync(m->fault_host, fault_flag_ptr(), sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess) {
      set_error("capture: result copy");
      rc = LUMINA_E_CUDA;
    }
  } while (0);
  const cudaError_t e = cudaStreamEndCapture(s, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) {
    set_error("capture: %s", cudaGetErrorString(e));
    return LUMINA_E_CUDA;
  }
  const cudaError_t ei = cudaGraphInstantiate(&m->step_graph, g, 0);
  cudaGraphDestroy(g);
  if (ei != cudaSuccess) {
    set_error("graph instantiate: %s", cudaGetErrorString(ei));
    m->step_graph = nullptr;
    return LUMINA_E_CUDA;
  }
  return LUMINA_OK;
}

// End of a chained greedy step: the argmax becomes the next step's token
// and every per-step value advances by one row.
__global__ void greedy_commit_kernel(const unsigned long long* key, const int* argmax, int* tokens, DevParams* P,
                                     int* rowpos, int* out, int* count) {
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const int tok = key ? (int)(0xFFFFFFFFu - (unsigned)(*key & 0xFFFFFFFFull)) : *argmax;
  tokens[0] = tok;
  out[*count] = tok;
  *count += 1;
  P->t_prev += 1;
  P->t_tot += 1;
  rowpos[0] += 1;
}

int capture_chain(lumina_model* m) {
  cudaStream_t s = m->stream;
  cudaGraph_t g = nullptr;
  FuseExchanges fuse(m);
  LUMINA_CUDA_TRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  int rc = LUMINA_OK;
  const int V = m->head_rows * std::max(1, m->c.tp_size);
  const bool fused_argmax = m->c.tp_size <= 1;
  do {
    if ((rc = launch_embed(m->embed, m->d, m->embed_rows, m->tokens_dev, m->P_dev, m->x, 1,
                           fused_argmax ? m->amax_key_dev : nullptr, s)))
      break;
    for (int l = 0; l < m->c.n_layer && !rc; ++l) rc = run_layer(m, l, 1, nullptr);
    if (rc) break;
    if ((rc = run_head(m, 0, 1, fused_argmax ? m->amax_key_dev : nullptr))) break;
    if (!fused_argmax && (rc = launch_argmax(m->logits, V, m->argmax_dev, s))) break;
    const cudaError_t e =
        launch_pdl(greedy_commit_kernel, dim3(1), dim3(32), 0, s, (const unsigned long long*)(fused_argmax ? m->amax_key_dev : nullptr),
                   (const int*)m->argmax_dev, m->tokens_dev, m->P_dev, m->rowpos_dev, m->chain_tokens, m->chain_count);
    if (e != cudaSuccess) {
      set_error("capture: commit launch: %s", cudaGetErrorString(e));
      rc = LUMINA_E_CUDA;
    }
  } while (0);
  const cudaError_t e = cudaStreamEndCapture(s, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) {
    set_error("capture: %s", cudaGetErrorString(e));
    return LUMINA_E_CUDA;
  }
  size_t n_nodes = 0;
  cudaGraphGetNodes(g, nullptr, &n_nodes);
  std::vector<cudaGraphNode_t> nodes(n_nodes);
  if (n_nodes) cudaGraphGetNodes(g, nodes.data(), &n_nodes);
  m->chain_kernels = 0;
  for (auto nd : nodes) {
    cudaGraphNodeType t;
    if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++m->chain_kernels;
  }
  const cudaError_t ei = cudaGraphInstantiate(&m->chain_graph, g, 0);
  cudaGraphDestroy(g);
  if (ei != cudaSuccess) {
    set_error("graph instantiate: %s", cudaGetErrorString(ei));
    m->chain_graph = nullptr;
    return LUMINA_E_CUDA;
  }
  return LUMINA_OK;
}

size_t packed_bytes(const lumina_weight* w) {
  return (size_t)w->rows * (((size_t)w->cols * w->bits + 7) / 8) +
         (size_t)w->rows * w->n_groups * (w->fp16_scales ? 2 : 4);
}

}  // namespace

extern "C" {

int lumina_model_create(int device, const lumina_model_config* cfg, lumina_model** out) {
  LUMINA_CHECK_ARG(cfg && out, "model_create: null pointer");
  *out = nullptr;
  const lumina_model_config& c = *cfg;
  LUMINA_CHECK_ARG(c.n_layer > 0 && c.d_model > 0 && c.n_heads > 0 && c.n_kv > 0 && c.head_dim > 0 && c.ffn > 0 &&
                       c.vocab > 0,
                   "model_create: non-positive dimension");
  LUMINA_CHECK_ARG(c.n_heads % c.n_kv == 0, "model_create: n_heads %d not a multiple of n_kv %d", c.n_heads, c.n_kv);
  LUMINA_CHECK_ARG(c.head_dim % 2 == 0, "model_create: odd head_dim %d", c.head_dim);
  LUMINA_CHECK_ARG(c.block_size > 0 && c.max_seq > 0 && c.max_rows > 0, "model_create: bad KV / row capacity");
  const int tp = std::max(1, c.tp_size);
  LUMINA_CHECK_ARG(c.tp_rank >= 0 && c.tp_rank < tp, "model_create: tp_rank %d of %d", c.tp_rank, tp);
  LUMINA_CHECK_ARG(c.n_kv % tp == 0 && c.n_heads % tp == 0, "model_create: heads not divisible by tp %d", tp);
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
    cudaGetLastError();
    set_error("model_create: device %d not available", device);
    return LUMINA_E_ARG;
  }
  lumina_model* m = new lumina_model();
  m->device = device;
  m->c = c;
  m->c.tp_size = tp;
  m->nh = c.n_heads / tp;
  m->nkv = c.n_kv / tp;
  m->hd = c.head_dim;
  m->d = c.d_model;
  m->ffn = 0;  // from the shard shapes
  m->L.resize(c.n_layer);
  m->layer_len.assign(c.n_layer, 0);
  *out = m;
  return LUMINA_OK;
}

int lumina_model_set_weight(lumina_model* m, const char* name, lumina_weight* w) {
  LUMINA_CHECK_ARG(m && name && w, "model_set_weight: null pointer");
  LUMINA_CHECK_ARG(!m->finalized, "model_set_weight: model already finalized");
  LUMINA_CHECK_ARG(w->device == m->device, "model_set_weight: weight on device %d, model on %d", w->device, m->device);
  LUMINA_CHECK_ARG(!w->mma || w->bits == 4,
                   "model_set_weight: int%d codes in the fragment layout serve lumina_gemv only; a model takes them "
                   "row-major", w->bits);
  int l = -1;
  std::string what;
  if (!parse_layer_name(name, &l, &what) || l < 0 || l >= m->c.n_layer) {
    set_error("model_set_weight: %s is not a layer projection", name);
    return LUMINA_E_ARG;
  }
  Layer& Ly = m->L[l];
  lumina_weight** slot = nullptr;
  if (what == "self_attn.q_proj.weight") slot = &Ly.q;
  else if (what == "self_attn.k_proj.weight") slot = &Ly.k;
  else if (what == "self_attn.v_proj.weight") slot = &Ly.v;
  else if (what == "self_attn.o_proj.weight") slot = &Ly.o;
  else if (what == "mlp.gate_proj.weight") slot = &Ly.gate;
  else if (what == "mlp.up_proj.weight") slot = &Ly.up;
  else if (what == "mlp.down_proj.weight") slot = &Ly.down;
  else if (what == "mlp.experts.gate_up_proj") slot = &Ly.moe_gu;
  else if (what == "mlp.experts.down_proj") slot = &Ly.moe_down;
  if (!slot) {
    set_error("model_set_weight: unknown projection %s", name);
    return LUMINA_E_UNSUPPORTED;
  }
  if (*slot) lumina_weight_free(*slot);
  *slot = w;
  return LUMINA_OK;
}

int lumina_model_set_moe(lumina_model* m, int layer, int experts, int ie, int top_k) {
  LUMINA_CHECK_ARG(m, "model_set_moe: null model");
  LUMINA_CHECK_ARG(!m->finalized, "model_set_moe: model already finalized");
  LUMINA_CHECK_ARG(layer >= 0 && layer < m->c.n_layer, "model_set_moe: layer %d outside 0..%d", layer,
                   m->c.n_layer - 1);
  LUMINA_CHECK_ARG(experts >= 1 && experts <= MOE_MAX_E && ie >= 1 && top_k >= 1 && top_k <= experts &&
                       top_k <= MOE_MAX_K,
                   "model_set_moe: experts %d / ie %d / top_k %d outside 1..%d / >= 1 / 1..min(experts, %d)",
                   experts, ie, top_k, MOE_MAX_E, MOE_MAX_K);
  // under tensor parallelism the experts are sharded: rank r holds the
  // contiguous experts [r E / tp, (r + 1) E / tp)
  const int tp = std::max(1, m->c.tp_size);
  LUMINA_CHECK_ARG(experts % tp == 0, "model_set_moe: %d experts do not split over %d ranks", experts, tp);
  Layer& Ly = m->L[layer];
  Ly.moe_e = experts;
  Ly.moe_ie = ie;
  Ly.moe_k = top_k;
  Ly.moe_e_n = experts / tp;
  Ly.moe_e_lo = m->c.tp_rank * Ly.moe_e_n;
  return LUMINA_OK;
}

int lumina_model_set_tensor(lumina_model* m, const char* name, const float* host, int rows, int cols) {
  LUMINA_CHECK_ARG(m && name && host && rows > 0 && cols > 0, "model_set_tensor: bad arguments");
  LUMINA_CHECK_ARG(!m->finalized, "model_set_tensor: model already finalized");
  Guard g(m->device);
  const std::string n(name);
  const size_t cnt = (size_t)rows * cols;
  if (n == "model.embed_tokens.weight" || n == "lm_head.weight") {
    LUMINA_CHECK_ARG(cols == m->d, "%s: %d columns, d_model %d", name, cols, m->d);
    std::vector<__half> h(cnt);
    for (size_t i = 0; i < cnt; ++i) h[i] = __float2half_rn(host[i]);  // chat.py:140
    void* p = nullptr;
    TRY(dalloc(m, &p, cnt * 2));
    LUMINA_CUDA_TRY(cudaMemcpy(p, h.data(), cnt * 2, cudaMemcpyHostToDevice));
    if (n[0] == 'm') {
      m->embed = (__half*)p;
      m->embed_rows = rows;
    } else {
      m->head = (__half*)p;
      m->head_rows = rows;
    }
    return LUMINA_OK;
  }
  if (n == "rope.cos" || n == "rope.sin") {
    LUMINA_CHECK_ARG(cols == m->hd / 2 && rows >= m->c.max_seq + 1, "%s: want (>= %d, %d)", name, m->c.max_seq + 1,
                     m->hd / 2);
    auto& v = n == "rope.cos" ? m->rope_cos_h : m->rope_sin_h;
    v.assign(host, host + (size_t)(m->c.max_seq + 1) * cols);
    return LUMINA_OK;
  }
  int l = -1;
  std::string what;
  if (parse_layer_name(name, &l, &what) && l >= 0 && l < m->c.n_layer &&
      (what == "input_layernorm.weight" || what == "post_attention_layernorm.weight")) {
    LUMINA_CHECK_ARG(cnt == (size_t)m->d, "%s: %zu values, d_model %d", name, cnt, m->d);
    std::vector<float> f(cnt);
    for (size_t i = 0; i < cnt; ++i) f[i] = __half2float(__float2half_rn(host[i]));  // fp16 model copy
    void* p = nullptr;
    TRY(dalloc(m, &p, cnt * 4));
    LUMINA_CUDA_TRY(cudaMemcpy(p, f.data(), cnt * 4, cudaMemcpyHostToDevice));
    (what[0] == 'i' ? m->L[l].in_norm : m->L[l].post_norm) = (float*)p;
    return LUMINA_OK;
  }
  if (parse_layer_name(name, &l, &what) && l >= 0 && l < m->c.n_layer &&
      (what == "mlp.gate.weight" || what == "mlp.gate_bias")) {
    // virtual-MoE router (E, d) and its bias (E), kept raw by the converter
    // and rounded to fp16 with every other tensor (chat.py:140)
    const bool is_w = what == "mlp.gate.weight";
    LUMINA_CHECK_ARG(is_w ? cols == m->d : cnt <= (size_t)MOE_MAX_E, "%s: shape (%d, %d) does not fit d_model %d",
                     name, rows, cols, m->d);
    std::vector<float> f(cnt);
    for (size_t i = 0; i < cnt; ++i) f[i] = __half2float(__float2half_rn(host[i]));
    void* p = nullptr;
    TRY(dalloc(m, &p, cnt * 4));
    LUMINA_CUDA_TRY(cudaMemcpy(p, f.data(), cnt * 4, cudaMemcpyHostToDevice));
    if (is_w) {
      m->L[l].router_w = (float*)p;
      m->L[l].router_rows = rows;
    } else {
      m->L[l].router_b = (float*)p;
      m->L[l].router_blen = (int)cnt;
    }
    return LUMINA_OK;
  }
  set_error("model_set_tensor: %s is not a raw tensor this model uses (raw projections are not built)", name);
  return LUMINA_E_UNSUPPORTED;
}

int lumina_model_finalize(lumina_model* m) {
  LUMINA_CHECK_ARG(m, "model_finalize: null model");
  if (m->finalized) return LUMINA_OK;
  Guard g(m->device);
  const lumina_model_config& c = m->c;
  if (!m->embed) {
    set_error("model_finalize: missing model.embed_tokens.weight");
    return LUMINA_E_STATE;
  }
  if (!m->head) {  // tied head (chat.py:194-195)
    if (c.tp_size > 1) {
      set_error("model_finalize: a tied head needs lm_head.weight shards under TP");
      return LUMINA_E_STATE;
    }
    m->head = m->embed;
    m->head_rows = m->embed_rows;
  }
  const int qw = m->nh * m->hd, kw = m->nkv * m->hd;
  bool any_moe = false;
  int moe_k = 1, moe_ie = 1;
  for (int l = 0; l < c.n_layer; ++l) {
    Layer& Ly = m->L[l];
    const bool moe = Ly.moe_e > 0;
    if (!Ly.q || !Ly.k || !Ly.v || !Ly.o || !Ly.in_norm || !Ly.post_norm ||
        (!moe && (!Ly.gate || !Ly.up || !Ly.down))) {
      set_error("model_finalize: layer %d is missing a tensor", l);
      return LUMINA_E_STATE;
    }
    if (Ly.q->rows != qw || Ly.k->rows != kw || Ly.v->rows != kw || Ly.q->cols != m->d || Ly.o->rows != m->d ||
        Ly.o->cols != qw ||
        (!moe && (Ly.gate->cols != m->d || Ly.up->rows != Ly.gate->rows || Ly.down->rows != m->d ||
                  Ly.down->cols != Ly.gate->rows))) {
      set_error("model_finalize: layer %d shapes do not match the config", l);
      return LUMINA_E_ARG;
    }
    if (moe) {
      // virtual-MoE MLP: under tensor parallelism each rank holds E / tp of
      // the experts (lumina_model_set_moe) and the full router
      if (Ly.router_rows != Ly.moe_e || (Ly.router_b && Ly.router_blen != Ly.moe_e)) {
        set_error("model_finalize: layer %d router has %d rows / %d biases for %d experts", l, Ly.router_rows,
                  Ly.router_blen, Ly.moe_e);
        return LUMINA_E_ARG;
      }
      MoeLayerArgs ma{Ly.moe_gu, Ly.moe_down, Ly.router_w, Ly.router_b, Ly.post_norm, c.eps,
                      Ly.moe_e, Ly.moe_ie, Ly.moe_k, m->d};
      ma.e_lo = Ly.moe_e_lo;
      ma.e_n = Ly.moe_e_n;
      TRY(moe_check(ma));
      any_moe = true;
      moe_k = std::max(moe_k, Ly.moe_k);
      moe_ie = std::max(moe_ie, Ly.moe_ie);
    } else {
      if (m->ffn == 0) m->ffn = Ly.gate->rows;
      if (Ly.gate->rows != m->ffn) {
        set_error("model_finalize: layer %d ffn %d != %d", l, Ly.gate->rows, m->ffn);
        return LUMINA_E_ARG;
      }
    }
    int rc = LUMINA_OK;
    if (compatible(Ly.q, Ly.k) && compatible(Ly.q, Ly.v)) {
      Ly.qkv = build_qkv(Ly.q, Ly.k, Ly.v, m->hd, &rc, wants_tc(Ly.q));
      if (rc) return rc;
      lumina_weight_free(Ly.q);
      lumina_weight_free(Ly.k);
      lumina_weight_free(Ly.v);
      Ly.q = Ly.k = Ly.v = Ly.qkv;  // keep non-null for the shape checks; freed once
    }
    if (moe) {
      if (!Ly.o->mma && wants_tc(Ly.o)) {
        lumina_weight* t = to_fragment_layout(Ly.o, &rc);
        if (rc) return rc;
        lumina_weight_free(Ly.o);
        Ly.o = t;
      }
      continue;
    }
    if (compatible(Ly.gate, Ly.up)) {
      Ly.gu = build_gu(Ly.gate, Ly.up, &rc, wants_tc(Ly.gate));
      if (rc) return rc;
      lumina_weight_free(Ly.gate);
      lumina_weight_free(Ly.up);
      Ly.gate = Ly.up = Ly.gu;
    }
    for (lumina_weight** pw : {&Ly.o, &Ly.down}) {
      if ((*pw)->mma || !wants_tc(*pw)) continue;
      lumina_weight* t = to_fragment_layout(*pw, &rc);
      if (rc) return rc;
      lumina_weight_free(*pw);
      *pw = t;
    }
  }
  // rope tables
  if (m->rope_cos_h.empty() || m->rope_sin_h.empty()) default_rope(m);
  const size_t rbytes = m->rope_cos_h.size() * 4;
  TRY(dalloc(m, (void**)&m->rope_cos, rbytes));
  TRY(dalloc(m, (void**)&m->rope_sin, rbytes));
  LUMINA_CUDA_TRY(cudaMemcpy(m->rope_cos, m->rope_cos_h.data(), rbytes, cudaMemcpyHostToDevice));
  LUMINA_CUDA_TRY(cudaMemcpy(m->rope_sin, m->rope_sin_h.data(), rbytes, cudaMemcpyHostToDevice));
  // KV pool [layer][block][nkv][bs][hd]
  m->n_blocks = (c.max_seq + c.block_size - 1) / c.block_size;
  m->layer_elems = (size_t)m->n_blocks * m->nkv * c.block_size * m->hd;
  TRY(dalloc(m, &m->kpool, m->layer_elems * c.n_layer * kv_es(m)));
  TRY(dalloc(m, &m->vpool, m->layer_elems * c.n_layer * kv_es(m)));
  TRY(dalloc(m, (void**)&m->bt_dev, (size_t)m->n_blocks * 4));
  m->free_blocks.clear();
  for (int b = m->n_blocks - 1; b >= 0; --b) m->free_blocks.push_back(b);
  // activations
  const int R = c.max_rows, V = m->head_rows * c.tp_size;
  TRY(dalloc(m, (void**)&m->x, (size_t)R * m->d * 4));
  TRY(dalloc(m, (void**)&m->qkv_buf, (size_t)R * (qw + 2 * kw) * 4));
  TRY(dalloc(m, (void**)&m->q_buf, (size_t)R * qw * 4));
  TRY(dalloc(m, (void**)&m->attn, (size_t)R * qw * 4));
  TRY(dalloc(m, (void**)&m->ffn_buf, (size_t)R * m->ffn * 4));
  TRY(dalloc(m, (void**)&m->g_buf, (size_t)R * m->ffn * 4));
  TRY(dalloc(m, (void**)&m->u_buf, (size_t)R * m->ffn * 4));
  TRY(dalloc(m, (void**)&m->part, (size_t)std::max(R * m->d, m->head_rows) * 4));
  TRY(dalloc(m, (void**)&m->logits, (size_t)R * V * 4));
  const int kmax = std::max(std::max(m->d, qw), m->ffn);
  const int nblk_pad = ((kmax + 31) / 32 + 4) / 4 * 4;  // whole chunks for every kind
  if (R >= TC05_MIN_ROWS) {
    m->x16_bytes = gemm_tc05_x16_elems(R, kmax) * 2;
    TRY(dalloc(m, (void**)&m->x16, m->x16_bytes));
    TRY(dalloc(m, (void**)&m->split.ws, SPLIT_WS_ELEMS * sizeof(float)));
    TRY(dalloc(m, (void**)&m->split.cnt, SPLIT_COUNTERS * sizeof(int)));
    LUMINA_CUDA_TRY(cudaMemset(m->split.cnt, 0, SPLIT_COUNTERS * sizeof(int)));
    LUMINA_CUDA_TRY(cudaDeviceSynchronize());  // zero before the model's non-blocking stream starts
    m->split.ws_elems = SPLIT_WS_ELEMS;
    m->split.cnt_n = SPLIT_COUNTERS;
  }
  void* aqb = nullptr;
  TRY(dalloc(m, &aqb, actq_scratch_bytes(R, nblk_pad)));
  actq_carve(aqb, R, nblk_pad, &m->aq);
  TRY(dalloc(m, &m->kv_tmp, (size_t)R * 2 * m->nkv * m->hd * kv_es(m)));
  m->bias_rows = std::min(64, R);
  TRY(dalloc(m, (void**)&m->bias_dev, (size_t)m->bias_rows * (c.max_seq + 1) * 4));
  TRY(dalloc(m, (void**)&m->P_dev, sizeof(DevParams)));
  TRY(dalloc(m, (void**)&m->rowpos_dev, (size_t)R * 4));
  TRY(dalloc(m, (void**)&m->tokens_dev, (size_t)R * 4));
  TRY(dalloc(m, (void**)&m->argmax_dev, 4));
  TRY(dalloc(m, (void**)&m->amax_key_dev, 8));
  TRY(dalloc(m, (void**)&m->chain_tokens, (size_t)(c.max_seq + 1) * 4));
  TRY(dalloc(m, (void**)&m->chain_count, 4));
  if (c.tp_size > 1) {
    // the exchange region other ranks map (peer.cu): flags, then three slots
    // (o_proj sums, down_proj sums, a logits shard) of this rank's contribution
    static_assert(PEER_CTAS * PEER_MAX * 4 <= PEER_FLAG_BYTES, "exchange flags");
    LUMINA_CHECK_ARG(c.tp_size <= PEER_MAX, "model_finalize: tp_size %d > %d", c.tp_size, PEER_MAX);
    m->exch_slot = (std::max((size_t)R * m->d, (size_t)m->head_rows) + 63) / 64 * 64;
    // [flags][slot 0..2][receive slots: 2 kinds x PEER_MAX ranks x TP_PUSH_ROWS rows]
    const size_t push_floats = 2 * (size_t)PEER_MAX * TP_PUSH_ROWS * m->d;
    TRY(dalloc(m, (void**)&m->exch, PEER_FLAG_BYTES + (3 * m->exch_slot + push_floats) * 4));
    LUMINA_CUDA_TRY(cudaMemset(m->exch, 0, PEER_FLAG_BYTES));
    TRY(dalloc(m, (void**)&m->peer_epoch, PEER_CTAS * 4));
    LUMINA_CUDA_TRY(cudaMemset(m->peer_epoch, 0, PEER_CTAS * 4));
    TRY(dalloc(m, (void**)&m->tp_epoch, 2 * sizeof(unsigned)));
    TRY(dalloc(m, (void**)&m->tp_ticket, 2 * sizeof(int)));
    LUMINA_CUDA_TRY(cudaMemset(m->tp_epoch, 0, 2 * sizeof(unsigned)));
    LUMINA_CUDA_TRY(cudaMemset(m->tp_ticket, 0, 2 * sizeof(int)));
    TRY(dalloc(m, (void**)&m->xa, (size_t)TP_PUSH_ROWS * m->d * 4));
    TRY(dalloc(m, (void**)&m->xb, (size_t)TP_PUSH_ROWS * m->d * 4));
  }
  if (any_moe) {
    TRY(moe_prepare(m->d));
    TRY(dalloc(m, (void**)&m->moe.h, (size_t)R * m->d * 4));
    TRY(dalloc(m, (void**)&m->moe.score, (size_t)R * MOE_MAX_E * 4));
    TRY(dalloc(m, (void**)&m->moe.act, (size_t)R * moe_k * moe_ie * 4));
    TRY(dalloc(m, (void**)&m->moe.part, moe_part_rows(R) * m->d * 4));
    TRY(dalloc(m, (void**)&m->moe.counters, (size_t)(m->d / 64) * 4));
    LUMINA_CUDA_TRY(cudaMemset(m->moe.counters, 0, (size_t)(m->d / 64) * 4));
  }
  if (!fault_flag_ptr()) {
    set_error("model_finalize: fault flag unavailable");
    return LUMINA_E_CUDA;
  }
  TRY(dalloc(m, (void**)&m->src_dev, (size_t)R * 4));
  if (cudaMallocHost(&m->P_host, sizeof(DevParams)) != cudaSuccess ||
      cudaMallocHost(&m->rowpos_host, (size_t)R * 4) != cudaSuccess ||
      cudaMallocHost(&m->tokens_host, (size_t)R * 4) != cudaSuccess ||
      cudaMallocHost(&m->argmax_host, 4) != cudaSuccess ||
      cudaMallocHost(&m->amax_key_host, 8) != cudaSuccess || cudaMallocHost(&m->fault_host, 4) != cudaSuccess ||
      cudaMallocHost(&m->logits_host, (size_t)V * 4) != cudaSuccess) {
    cudaGetLastError();
    set_error("model_finalize: pinned host allocation failed");
    return LUMINA_E_OOM;
  }
  LUMINA_CUDA_TRY(cudaEventCreate(&m->ev0));
  LUMINA_CUDA_TRY(cudaEventCreate(&m->ev1));
  LUMINA_CUDA_TRY(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
  m->finalized = true;
  return LUMINA_OK;
}

int lumina_model_free(lumina_model* m) {
  if (!m) return LUMINA_OK;
  Guard g(m->device);
  if (m->stream) cudaStreamSynchronize(m->stream);
  if (m->step_graph) cudaGraphExecDestroy(m->step_graph);
  if (m->chain_graph) cudaGraphExecDestroy(m->chain_graph);
  if (m->ev0) cudaEventDestroy(m->ev0);
  if (m->ev1) cudaEventDestroy(m->ev1);
  for (int r = 0; r < PEER_MAX; ++r)
    if (m->peer_exch[r] && m->peer_exch[r] != m->exch) cudaIpcCloseMemHandle(m->peer_exch[r]);
  for (Layer& Ly : m->L) {
    if (Ly.qkv) {
      lumina_weight_free(Ly.qkv);
    } else {
      lumina_weight_free(Ly.q);
      lumina_weight_free(Ly.k);
      lumina_weight_free(Ly.v);
    }
    if (Ly.gu) {
      lumina_weight_free(Ly.gu);
    } else {
      lumina_weight_free(Ly.gate);
      lumina_weight_free(Ly.up);
    }
    lumina_weight_free(Ly.o);
    lumina_weight_free(Ly.down);
    lumina_weight_free(Ly.moe_gu);
    lumina_weight_free(Ly.moe_down);
  }
  for (void* p : m->allocs) cudaFree(p);
  if (m->P_host) cudaFreeHost(m->P_host);
  if (m->rowpos_host) cudaFreeHost(m->rowpos_host);
  if (m->tokens_host) cudaFreeHost(m->tokens_host);
  if (m->argmax_host) cudaFreeHost(m->argmax_host);
  if (m->amax_key_host) cudaFreeHost(m->amax_key_host);
  if (m->fault_host) cudaFreeHost(m->fault_host);
  if (m->logits_host) cudaFreeHost(m->logits_host);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
  return LUMINA_OK;
}

int lumina_model_peer_handle(lumina_model* m, uint8_t* handle64) {
  TRY(check_ready(m));
  LUMINA_CHECK_ARG(handle64, "model_peer_handle: null out");
  LUMINA_CHECK_ARG(m->c.tp_size > 1 && m->exch, "model_peer_handle: the model is not tensor-parallel");
  Guard g(m->device);
  cudaIpcMemHandle_t h;
  static_assert(sizeof(h) == 64, "cudaIpcMemHandle_t size");
  LUMINA_CUDA_TRY(cudaIpcGetMemHandle(&h, m->exch));
  memcpy(handle64, &h, 64);
  return LUMINA_OK;
}

int lumina_model_init_peers(lumina_model* m, const uint8_t* handles) {
  TRY(check_ready(m));
  LUMINA_CHECK_ARG(handles, "model_init_peers: null handles");
  LUMINA_CHECK_ARG(m->c.tp_size > 1 && m->exch, "model_init_peers: the model is not tensor-parallel");
  LUMINA_CHECK_ARG(!m->peers_ready, "model_init_peers: already joined");
  Guard g(m->device);
  for (int r = 0; r < m->c.tp_size; ++r) {
    if (r == m->c.tp_rank) {
      m->peer_exch[r] = m->exch;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, handles + (size_t)r * 64, 64);
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      cudaGetLastError();
      set_error("model_init_peers: opening rank %d's exchange region: %s", r, cudaGetErrorString(e));
      return LUMINA_E_CUDA;
    }
    m->peer_exch[r] = static_cast<char*>(p);
  }
  m->peers_ready = true;
  // LUMINA_TP_FUSED_EXCHANGE=1: the decode step fuses its exchanges into the
  // GEMVs when every projection it needs runs on the tensor-pipe GEMV (int4
  // fragment layout, fused q/k/v and gate/up). Off by default: measured at
  // 447 tok/s against 523 for the exchange kernels on two B200s (7B int4).
  const char* fe = getenv("LUMINA_TP_FUSED_EXCHANGE");
  m->tp_fusable = fe && fe[0] == '1';
  for (const Layer& Ly : m->L) {
    const lumina_weight* ws[4] = {Ly.qkv, Ly.o, Ly.gu, Ly.down};
    for (const lumina_weight* w : ws)
      if (!w || !w->mma || w->bits != 4 || w->group % 64) m->tp_fusable = false;
    if (Ly.moe_e) m->tp_fusable = false;
  }
  return LUMINA_OK;
}

int lumina_kv_length(const lumina_model* m, int layer, int* len) {
  LUMINA_CHECK_ARG(m && len, "kv_length: null pointer");
  if (layer < 0) return uniform_len(m, len);
  LUMINA_CHECK_ARG(layer < m->c.n_layer, "kv_length: layer %d", layer);
  *len = m->layer_len[layer];
  return LUMINA_OK;
}

int lumina_kv_truncate(lumina_model* m, int len) {
  TRY(check_ready(m));
  int cur = 0;
  for (int v : m->layer_len) cur = std::max(cur, v);
  LUMINA_CHECK_ARG(len >= 0 && len <= cur, "kv_truncate: %d not in [0, %d]", len, cur);
  for (auto& v : m->layer_len) v = std::min(v, len);
  release_blocks(m, len);
  return LUMINA_OK;
}

int lumina_kv_read(const lumina_model* mc, int layer, int start, int n, float* k_host, float* v_host) {
  lumina_model* m = const_cast<lumina_model*>(mc);
  TRY(check_ready(m));
  LUMINA_CHECK_ARG(k_host && v_host, "kv_read: null output");
  LUMINA_CHECK_ARG(layer >= 0 && layer < m->c.n_layer, "kv_read: layer %d", layer);
  LUMINA_CHECK_ARG(start >= 0 && n >= 0 && start + n <= m->layer_len[layer], "kv_read: rows [%d, %d) beyond %d", start,
                   start + n, m->layer_len[layer]);
  if (n == 0) return LUMINA_OK;
  Guard g(m->device);
  float* tmp = nullptr;
  const size_t cnt = (size_t)n * m->nh * m->hd;
  LUMINA_CUDA_TRY(cudaMallocAsync((void**)&tmp, cnt * 8, m->stream));
  int rc = launch_kv_read(m->c.kv_fp16, layer_k(m, layer), layer_v(m, layer), m->bt_dev, m->c.block_size, m->nh,
                          m->nkv, m->hd, start, n, tmp, tmp + cnt, m->stream);
  if (!rc) {
    cudaMemcpyAsync(k_host, tmp, cnt * 4, cudaMemcpyDeviceToHost, m->stream);
    cudaMemcpyAsync(v_host, tmp + cnt, cnt * 4, cudaMemcpyDeviceToHost, m->stream);
  }
  cudaFreeAsync(tmp, m->stream);
  LUMINA_CUDA_TRY(cudaStreamSynchronize(m->stream));
  return rc;
}

int lumina_kv_commit_rows(lumina_model* m, int base, const int* src_host, int n) {
  TRY(check_ready(m));
  int len = 0;
  TRY(uniform_len(m, &len));
  LUMINA_CHECK_ARG(n >= 0 && n <= m->c.max_rows && base >= 0 && base + n <= len, "kv_commit_rows: bad range");
  LUMINA_CHECK_ARG(n == 0 || src_host, "kv_commit_rows: null src");
  for (int i = 0; i < n; ++i)
    LUMINA_CHECK_ARG(src_host[i] >= 0 && base + src_host[i] < len, "kv_commit_rows: src[%d]=%d out of range", i,
                     src_host[i]);
  Guard g(m->device);
  if (n) {
    for (int i = 0; i < n; ++i) m->tokens_host[i] = src_host[i];
    LUMINA_CUDA_TRY(cudaMemcpyAsync(m->src_dev, m->tokens_host, n * 4, cudaMemcpyHostToDevice, m->stream));
    for (int l = 0; l < m->c.n_layer; ++l)
      TRY(launch_kv_gather(m->c.kv_fp16, layer_k(m, l), layer_v(m, l), m->bt_dev, m->c.block_size, m->nkv, m->hd, base,
                           m->src_dev, n, m->kv_tmp, m->stream));
    LUMINA_CUDA_TRY(cudaStreamSynchronize(m->stream));
  }
  for (auto& v : m->layer_len) v = base + n;
  release_blocks(m, base + n);
  return LUMINA_OK;
}

int lumina_kv_attend(lumina_model* m, int layer, const float* q_host, float* out_host) {
  TRY(check_ready(m));
  LUMINA_CHECK_ARG(q_host && out_host, "kv_attend: null pointer");
  LUMINA_CHECK_ARG(layer >= 0 && layer < m->c.n_layer, "kv_attend: layer %d", layer);
  const int len = m->layer_len[layer];
  LUMINA_CHECK_ARG(len >= 1, "kv_attend: layer %d holds no rows", layer);
  Guard g(m->device);
  const size_t qn = (size_t)m->nh * m->hd;
  DevParams& P = *m->P_host;
  P.n = 1;
  P.t_prev = len;  // no row of this call is new: every key is read after the dependency wait
  P.t_tot = len;
  P.n_splits = 1;
  P.bias_ld = 0;
  LUMINA_CUDA_TRY(cudaMemcpyAsync(m->P_dev, m->P_host, sizeof(DevParams), cudaMemcpyHostToDevice, m->stream));
  LUMINA_CUDA_TRY(cudaMemcpyAsync(m->q_buf, q_host, qn * 4, cudaMemcpyHostToDevice, m->stream));
  TRY(launch_attention_cluster(m->c.kv_fp16, m->hd, m->q_buf, m->nh, m->nkv, layer_k(m, layer), layer_v(m, layer),
                               m->bt_dev, m->c.block_size, m->P_dev, m->attn, m->stream));
  LUMINA_CUDA_TRY(cudaMemcpyAsync(out_host, m->attn, qn * 4, cudaMemcpyDeviceToHost, m->stream));
  LUMINA_CUDA_TRY(cudaStreamSynchronize(m->stream));
  return LUMINA_OK;
}

int lumina_layer_forward(lumina_model* m, int layer, float* x_dev, int n, int pos0, const int* pos_override_host,
                         const float* bias_host, void* stream) {
  TRY(check_ready(m));
  TRY(check_peers(m));
  LUMINA_CHECK_ARG(x_dev, "layer_forward: null x");
  LUMINA_CHECK_ARG(layer >= 0 && layer < m->c.n_layer, "layer_forward: layer %d", layer);
  LUMINA_CHECK_ARG(n >= 1 && n <= m->c.max_rows, "layer_forward: %d rows not in [1, %d]", n, m->c.max_rows);
  LUMINA_CHECK_ARG(!bias_host || n <= m->bias_rows, "layer_forward: bias with %d rows > %d", n, m->bias_rows);
  Guard g(m->device);
  cudaStream_t user = (cudaStream_t)stream;
  const int t_prev = m->layer_len[layer];
  TRY(ensure_blocks(m, t_prev + n));
  std::vector<int> pos(n);
  for (int i = 0; i < n; ++i) pos[i] = pos_override_host ? pos_override_host[i] : pos0 + i;
  for (int i = 0; i < n; ++i)
    LUMINA_CHECK_ARG(pos[i] >= 0 && pos[i] <= m->c.max_seq, "layer_forward: position %d beyond RoPE table", pos[i]);
  // order the model stream after the caller's work on x
  cudaEvent_t ev;
  LUMINA_CUDA_TRY(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  cudaEventRecord(ev, user);
  cudaStreamWaitEvent(m->stream, ev, 0);
  TRY(upload_params(m, n, t_prev, pos.data(), nullptr, t_prev + n));
  if (bias_host) {
    LUMINA_CUDA_TRY(cudaMemcpy2DAsync(m->bias_dev, (size_t)(t_prev + n) * 4, bias_host, (size_t)(t_prev + n) * 4,
                                      (size_t)(t_prev + n) * 4, n, cudaMemcpyHostToDevice, m->stream));
  }
  LUMINA_CUDA_TRY(cudaMemcpyAsync(m->x, x_dev, (size_t)n * m->d * 4, cudaMemcpyDeviceToDevice, m->stream));
  int rc = clear_fault_async(m->stream);
  if (!rc) rc = run_layer(m, layer, n, bias_host ? m->bias_dev : nullptr);
  if (!rc) {
    cudaMemcpyAsync(x_dev, m->x, (size_t)n * m->d * 4, cudaMemcpyDeviceToDevice, m->stream);
    cudaEventRecord(ev, m->stream);
    cudaStreamWaitEvent(user, ev, 0);
    m->layer_len[layer] = t_prev + n;
  }
  // pinned params / host bias must outlive the copies that read them
  const int rc2 = finish_checked(m, "layer_forward");
  cudaEventDestroy(ev);
  return rc ? rc : rc2;
}

int lumina_forward(lumina_model* m, const int* tokens_host, int n, int pos0, const int* pos_override_host,
                   const float* bias_host, float* logits_host, int all_rows) {
  TRY(check_ready(m));
  TRY(check_peers(m));
  LUMINA_CHECK_ARG(tokens_host && n >= 1, "forward: no tokens");
  Guard g(m->device);
  return forward_rows(m, tokens_host, n, pos0, pos_override_host, bias_host, all_rows, logits_host);
}

int lumina_decode_step(lumina_model* m, int token, float* logits_host, int* argmax_host) {
  TRY(check_ready(m));
  TRY(check_peers(m));
  LUMINA_CHECK_ARG(token >= 0 && token < m->embed_rows, "decode_step: token %d out of range", token);
  Guard g(m->device);
  int len = 0;
  TRY(uniform_len(m, &len));
  TRY(ensure_blocks(m, len + 1));
  DevParams& P = *m->P_host;
  P.n = 1;
  P.t_prev = len;
  P.t_tot = len + 1;
  P.n_splits = 1;
  P.bias_ld = 0;
  m->rowpos_host[0] = len;
  m->tokens_host[0] = token;
  if (!m->step_graph) TRY(capture_step(m));
  LUMINA_CUDA_TRY(cudaGraphLaunch(m->step_graph, m->stream));
  LUMINA_CUDA_TRY(cudaStreamSynchronize(m->stream));
  for (auto& v : m->layer_len) v = len + 1;
  if (*m->fault_host) {
    // the step graph clears the word as it starts, so the bits are this step's
    const int word = *m->fault_host;
    *m->fault_host = 0;
    return fault_error("decode_step", word);
  }
  const int V = m->head_rows * m->c.tp_size;
  if (logits_host) memcpy(logits_host, m->logits_host, (size_t)V * 4);
  if (argmax_host)
    *argmax_host = m->c.tp_size > 1 ? *m->argmax_host
                                    : (int)(0xFFFFFFFFu - (unsigned)(*m->amax_key_host & 0xFFFFFFFFull));
  return LUMINA_OK;
}

int lumina_decode_greedy(lumina_model* m, int token, int n, int* tokens_host, float* device_ms,
                         int* kernels_per_step) {
  TRY(check_ready(m));
  TRY(check_peers(m));
  LUMINA_CHECK_ARG(token >= 0 && token < m->embed_rows, "decode_greedy: token %d out of range", token);
  LUMINA_CHECK_ARG(n >= 1 && tokens_host, "decode_greedy: bad n / output");
  Guard g(m->device);
  int len = 0;
  TRY(uniform_len(m, &len));
  TRY(ensure_blocks(m, len + n));
  std::vector<int> pos(1, len);
  TRY(upload_params(m, 1, len, pos.data(), &token, 0));
  LUMINA_CUDA_TRY(cudaMemsetAsync(m->chain_count, 0, 4, m->stream));
  LUMINA_CUDA_TRY(cudaMemsetAsync(fault_flag_ptr(), 0, 4, m->stream));
  if (!m->chain_graph) TRY(capture_chain(m));
  if (device_ms) LUMINA_CUDA_TRY(cudaEventRecord(m->ev0, m->stream));
  for (int i = 0; i < n; ++i) LUMINA_CUDA_TRY(cudaGraphLaunch(m->chain_graph, m->stream));
  if (device_ms) LUMINA_CUDA_TRY(cudaEventRecord(m->ev1, m->stream));
  LUMINA_CUDA_TRY(cudaMemcpyAsync(tokens_host, m->chain_tokens, (size_t)n * 4, cudaMemcpyDeviceToHost, m->stream));
  LUMINA_CUDA_TRY(cudaMemcpyAsync(m->fault_host, fault_flag_ptr(), 4, cudaMemcpyDeviceToHost, m->stream));
  LUMINA_CUDA_TRY(cudaStreamSynchronize(m->stream));
  for (auto& v : m->layer_len) v = len + n;
  if (device_ms) LUMINA_CUDA_TRY(cudaEventElapsedTime(device_ms, m->ev0, m->ev1));
  if (kernels_per_step) *kernels_per_step = m->chain_kernels;
  if (*m->fault_host) {
    const int word = *m->fault_host;
    *m->fault_host = 0;
    cudaMemset(fault_flag_ptr(), 0, sizeof(int));
    return fault_error("decode_greedy", word);
  }
  return LUMINA_OK;
}

int lumina_profile_attention(lumina_model* m, int iters, float* ms_per_launch, double* bytes_per_launch) {
  TRY(check_ready(m));
  LUMINA_CHECK_ARG(iters >= 1 && ms_per_launch, "profile_attention: bad arguments");
  int len = 0;
  TRY(uniform_len(m, &len));
  LUMINA_CHECK_ARG(len >= 1, "profile_attention: the KV cache is empty");
  Guard g(m->device);
  // the decode row's attention at the current length: every key visible, the
  // last cached row standing in for the step's new row
  DevParams& P = *m->P_host;
  P.n = 1;
  P.t_prev = len - 1;
  P.t_tot = len;
  P.n_splits = 1;
  P.bias_ld = 0;
  LUMINA_CUDA_TRY(cudaMemcpyAsync(m->P_dev, m->P_host, sizeof(DevParams), cudaMemcpyHostToDevice, m->stream));
  auto all_layers = [&]() -> int {
    for (int l = 0; l < m->c.n_layer; ++l)
      TRY(launch_attention_cluster(m->c.kv_fp16, m->hd, m->q_buf, m->nh, m->nkv, layer_k(m, l), layer_v(m, l),
                                   m->bt_dev, m->c.block_size, m->P_dev, m->attn, m->stream));
    return LUMINA_OK;
  };
  TRY(all_layers());  // warm outside the capture
  LUMINA_CUDA_TRY(cudaStreamSynchronize(m->stream));
  cudaGraph_t gr = nullptr;
  cudaGraphExec_t ge = nullptr;
  LUMINA_CUDA_TRY(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
  int rc = LUMINA_OK;
  for (int i = 0; i < iters && !rc; ++i) rc = all_layers();
  const cudaError_t ec = cudaStreamEndCapture(m->stream, &gr);
  if (rc || ec != cudaSuccess) {
    if (gr) cudaGraphDestroy(gr);
    if (!rc) set_error("profile_attention capture: %s", cudaGetErrorString(ec));
    return rc ? rc : LUMINA_E_CUDA;
  }
  if (cudaGraphInstantiate(&ge, gr, 0) != cudaSuccess) {
    cudaGraphDestroy(gr);
    set_error("profile_attention: instantiate failed");
    return LUMINA_E_CUDA;
  }
  cudaGraphDestroy(gr);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaGraphLaunch(ge, m->stream);
  cudaEventRecord(e0, m->stream);
  cudaGraphLaunch(ge, m->stream);
  cudaEventRecord(e1, m->stream);
  const cudaError_t es = cudaEventSynchronize(e1);
  float ms = 0.f;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaGraphExecDestroy(ge);
  if (es != cudaSuccess) {
    set_error("profile_attention: %s", cudaGetErrorString(es));
    return LUMINA_E_CUDA;
  }
  *ms_per_launch = ms / (float)(iters * m->c.n_layer);
  // K and V rows read (this shard's heads), q read, output written
  if (bytes_per_launch)
    *bytes_per_launch = (double)len * 2.0 * m->nkv * m->hd * kv_es(m) + 2.0 * m->nh * m->hd * 4;
  return LUMINA_OK;
}

int lumina_profile_gemv(lumina_model* m, int iters, float* ms_per_launch, int* launches_per_token,
                        double* bytes_per_token) {
  TRY(check_ready(m));
  LUMINA_CHECK_ARG(iters >= 1 && ms_per_launch, "profile_gemv: bad arguments");
  Guard g(m->device);
  const int d = m->d, qw = m->nh * m->hd, width = qw + 2 * m->nkv * m->hd;
  int launches = 0;
  double bytes = 0.0;
  // the decode token's packed GEMVs, epilogues that write only scratch
  auto one_token = [&](bool count) -> int {
    for (int l = 0; l < m->c.n_layer; ++l) {
      Layer& Ly = m->L[l];
      const lumina_weight* ws[4] = {Ly.qkv ? Ly.qkv : Ly.q, Ly.o, Ly.gu ? Ly.gu : Ly.gate, Ly.down};
      const float* xs[4] = {m->x, m->attn, m->x, m->ffn_buf};
      const float* norms[4] = {Ly.in_norm, nullptr, Ly.post_norm, nullptr};
      float* ys[4] = {m->qkv_buf, m->part, m->ffn_buf, m->part};
      const int epis[4] = {EPI_STORE, EPI_STORE, Ly.gu ? EPI_SWIGLU : EPI_STORE, EPI_STORE};
      const int lds[4] = {width, d, m->ffn, d};
      const int ldx[4] = {d, qw, d, m->ffn};
      const int nproj = Ly.moe_e ? 2 : 4;  // a virtual-MoE MLP is not a packed GEMV
      for (int i = 0; i < nproj; ++i) {
        // each GEMV pulls the next one's weights into L2, as in the decode step
        const lumina_weight* nxt = i + 1 < nproj ? ws[i + 1] : qkv_weight(m, (l + 1) % m->c.n_layer);
        const L2Prefetch pf = prefetch_of(nxt);
        TRY(gemv_any(m, ws[i], xs[i], ldx[i], 1, norms[i], ys[i], lds[i], epis[i], nullptr, 0, nullptr, &pf));
        if (count) {
          ++launches;
          const int out_rows = epis[i] == EPI_SWIGLU ? ws[i]->rows / 2 : ws[i]->rows;
          bytes += (double)packed_bytes(ws[i]) + (double)ws[i]->cols * 4 + (double)out_rows * 4;
        }
      }
    }
    return LUMINA_OK;
  };
  // warm (attributes, first-use setup) outside the capture
  TRY(clear_fault_async(m->stream));
  TRY(one_token(true));
  LUMINA_CUDA_TRY(cudaStreamSynchronize(m->stream));
  cudaGraph_t gr = nullptr;
  cudaGraphExec_t ge = nullptr;
  LUMINA_CUDA_TRY(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
  int rc = LUMINA_OK;
  for (int i = 0; i < iters && !rc; ++i) rc = one_token(false);
  const cudaError_t ec = cudaStreamEndCapture(m->stream, &gr);
  if (rc || ec != cudaSuccess) {
    if (gr) cudaGraphDestroy(gr);
    if (!rc) set_error("profile_gemv capture: %s", cudaGetErrorString(ec));
    return rc ? rc : LUMINA_E_CUDA;
  }
  if (cudaGraphInstantiate(&ge, gr, 0) != cudaSuccess) {
    cudaGraphDestroy(gr);
    set_error("profile_gemv: instantiate failed");
    return LUMINA_E_CUDA;
  }
  cudaGraphDestroy(gr);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaGraphLaunch(ge, m->stream);  // warm replay
  cudaEventRecord(e0, m->stream);
  cudaGraphLaunch(ge, m->stream);
  cudaEventRecord(e1, m->stream);
  const cudaError_t es = cudaEventSynchronize(e1);
  float ms = 0.f;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaGraphExecDestroy(ge);
  if (es != cudaSuccess) {
    set_error("profile_gemv: %s", cudaGetErrorString(es));
    return LUMINA_E_CUDA;
  }
  TRY(finish_checked(m, "profile_gemv"));
  *ms_per_launch = ms / (float)(iters * launches);
  if (launches_per_token) *launches_per_token = launches;
  if (bytes_per_token) *bytes_per_token = bytes;
  return LUMINA_OK;
}

}  // extern "C"
