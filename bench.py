#!/usr/bin/env python3
"""Decode benchmark of the Lumina decode path on B200.

Workload (the reference's headline decode configuration): a Llama-2-7B-shape
decoder (32 layers, d_model 4096, 32 heads x 128, SwiGLU 11008, vocab 32000,
RoPE theta 1e4), every projection Lumina int4 with groups of 64 and
fp16-valued scales, embedding and lm_head raw; batch 1; a 512-token random
prompt is prefilled, then greedy decode tokens follow with an fp16 KV cache
paged in 16-token blocks. Weights are N(0, 0.02), seeded, quantized on the
GPU with the reference's round-to-nearest + MSE scale search (synthetic: no
checkpoint is involved).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

A step is one decode token. The timed region is K device-chained greedy
steps (one CUDA-graph replay each, the argmax fed back on the device),
bracketed by barriers and synchronizes and timed with CUDA events on the
model's stream; the max over ranks is reported. With N > 1 (torchrun, one
rank per GPU) the model is tensor-parallel over the N GPUs (NCCL all-reduce
after o_proj and down_proj, vocab-sharded head): one sequence, fixed total
work, so scaling is strong.

Besides the device-chained loop the line carries
  * e2e: the same K tokens through the public per-token call
    (``CudaChatModel.decode_step`` + the host greedy sampler, as
    ``generate`` runs them): host->device token/position parameters and the
    device->host logits every step, wall clock;
  * roofline: the packed-weight GEMV kernels (the dominant kernel) replayed
    alone for one token's 128 launches, CUDA events on their stream;
    algorithmic bytes (codes + scales + activations + outputs) / time
    against the measured HBM copy bandwidth;
  * cpu_baseline (N = 1): the reference's CPU decode path (the oracle's
    numpy restatement of ChatModel._layer with fp32 weights converted once,
    all BLAS threads) timed on a bounded sample of the same workload;
  * clocks: nvidia-smi samples taken during the timed region.

``--impl reference`` runs only that CPU path (rank 0; other ranks exit 0).
``--moe`` measures the same decode on the virtual-MoE variant of the 7B
shape (every SwiGLU split into 8 routed experts of 1376, top-2); with
``--gpus N`` the attention is tensor-parallel and the experts are split over
the ranks (E/N each, expert parallelism).
``--tiny`` runs the reference's CPU-runnable tiny configuration (64-token
prompt, 128 greedy tokens) on the device and the reference's algorithm on
the host.
``--verify`` times the EAGLE tree verification of a 32-node draft tree over a
4096-token prompt, and the prefill of that prompt.
``--shared-prefix`` decodes 8 sequences over one 2048-token shared prefix
(with ``--moe`` the virtual-MoE shape; ``--gpus N`` TP attention and
expert-parallel experts).
``--sweep`` prints one line per case of the decode-only GEMV sweep (int4 /
int3 / int2 / binary x the four 7B projection shapes x batch 1, 4, 16).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "lumina-studio_b200"))
sys.path.insert(0, REPO)

METRIC = "decode tokens/s and dequant-GEMV HBM GB/s (% peak), 7B int4, 1/2/4/8 B200"
UNIT = "tokens/s"
PROMPT = 512
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126 * 2 ** 20
# kv rows a 7B decode token reads per layer-row: k and v, 4096 fp16 each
KV_BYTES_PER_ROW = 32 * 2 * 4096 * 2


MOE_EXPERTS, MOE_TOP_K = 8, 2


def workload(cfg, tp, moe=False):
    mlp = (f"every SwiGLU split into {MOE_EXPERTS} virtual-MoE experts of "
           f"{cfg['intermediate_size'] // MOE_EXPERTS}, sigmoid router, top-{MOE_TOP_K}, ") if moe else ""
    return {"workload": "llama2-7b-shape decoder, " + mlp + "Lumina int4 g64 fp16 scales, batch 1, "
                        "512-token random prompt prefill then greedy decode, fp16 KV paged in 16-token blocks",
            "layers": cfg["num_hidden_layers"], "d_model": cfg["hidden_size"],
            "heads": cfg["num_attention_heads"], "head_dim": cfg["hidden_size"] // cfg["num_attention_heads"],
            "ffn": cfg["intermediate_size"], "vocab": cfg["vocab_size"], "batch": 1, "prompt": PROMPT,
            "l2": "no flush: each token streams 3.7 GB of weights, > 126 MB L2",
            "parallelism": f"tp{tp}" + (f" attention, ep{tp} experts" if moe and tp > 1 else "")}


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.proc, self.path = gpu, None, None

    def start(self):
        import tempfile
        fd, self.path = tempfile.mkstemp(prefix="clocks", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.5)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for name, v in zip(self.NAMES, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# the reference's CPU decode path (oracle restatement), bounded sample
# ---------------------------------------------------------------------------
def blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 0) for i in threadpool_info() if i.get("user_api") == "blas"]
        return max(n) if n else (os.cpu_count() or 1)
    except Exception:  # noqa: BLE001
        return os.cpu_count() or 1


class CpuDecodeSample:
    """ChatModel._layer decode steps (chat.py:232-304: fp32 weights converted
    once, chat.py:223-230; numpy BLAS on every host core) through all the
    layers of the 7B shape plus the 32000 x 4096 head GEMV (chat.py:322,388),
    the KV cache starting at the 512 prompt rows: one step is one whole
    token, nothing is scaled. The layers cycle through `weight_sets` distinct
    sets of weights (0.8 GB of fp32 each), so a set comes round again only
    after 3 x 0.8 GB of other weights have streamed through the caches: every
    layer reads its weights from DRAM, as the reference's 32 distinct layers
    do, while the host holds 3.2 GB instead of 26 GB of converted weights."""

    def __init__(self, cfg, weight_sets=4, seed=0):
        from oracle.decode import OracleModel
        from lumina_b200 import synthetic
        self.n_layers = cfg["num_hidden_layers"]
        rng = np.random.default_rng(seed)
        vals, t, kind_of = {}, {}, {}
        for name, shape in synthetic.tensor_order(cfg):
            if len(shape) == 1:
                t[name] = np.ones(shape, np.float16)
                continue
            kind = name.split(".")[-2] if name.startswith("model.layers.") else name
            if kind not in vals:
                # std 0.02 (uniform): the CPU path's time does not depend on values
                vals[kind] = ((rng.random(shape, dtype=np.float32) - 0.5) * 0.0693).astype(np.float16)
            t[name] = vals[kind]
            if name.startswith("model.layers."):
                kind_of[name] = (int(name.split(".")[2]) % weight_sets, kind)
        self.m = OracleModel(t, cfg, theta=1e4)
        # the fp32 conversion (OracleModel.W: w.T as fp32, cached by name),
        # one per set and tensor kind; the sets hold equal values in distinct
        # memory (the values do not change the time, the DRAM reads do)
        conv = {}
        for name, key in kind_of.items():
            if key not in conv:
                first = conv.get((0, key[1]))
                conv[key] = t[name].T.astype(np.float32) if first is None else first.copy(order="K")
            self.m._wcache[name] = conv[key]
        self.head_t = self.m.head_t()
        self.emb = self.m.embed()
        nh, hd = self.m.n_heads, self.m.hd
        self.cache = {l: ((rng.random((PROMPT, nh, hd), dtype=np.float32) - 0.5),
                          (rng.random((PROMPT, nh, hd), dtype=np.float32) - 0.5)) for l in range(self.n_layers)}
        self.weight_sets = weight_sets
        self.pos = PROMPT
        self.tok = 1
        self.buf = np.empty((1, self.head_t.shape[1]), np.float32)

    def step(self) -> float:
        """One decode token through every layer and the head; returns its
        seconds."""
        t0 = time.perf_counter()
        h = self.emb[[self.tok]]
        for l in range(self.n_layers):
            h = self.m.layer(h, l, self.cache, self.pos)
        np.dot(h[-1:], self.head_t, out=self.buf)
        self.tok = int(np.argmax(self.buf[0].astype(np.float64)))
        t1 = time.perf_counter()
        self.pos += 1
        return t1 - t0

    def describe(self, tokens):
        return (f"all {self.n_layers} 7B-shape layers ({self.weight_sets} distinct weight sets cycled, "
                f"each re-read from DRAM) + the 32000x4096 head, {tokens} whole decode tokens from KV "
                f"length {PROMPT}; numpy fp32 BLAS over weights converted once")


def cpu_numba_gemv(N=11008, K=4096, calls=5):
    """The reference's numba int8 GEMV (fused._gemv_int8, restated in
    oracle/tops.py) on one host core at the 7B gate/up shape, batch 1: the
    kernel that serves fused_gemv_int8 when the compiled tops kernel is
    absent (tops_int8.c is ARM-only). Median of `calls` after a compiling
    call; bytes = int8 weights + row scales + activations + outputs."""
    from oracle.tops import numba_gemv_int8, q8_repack
    gemv = numba_gemv_int8()
    if gemv is None:
        return {"unavailable": "numba is not importable"}
    rng = np.random.default_rng(0)
    wq = rng.integers(-127, 128, (N, K), dtype=np.int8)
    ws = (rng.random(N, dtype=np.float32) * 0.01 + 1e-3).astype(np.float32)
    xq, xs = q8_repack(rng.standard_normal(K).astype(np.float32))
    out = np.empty(N, np.float32)
    gemv(xq, xs, wq, ws, out)
    ts = []
    for _ in range(calls):
        t0 = time.perf_counter()
        gemv(xq, xs, wq, ws, out)
        ts.append(time.perf_counter() - t0)
    ms = float(np.median(ts)) * 1e3
    nbytes = N * K + N * 4 + K + (K // 32) * 4 + N * 4
    return {"shape": f"{N}x{K} int8, batch 1", "ms": ms, "gb_s": nbytes / ms / 1e6, "cores": 1,
            "impl": "fused._gemv_int8 (fused.py:163-184) restated, numba"}


def numba_leg():
    """cpu_numba_gemv, or why it could not run: the leg reports beside the
    decode baseline and never takes the bench line down with it."""
    try:
        return cpu_numba_gemv()
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"{type(e).__name__}: {e}"[:200]}


def cpu_baseline(cfg, tokens=16, budget_s=20.0):
    s = CpuDecodeSample(cfg)
    s.step()  # converts the fp32 weights (outside the timing, as the reference caches them)
    tot, n = 0.0, 0
    t0 = time.perf_counter()
    while n < tokens and time.perf_counter() - t0 < budget_s:
        tot += s.step()
        n += 1
    return {"value": n / tot, "unit": UNIT, "cores": blas_threads(), "kind": "port",
            "sample": s.describe(n), "numba_gemv_int8": numba_leg()}


def run_reference(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    s = CpuDecodeSample(cfg)
    for _ in range(max(1, args.warmup)):
        s.step()
    tot = 0.0
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tot += s.step()
    wall = time.perf_counter() - t0
    value = args.steps / tot
    cb = {"value": value, "unit": UNIT, "cores": blas_threads(), "kind": "port", "sample": s.describe(args.steps),
          "numba_gemv_int8": numba_leg()}
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": tot / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random weights of the 7B shape)", "config": workload(cfg, 1),
            "cpu_baseline": cb, "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0},
            "sample_wall_s": wall}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# the B200 path
# ---------------------------------------------------------------------------
def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        try:
            return float(json.load(open(p))["hbm_gbs"]), "measured"
        except Exception:  # noqa: BLE001
            pass
    return FALLBACK_HBM_GBS, "fallback"


def traffic_ratio():
    """DRAM bytes / algorithmic bytes of the decode GEMV from the committed
    ncu summary (profiles/gemv_tc_7b_int4_traffic.json), or None."""
    p = os.path.join(REPO, "profiles", "gemv_tc_7b_int4_traffic.json")
    try:
        d = json.load(open(p))
        return float(d["dram_bytes"]) / float(d["algorithmic_bytes"]), d.get("source", p)
    except Exception:  # noqa: BLE001
        return None, None


# GEMV sweep over the per-layer 7B shapes (out rows N, in cols K) and bit widths
SWEEP_SHAPES = ((4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096))
SWEEP_KINDS = (("int4", 4, 64), ("int3", 3, 64), ("int2", 2, 128), ("binary", 1, 128))
SWEEP_BATCHES = (1, 4, 16)


def sweep_bytes(N, K, bits, group, batch):
    """Algorithmic bytes of one GEMV call: packed codes + fp16 scales +
    fp32 activations in + fp32 outputs."""
    return N * ((K * bits + 7) // 8) + N * (-(-K // group)) * 2 + batch * K * 4 + batch * N * 4


def cpu_gemv_us(N, K, batch, cache):
    """The reference's chat-path GEMV on the host cores: fp32 BLAS
    ``h @ W`` over weights dequantized once and kept transposed
    (chat.py:223-243), whatever the code width. Median of 3 calls after a
    warm one; memoised per shape and batch."""
    key = (N, K, batch)
    if key not in cache:
        rng = np.random.default_rng(N + K)
        wt = ((rng.random((K, N), dtype=np.float32) - 0.5) * 0.07).astype(np.float32)
        x = rng.standard_normal((batch, K)).astype(np.float32)
        out = np.empty((batch, N), np.float32)
        np.dot(x, wt, out=out)
        ts = []
        for _ in range(3):
            t0 = time.perf_counter()
            np.dot(x, wt, out=out)
            ts.append(time.perf_counter() - t0)
        cache[key] = float(np.median(ts)) * 1e6
    return cache[key]


def run_sweep(args):
    """Decode-only GEMV sweep: each bit width x shape x batch through the
    public lumina_gemv entry point. A set of weight copies larger than 3x the
    L2 is cycled so every call streams its weights from HBM; the calls are
    captured in one CUDA graph and timed with CUDA events on its stream.
    Beside each case, the reference's own GEMV on the host cores
    (``cpu_gemv_us``). Prints one JSON line per case."""
    import torch
    from lumina_b200.cuda import Weight
    from lumina_b200.packing import to_file_layout
    torch.cuda.set_device(0)
    peak, peak_kind = peaks()
    os.environ["LUMINA_INT4_LAYOUT"] = "mma"  # int4 in the decode model's tensor-pipe layout
    rng = np.random.default_rng(0)
    cpu_cache = {}
    # narrow kinds twice: packed row-major (CUDA-core kernels) and one code
    # per nibble in the fragment layout (the tensor-pipe kernels)
    cases = [(kind, bits, group, lay) for kind, bits, group in SWEEP_KINDS
             for lay in (("mma",) if bits == 4 else ("row", "mma"))]
    for kind, bits, group, lay in cases:
        if bits < 4:
            os.environ["LUMINA_NARROW_LAYOUT"] = lay
        for N, K in SWEEP_SHAPES:
            ng = -(-K // group)
            if kind == "binary":
                blob, pack = rng.integers(0, 256, (N, K // 8), dtype=np.uint8), "none"
            else:
                blob, pack, _ = to_file_layout(kind, rng.integers(0, 1 << bits, (N, K), dtype=np.uint8))
            scales = (np.abs(rng.standard_normal((N, ng))) * 0.02 + 1e-3).astype(np.float16).astype(np.float32)
            wb = sweep_bytes(N, K, bits, group, 0)
            copies = max(2, -(-3 * L2_BYTES // wb))
            ws = [Weight.upload(kind, group, pack, blob, scales, N, K) for _ in range(copies)]
            reps = max(1, -(-64 // copies))
            for batch in SWEEP_BATCHES:
                x = torch.randn(batch, K, device="cuda")
                y = torch.empty(batch, N, device="cuda")
                s = torch.cuda.Stream()
                with torch.cuda.stream(s):
                    for w in ws:  # first-use setup (attributes, scratch) outside the capture
                        w.gemv(x.data_ptr(), batch, K, y.data_ptr(), N, s.cuda_stream)
                    s.synchronize()
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
                        for _ in range(reps):
                            for w in ws:
                                w.gemv(x.data_ptr(), batch, K, y.data_ptr(), N, s.cuda_stream)
                    g.replay()
                    times = []
                    for _ in range(5):
                        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        e0.record(s)
                        g.replay()
                        e1.record(s)
                        e1.synchronize()
                        times.append(e0.elapsed_time(e1) / (reps * copies))
                    del g
                ms = float(np.median(times))
                b = sweep_bytes(N, K, bits, group, batch)
                db = ws[0].info()["device_bytes"] + batch * K * 4 + batch * N * 4
                print(json.dumps({"sweep": "gemv", "kind": kind, "group": group, "N": N, "K": K, "batch": batch,
                                  "layout": "fragment (one code per nibble)" if lay == "mma" and bits < 4 else
                                  ("fragment" if lay == "mma" else "row-major packed"),
                                  "device_bytes_per_call": db,
                                  "us_per_call": ms * 1e3, "bytes_per_call": b, "gbs": b / (ms * 1e-3) / 1e9,
                                  "frac": b / (ms * 1e-3) / 1e9 / peak, "peak_gbs": peak, "peak_kind": peak_kind,
                                  "weight_copies": copies,
                                  "cpu_us_per_call": cpu_gemv_us(N, K, batch, cpu_cache), "cpu_cores": blas_threads(),
                                  "cpu_kind": "the reference's chat-path GEMV: fp32 BLAS over dequantized weights"}),
                      flush=True)
            del ws
    return 0


class _IdTok:
    """Token ids in, token ids out (the prompts here are id lists)."""

    def encode(self, p):
        return [int(t) for t in p]

    def decode(self, ids):
        return " ".join(str(int(i)) for i in ids)


TINY_PROMPT, TINY_DECODE = 64, 128


def run_tiny(args):
    """The reference's CPU-runnable configuration (4 layers, d 256, vocab
    4096, int4 g64, fp32 KV): a 64-token random prompt, then 128 greedy
    decode tokens at batch 1. Device-chained decode (CUDA events), the public
    ``generate`` call end to end (prefill + host sampler, wall clock, the
    way the reference reports tokens_per_second, chat.py:404-407), and the
    reference's algorithm on the host cores (the oracle port over the same
    quantized weights). Prints one JSON line; the config is latency-bound,
    so no roofline fraction is reported."""
    import torch
    from lumina_b200 import synthetic
    from lumina_b200.engine import CudaChatModel, generate
    torch.cuda.set_device(0)
    cfg = dict(synthetic.TINY)
    recs = synthetic.QuantizedRecords(cfg, bits=4, group=64, seed=0, device=0)
    model = CudaChatModel._from_records(recs, synthetic.hf_cfg(cfg), _IdTok(), 4, 4, 1e-6, cfg["rope_theta"], 0,
                                        False, 512, 128, 16, 0, 1)
    try:
        prompt = synthetic.prompt_ids(cfg, TINY_PROMPT, seed=0)
        first = int(np.argmax(model.forward(prompt, 0)[0].astype(np.float64)))
        for _ in range(args.warmup):
            model.decode_greedy(first, TINY_DECODE)
            model.kv_truncate(TINY_PROMPT)
        toks, dev_ms, kernels = model.decode_greedy(first, TINY_DECODE, timed=True)
        generate(model, prompt, max_tokens=TINY_DECODE)  # warm the per-token graph
        r = generate(model, prompt, max_tokens=TINY_DECODE)
        recs_host = {name: recs[name] for name in recs.order}  # the same seeded, quantized tensors
    finally:
        model.close()
    cb = None
    if not args.no_cpu_baseline:
        from oracle import lumina_format as lf
        from oracle.decode import OracleModel, generate as ogen
        # the reference's load-time dequant of the same codes (adapters/lumina.py:135-150)
        t = {n: (np.asarray(r.data, np.float32) if r.kind == "raw" else
                 lf.dequant(r.kind, lf.unpack_codes(r.codes, r.shape, r.pack), r.scales, r.group))
             for n, r in recs_host.items()}
        om = OracleModel(t, synthetic.hf_cfg(cfg), theta=cfg["rope_theta"])
        ogen(om, prompt, 4)  # converts the fp32 weights once, as the reference caches them
        t0 = time.perf_counter()
        otoks = ogen(om, prompt, TINY_DECODE)
        cpu_s = time.perf_counter() - t0
        cb = {"value": TINY_DECODE / cpu_s, "unit": UNIT, "cores": blas_threads(), "kind": "port",
              "sample": f"the whole workload: {TINY_PROMPT}-token prefill + {TINY_DECODE} greedy tokens, numpy fp32",
              "same_tokens": list(otoks) == list(r["tokens"])}
    print(json.dumps({"bench": "tiny_decode", "workload": "tiny decoder (4 layers, d 256, 4 heads x 64, ffn 688, "
                      "vocab 4096), Lumina int4 g64, fp32 KV, 64-token prompt, 128 greedy tokens, batch 1",
                      "decode_tokens_per_s": TINY_DECODE / (dev_ms / 1e3), "ms_per_token": dev_ms / TINY_DECODE,
                      "kernels_per_token": kernels,
                      "e2e_generate_tokens_per_s": r["tokens_per_second"], "e2e_seconds": r["seconds"],
                      # generate's first token is the prefill argmax; the chain starts after it
                      "same_tokens_chained_and_generate": [first] + list(toks)[:-1] == list(r["tokens"]),
                      "cpu_baseline": cb}), flush=True)
    return 0


# EAGLE draft tree of the 7B tree-speculation workload: depth 5, 32 nodes (root + 31 to verify)
VERIFY_PROMPT = 4096
VERIFY_BRANCHING = (4, 2, 1, 1)  # children per node at depths 0..3


def verify_tree_shape():
    """parents, depths of a depth-5, 32-node draft tree: the root's 4
    children, 2 children each, then single chains, plus 3 nodes at depth 5."""
    parents, depths, frontier = [-1], [0], [0]
    for b in VERIFY_BRANCHING:
        nxt = []
        for p in frontier:
            for _ in range(b):
                parents.append(p)
                depths.append(depths[p] + 1)
                nxt.append(len(parents) - 1)
        frontier = nxt
    for p in frontier[:32 - len(parents)]:
        parents.append(p)
        depths.append(depths[p] + 1)
    return parents, depths


def run_verify(args):
    """Tree verification on the 7B int4 model: prefill a 4096-token random
    prompt (time to first token), then repeat the one-forward verification
    of a 31-child draft tree (ancestry bias, true positions; the reference's
    verify_tree, eagle.py:259-291) through the public engine call, rolling
    the KV back after each. Wall clock around synchronous calls; prints one
    JSON line."""
    import torch
    from lumina_b200 import synthetic
    from lumina_b200.engine import CudaChatModel, verify_tree
    torch.cuda.set_device(0)
    cfg = dict(synthetic.LLAMA7B)
    if args.layers:
        cfg["num_hidden_layers"] = args.layers
    recs = synthetic.QuantizedRecords(cfg, bits=4, group=64, seed=0, device=0)
    model = CudaChatModel._from_records(recs, synthetic.hf_cfg(cfg), None, 32, 32, 1e-6, 1e4, 0, True,
                                        VERIFY_PROMPT + 64, 512, 16, 0, 1)
    try:
        prompt = synthetic.prompt_ids(cfg, VERIFY_PROMPT, seed=0)
        model.forward(prompt[:512], 0)  # warm the prefill kernels
        model.kv_truncate(0)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        model.forward(prompt, 0)
        torch.cuda.synchronize()
        prefill_s = time.perf_counter() - t0
        parents, depths = verify_tree_shape()
        rng = np.random.default_rng(5)
        ids = [prompt[-1]] + [int(t) for t in rng.integers(0, cfg["vocab_size"], len(parents) - 1)]
        for _ in range(args.warmup):
            verify_tree(model, VERIFY_PROMPT, ids, parents, depths)
            model.kv_truncate(VERIFY_PROMPT)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            lg, order = verify_tree(model, VERIFY_PROMPT, ids, parents, depths)
            model.kv_truncate(VERIFY_PROMPT)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        print(json.dumps({"bench": "tree_verify", "workload": "llama2-7b-shape int4 g64, fp16 KV, "
                          f"{VERIFY_PROMPT}-token prompt, depth-{max(depths)} {len(parents)}-node draft tree",
                          "verify_rows": len(order), "ms_per_verify": dt / args.steps * 1e3,
                          "verify_rows_per_s": len(order) * args.steps / dt,
                          "prefill_tokens_per_s": VERIFY_PROMPT / prefill_s, "prefill_s": prefill_s,
                          "steps": args.steps, "warmup": args.warmup,
                          "timing": "wall clock around synchronous engine calls (bias build, logits D2H included)"}),
              flush=True)
    finally:
        model.close()
    return 0


SHARED_PREFIX, SHARED_SEQS, SHARED_SUFFIX, SHARED_TOKENS = 2048, 8, 16, 128


def run_shared(args, cfg):
    """Several sequences over a shared prefix on the 7B shape (the virtual-
    MoE variant with --moe): a 2048-token random prefix prefilled once,
    8 sequences that add 16 random tokens each, then 128 greedy tokens per
    sequence through engine.generate_shared_prefix (one forward of the
    live sequences per step; attention over the shared cache with a
    per-sequence bias). With --gpus N the attention is tensor-parallel and
    the experts expert-parallel. Wall clock around the synchronous decode
    steps (logits of every row to the host included), max over ranks; the
    prefix prefill is reported beside it. Prints one JSON line."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from lumina_b200 import synthetic
    from lumina_b200.engine import CudaChatModel, generate_shared_prefix
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device(f"cuda:{local}"))
    moe = (MOE_EXPERTS, MOE_TOP_K) if args.moe else None
    recs = synthetic.QuantizedRecords(cfg, bits=4, group=64, seed=0, device=local, moe=moe)
    max_seq = SHARED_PREFIX + SHARED_SEQS * (SHARED_SUFFIX + SHARED_TOKENS) + 64
    model = CudaChatModel._from_records(recs, synthetic.hf_cfg(cfg), None, 32, 32, 1e-6, 1e4, local, True,
                                        max_seq, 512, 16, rank, world, moe_map=recs.moe_map)
    model.init_tp()
    try:
        rng = np.random.default_rng(3)
        prefix = synthetic.prompt_ids(cfg, SHARED_PREFIX, seed=2)
        sfx = [[int(t) for t in rng.integers(0, cfg["vocab_size"], SHARED_SUFFIX)] for _ in range(SHARED_SEQS)]
        generate_shared_prefix(model, prefix[:256], sfx, max_tokens=4)  # warm every kernel shape
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        model.kv_truncate(0)
        model.forward(prefix, 0)
        torch.cuda.synchronize()
        prefill_s = time.perf_counter() - t0
        res = generate_shared_prefix(model, prefix, sfx, max_tokens=SHARED_TOKENS, timed=True)
        dt = res["decode_s"]
        if world > 1:
            t = torch.tensor([dt, prefill_s], dtype=torch.float64, device=f"cuda:{local}")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dt, prefill_s = float(t[0]), float(t[1])
        decoded = sum(len(t) - 1 for t in res["tokens"])  # tokens the timed decode steps produced
        if rank == 0:
            mlp = (f"virtual-MoE ({MOE_EXPERTS} experts of {cfg['intermediate_size'] // MOE_EXPERTS}, "
                   f"top-{MOE_TOP_K})" if args.moe else "dense")
            print(json.dumps({
                "bench": "shared_prefix_batch",
                "workload": f"llama2-7b-shape {mlp} int4 g64, fp16 KV, {SHARED_SEQS} sequences over a "
                            f"{SHARED_PREFIX}-token shared prefix + {SHARED_SUFFIX} own tokens, "
                            f"{SHARED_TOKENS} greedy tokens each",
                "n_gpus": world,
                "parallelism": f"tp{world}" + (f" attention, ep{world} experts" if args.moe and world > 1 else ""),
                "decode_tokens_per_s": decoded / dt, "ms_per_step": dt / max(1, res["steps"]) * 1e3,
                "steps": res["steps"], "sequences": SHARED_SEQS,
                "prefix_prefill_tokens_per_s": SHARED_PREFIX / prefill_s, "prefix_prefill_s": prefill_s,
                "timing": "wall clock around synchronous engine calls (bias build, every row's logits to the "
                          "host included), max over ranks"}), flush=True)
    finally:
        model.close()
        if world > 1:
            dist.destroy_process_group()
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--sweep", action="store_true",
                    help="GEMV sweep over bit widths x 7B shapes x batch 1/4/16 (JSON line per case)")
    ap.add_argument("--tiny", action="store_true",
                    help="the reference's CPU-runnable tiny config: decode tok/s, generate e2e, CPU baseline")
    ap.add_argument("--verify", action="store_true",
                    help="EAGLE tree verification (4096-token prompt, 32-node tree) and prefill rate")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="b200", choices=("b200", "reference"))
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (development only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--shared-prefix", action="store_true",
                    help="8 sequences over a 2048-token shared prefix, 128 greedy tokens each (with --moe: "
                         "the virtual-MoE shape; --gpus N: TP attention, expert-parallel experts)")
    ap.add_argument("--moe", action="store_true",
                    help="the virtual-MoE 7B shape (8 experts x 1376, top-2) instead of the dense model")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    from lumina_b200 import synthetic
    cfg = dict(synthetic.LLAMA7B)
    if args.layers:
        cfg["num_hidden_layers"] = args.layers
    if args.impl == "reference":
        return run_reference(args, cfg)
    if args.sweep:
        return run_sweep(args)
    if args.verify:
        return run_verify(args)
    if args.shared_prefix:
        return run_shared(args, cfg)
    if args.tiny:
        return run_tiny(args)

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device(f"cuda:{local}"))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    from lumina_b200.engine import CudaChatModel, make_pick
    max_seq = max(4608, PROMPT + max(args.warmup, args.steps) + 16)
    moe = (MOE_EXPERTS, MOE_TOP_K) if args.moe else None
    recs = synthetic.QuantizedRecords(cfg, bits=4, group=64, seed=0, device=local, moe=moe)
    t0 = time.perf_counter()
    model = CudaChatModel._from_records(recs, synthetic.hf_cfg(cfg), None, 32, 32, 1e-6, 1e4, local, True,
                                        max_seq, 512, 16, rank, world, moe_map=recs.moe_map)
    build_s = time.perf_counter() - t0
    model.init_tp()
    try:
        prompt = synthetic.prompt_ids(cfg, PROMPT, seed=0)
        lg = model.forward(prompt, 0)[0]
        first = int(np.argmax(lg.astype(np.float64)))
        # warm-up: W chained steps (captures the step graph), then back to the prompt
        model.decode_greedy(first, args.warmup)
        model.kv_truncate(PROMPT)
        clocks = ClockSampler(local)
        barrier()
        torch.cuda.synchronize()
        clocks.start()
        toks, dev_ms, kernels = model.decode_greedy(first, args.steps, timed=True)
        torch.cuda.synchronize()
        barrier()
        clk = clocks.stop()
        dev_ms = max_over_ranks(dev_ms)
        value = args.steps / (dev_ms / 1e3)

        # e2e: the public per-token call with host buffers, greedy host pick
        model.kv_truncate(PROMPT)
        pick = make_pick()
        model.decode_step(first, want_logits=True)  # warm the per-token graph
        model.kv_truncate(PROMPT)
        barrier()
        lg, tok, e2e_toks = None, first, []
        t0 = time.perf_counter()
        for i in range(args.steps):
            lg, _ = model.decode_step(tok)
            tok = pick(lg, e2e_toks)
            e2e_toks.append(tok)
        e2e_s = max_over_ranks(time.perf_counter() - t0)
        barrier()
        # both loops decode the same greedy sequence
        same = toks == e2e_toks
        h2d = 32 + 4 + 4          # DevParams, row position, token
        d2h = model.vocab * 4 + 4 + 8 + 4  # logits, argmax, argmax key, fault word

        # decode attention alone (attnc_kernel, every layer) at the prompt's
        # KV length and at the 4096 rows of the tree-speculation workload
        attn = {}
        peak_a, _ = peaks()
        for T in (PROMPT, 4096):
            if model.kv_length() < T:
                extra = synthetic.prompt_ids(cfg, T, seed=1)[model.kv_length():T]
                model.forward(extra, model.kv_length())
            model.kv_truncate(T)
            torch.cuda.nvtx.range_push(f"attention_T{T}")  # ncu --nvtx-include "attention_T4096/"
            ms_a, by_a = model.profile_attention(4)
            torch.cuda.nvtx.range_pop()
            attn[f"T{T}"] = {"us_per_launch": ms_a * 1e3, "bytes_per_launch": by_a,
                             "GB/s": by_a / (ms_a * 1e-3) / 1e9, "frac": by_a / (ms_a * 1e-3) / 1e9 / peak_a}
        model.kv_truncate(PROMPT)

        # roofline of the dominant kernel (packed GEMV), replayed alone
        ms_launch, launches, alg_bytes = model.profile_gemv(4)
        per_launch = alg_bytes / launches
        achieved = per_launch / (ms_launch * 1e-3) / 1e9
        peak, peak_kind = peaks()
        ratio, tsrc = traffic_ratio()
        kv_mean = PROMPT + args.steps / 2
        tok_bytes = alg_bytes + model.vocab // world * 4096 * 2 + KV_BYTES_PER_ROW // world * kv_mean
        if args.moe:
            # the touched experts' gate/up/down codes + fp16 scales, and the fp32 router
            ie, d = cfg["intermediate_size"] // MOE_EXPERTS, cfg["hidden_size"]
            # (per rank: a rank streams the picks among its E / N experts,
            # top_k / N of them on average)
            tok_bytes += cfg["num_hidden_layers"] * (MOE_TOP_K * 3 * ie * (d // 2 + d // 64 * 2) / world
                                                     + MOE_EXPERTS * d * 4)
        cb = None
        if world == 1 and not args.no_cpu_baseline and not args.moe:
            model.close()
            cb = cpu_baseline(cfg)
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": dev_ms / args.steps, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "int4 weights x int16 activations, int32 dot, f32",
                "data": "synthetic (seeded N(0,0.02) weights quantized to Lumina int4 g64; random prompt)",
                "config": workload(cfg, world, args.moe),
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "peak_kind": peak_kind,
                             "traffic": (ratio * per_launch) if ratio else None,
                             "traffic_source": tsrc,
                             "kernel": f"gemv_tc_kernel (tensor-pipe int4 dequant GEMV: one token's {launches} "
                                       "packed projections, RMSNorm prologues, store / SwiGLU epilogues)",
                             "algorithmic_bytes_per_launch": per_launch, "ms_per_launch": ms_launch},
                "cpu_baseline": cb,
                "e2e": {"value": args.steps / e2e_s, "unit": UNIT, "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h, "api": "CudaChatModel.decode_step + host greedy pick",
                        "same_tokens_as_chained": same},
                "attention": attn,
                "clocks": clk, "gpu_launches": kernels * args.steps, "kernels_per_step": kernels,
                "token_hbm_bytes": tok_bytes, "token_hbm_frac": tok_bytes / (dev_ms / args.steps * 1e-3) / 1e9 / peak,
                "model_build_s": build_s}
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        model.close()
        if world > 1:
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
