"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run in a container that holds the reference checkout (read-only is fine):

    python tests/golden/make_golden.py [--reference /root/reference]

It imports the reference's own quantizer (lumina_format.codecs.ptq_ladder),
writer (scripts/lumina_convert.py:write_lumina), loader
(lumina_framework.adapters.load_model), decode model and drivers
(lumina_framework.chat), tree verifier (lumina_framework.eagle / spec) and the
TOPS self-test references (lumina_framework.tops), runs them on seeded inputs
and stores their outputs. Nothing in the tests or on the GPU box reads the
reference; they read these fixtures.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, os.path.join(REPO, "lumina-studio_b200"))

from lumina_b200 import synthetic  # noqa: E402


class StubTok:
    """Token ids in, token ids out: the prompt *is* the id list."""

    def encode(self, prompt):
        return [int(t) for t in prompt]

    def decode(self, ids):
        return " ".join(str(int(i)) for i in ids)


def sha(*arrs) -> str:
    h = hashlib.sha256()
    for a in arrs:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode() + str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


FORMAT_CASES = {
    # name: (rows, cols, kind, group)
    "model.layers.0.a.weight": (37, 96, "int4", 64),
    "model.layers.0.b.weight": (16, 200, "int4", 64),
    "model.layers.0.c.weight": (17, 33, "int4", 64),
    "model.layers.0.d.weight": (20, 130, "int3", 64),
    "model.layers.1.e.weight": (24, 256, "int2", 128),
    "model.layers.1.f.weight": (19, 70, "int2", 128),
    "model.layers.1.g.weight": (24, 256, "binary", 128),
    "model.layers.1.h.weight": (21, 384, "binary", 128),
}


def make_format(ref, tmp):
    from lumina_format.codecs.ptq_ladder import quantize_binary, quantize_int
    from lumina_convert import write_lumina
    from lumina_framework.adapters import load_model

    rng = np.random.default_rng(7)
    out = {}
    for group in (64, 128):
        payloads, stats = {}, []
        for name, (o, i, kind, g) in FORMAT_CASES.items():
            if g != group:
                continue
            W = rng.standard_normal((o, i)) * 0.02
            if kind == "binary":
                q = quantize_binary(W, None, group_size=g)
            else:
                q = quantize_int(W, int(kind[-1]), None, group_size=g)
            payloads[name] = (q.kind, (q.codes, q.scales))
            out[name + "|W"] = W
            out[name + "|codes"] = np.asarray(q.codes)
            out[name + "|scales"] = np.asarray(q.scales)
        path = os.path.join(tmp, f"small_g{group}.lumina")
        write_lumina(path, payloads, stats, "golden", "mixed", group_size=group)
        shutil.copy(path, os.path.join(HERE, f"small_g{group}.lumina"))
        lm = load_model(path)
        for name in payloads:
            out[name + "|dequant"] = np.asarray(lm.tensors.tensors[name])
    np.savez_compressed(os.path.join(HERE, "format_cases.npz"), **out)
    print("format cases:", len(FORMAT_CASES))


def tiny_lumina(tmp):
    """Reference-quantized tiny model written and read by the reference."""
    from lumina_convert import convert_arrays, write_lumina
    from lumina_framework.adapters import load_model
    cfg = synthetic.TINY
    w = synthetic.host_weights(cfg, seed=0)
    payloads, stats = convert_arrays(w, {}, "int4", group_size=64)
    hashes = {}
    fixed = {}
    for name, (kind, payload) in payloads.items():
        if kind == "raw":
            fixed[name] = (kind, payload)
            continue
        codes, scales = payload
        scales = np.asarray(scales, dtype=np.float32).astype(np.float16).astype(np.float32)
        fixed[name] = (kind, (codes, scales))
        hashes[name] = sha(np.asarray(codes).astype(np.uint8), scales)
    path = os.path.join(tmp, "tiny.lumina")
    write_lumina(path, fixed, stats, "tiny", "int4", group_size=64)
    lm = load_model(path)
    return lm.tensors.tensors, hashes, path


def make_tiny(ref, tmp):
    from lumina_framework import chat
    from lumina_framework.chat import ChatModel, generate, generate_cached

    cfg = synthetic.TINY
    tensors, hashes, path = tiny_lumina(tmp)
    import json
    import struct
    raw = open(path, "rb").read()
    hlen = struct.unpack("<IIQ", raw[:16])[2]
    hdr = json.loads(raw[16:16 + hlen])
    # the tensor index and the blob area; the header's "matrices" list holds
    # the converter's float error statistics and is not part of the payload
    file_sha = hashlib.sha256(json.dumps(hdr["tensors"]).encode() + raw[16 + hlen:]).hexdigest()
    hcfg = synthetic.hf_cfg(cfg)
    model = ChatModel.from_tensors(tensors, hcfg, StubTok(), theta=cfg["rope_theta"])
    prompt = synthetic.prompt_ids(cfg, 64, seed=0)

    # logits of every step: wrap the head product through a probe of np.dot
    r = generate(model, prompt, max_tokens=128, rng=np.random.default_rng(0))
    toks = r["tokens"]

    # teacher-forced logits at a few steps, straight from the reference layer
    emb = model.t["model.embed_tokens.weight"].astype(np.float32)
    head_t = model.head.T.astype(np.float32)
    cache = {}
    h = emb[np.array(prompt)]
    for lyr in range(model.n_layer):
        h = model._layer(h, lyr, cache, 0)
    lg0 = (h[-1:] @ head_t)[0]
    hid0 = h.copy()
    pos = len(prompt)
    steps = {}
    forced = [int(t) for t in np.random.default_rng(9).integers(0, cfg["vocab_size"], 16)]
    for s, tk in enumerate(forced):
        hh = emb[[tk]]
        for lyr in range(model.n_layer):
            hh = model._layer(hh, lyr, cache, pos)
        pos += 1
        if s in (0, 7, 15):
            steps[s] = (hh @ head_t)[0]

    # prefix-cache scenarios (tests/test_prefix_cache.py:67-96 with id prompts)
    rng = np.random.default_rng(3)
    extra = lambda n: [int(t) for t in rng.integers(0, cfg["vocab_size"], n)]  # noqa: E731
    p1 = prompt[:40]
    r1 = generate(model, p1, max_tokens=8)["tokens"]
    p2 = p1 + r1 + extra(10)
    r2 = generate(model, p2, max_tokens=8)["tokens"]
    p4 = p2 + r2 + extra(6)
    r4 = generate(model, p4, max_tokens=8)["tokens"]
    p3 = p1[:5] + extra(20)
    r3 = generate(model, p3, max_tokens=6)["tokens"]
    st = {"ids": [], "kv": {}, "pos": 0}
    cached = []
    for p, n in ((p1, 8), (p2, 8), (p3, 6), (p3, 6), (p4, 8)):
        c = generate_cached(model, p, max_tokens=n, state=st)
        cached.append((c["tokens"], c["stats"]["prefill_reused"], c["stats"]["prefill_computed"]))

    out = {
        "prompt": np.array(prompt), "tokens": np.array(toks), "forced": np.array(forced),
        "logits_prefill_last": lg0.astype(np.float32),
        "hidden_prefill_sha": np.array(sha(hid0.astype(np.float32))),
        "file_sha": np.array(file_sha),
        "quant_sha_names": np.array(sorted(hashes)),
        "quant_sha": np.array([hashes[k] for k in sorted(hashes)]),
        "scenario_prompts": np.array([len(p1), len(p2), len(p3), len(p4)]),
        "p1": np.array(p1), "p2": np.array(p2), "p3": np.array(p3), "p4": np.array(p4),
        "r1": np.array(r1), "r2": np.array(r2), "r3": np.array(r3), "r4": np.array(r4),
    }
    for s, lg in steps.items():
        out[f"logits_step{s}"] = lg.astype(np.float32)
    for j, (tk, reused, computed) in enumerate(cached):
        out[f"cached{j}_tokens"] = np.array(tk)
        out[f"cached{j}_stats"] = np.array([reused, computed])
    np.savez_compressed(os.path.join(HERE, "tiny_decode.npz"), **out)
    print("tiny tokens[:8]", toks[:8], "file", file_sha[:12])
    return model, prompt


def make_eagle(ref, model, prompt):
    from lumina_framework.eagle import commit_verified, verify_tree
    from lumina_framework.spec import SpecStats

    cfg = synthetic.TINY
    emb = model.t["model.embed_tokens.weight"].astype(np.float32)
    head_t = model.head.T.astype(np.float32)
    ids = prompt[:40]
    cache = {}
    h = emb[np.array(ids)]
    for lyr in range(model.n_layer):
        h = model._layer(h, lyr, cache, 0)
    pos = len(ids)
    root_lg = (h[-1:] @ head_t)[0]
    # tree: root + 3 children, 2 grandchildren each, 2 great-grandchildren each
    parents, depths = [-1], [0]
    frontier = [0]
    for b in (3, 2, 2):
        nxt = []
        for p in frontier:
            for _ in range(b):
                parents.append(p)
                depths.append(depths[p] + 1)
                nxt.append(len(parents) - 1)
        frontier = nxt
    rng = np.random.default_rng(5)
    toks = [int(ids[-1])] + [int(t) for t in rng.integers(0, cfg["vocab_size"], len(parents) - 1)]
    # make the path 0 -> 2 -> (first child of 2) -> (its first child) greedy-accepted
    path = [0, 2]
    toks[2] = int(np.argmax(root_lg))
    order = [i for i in range(len(parents)) if depths[i] >= 1]
    gidx = {old: new for new, old in enumerate(order)}
    for _ in range(2):
        lg, tc, _h = verify_tree(model, cache, pos, toks, parents, depths)
        cur = path[-1]
        kid = [i for i in range(1, len(parents)) if parents[i] == cur][0]
        toks[kid] = int(np.argmax(lg[gidx[cur]]))
        path.append(kid)
    lg, tc, hv = verify_tree(model, cache, pos, toks, parents, depths)

    def cur_lg(i):
        return root_lg if i == 0 else lg[gidx[i]]

    st = SpecStats()
    out_toks: list = []
    cache_c = dict(cache)
    done, pos2, h2, last = commit_verified(model, cache_c, tc, pos, emb, toks, parents, depths,
                                           cur_lg, st, 64, out_toks, ())
    kv_sha = [sha(cache_c[l][0].astype(np.float32), cache_c[l][1].astype(np.float32))
              for l in range(model.n_layer)]
    res = {"ids": np.array(ids), "parents": np.array(parents), "depths": np.array(depths),
           "toks": np.array(toks), "verify_argmax": lg.argmax(axis=1),
           "verify_logits_rows": lg[:3].astype(np.float32),
           "verify_norms": np.linalg.norm(lg, axis=1).astype(np.float64),
           "accepted": np.array(out_toks), "pos_after": np.array(pos2),
           "hidden_after": np.asarray(h2, dtype=np.float32),
           "kv_sha": np.array(kv_sha), "kv_len": np.array(cache_c[0][0].shape[0])}
    np.savez_compressed(os.path.join(HERE, "tiny_eagle.npz"), **res)
    print("eagle accepted", out_toks, "pos", pos2)


def make_tops(ref):
    from lumina_framework import tops
    sys.path.insert(0, os.path.join(REPO))
    from oracle.tops import self_test_inputs
    d = self_test_inputs()
    out = dict(d)
    out["ref_int8"] = tops._ref_int8(d["xq"], d["xs"], d["wq"], d["ws"])
    out["ref_q4_0"] = tops._ref_q4_0(d["xq"], d["xs"], d["q4"], d["q4s"])
    # fused.q8_repack on a seeded activation (fused.py:91-102)
    from lumina_framework.fused import q8_repack
    x = np.random.default_rng(12).standard_normal(1000).astype(np.float32)
    xq, xs = q8_repack(x)
    out["repack_x"], out["repack_xq"], out["repack_xs"] = x, xq, xs
    # kernels.cpu_binary_gemv bit-exact case (tests/test_format_framework.py I2 shape)
    from lumina_framework.kernels import cpu_binary_gemv, pack_signs
    rng = np.random.default_rng(0)
    S = np.where(rng.standard_normal((64, 512)) >= 0, 1, -1).astype(np.int8)
    s = (np.abs(rng.standard_normal(64)) + 0.1).astype(np.float32)
    xb = rng.standard_normal((1, 512)).astype(np.float32)
    out["bin_S"], out["bin_s"], out["bin_x"] = S, s, xb
    out["bin_y"] = cpu_binary_gemv(xb, pack_signs(S), s, 512)
    # the numba kernel behind fused_gemv_int8 (fused.py:163-184) on the KAT inputs
    from lumina_framework import fused
    if not fused._HAS_NUMBA:
        raise SystemExit("numba is needed for the fused._gemv_int8 fixture")
    y = np.empty(d["wq"].shape[0], np.float32)
    fused._gemv_int8(d["xq"], d["xs"], d["wq"], d["ws"], y)
    out["numba_gemv_int8"] = y
    np.savez_compressed(os.path.join(HERE, "tops_kat.npz"), **out)
    print("tops KAT written")


MOE = {"experts": 8, "top_k": 2, "router_std": 0.1}  # tiny shape, every layer routed


def make_moe(ref, tmp):
    """Virtual-MoE decode (chat.py:285-299 -> qwen_next.moe_grouped_forward):
    the tiny model with every SwiGLU split into 8 experts (top-2), quantized
    by the reference's converter, written with its virtual_moe header entry,
    read back by the reference loader and decoded by ChatModel with the
    moe_map serve._api_load_lumina builds. Records the prefill and
    teacher-forced logits, 16 greedy tokens, the quantized-tensor hashes and
    the smallest top-k score gap over every routing decision (so the device
    test knows its routing margin)."""
    import json
    import re
    import struct
    from lumina_convert import convert_arrays, write_lumina
    from lumina_framework import qwen_next
    from lumina_framework.adapters import load_model
    from lumina_framework.chat import ChatModel, generate

    cfg = synthetic.TINY
    w, meta = synthetic.virtual_moe_weights(cfg, MOE["experts"], MOE["top_k"], seed=0,
                                            router_std=MOE["router_std"])
    payloads, stats = convert_arrays(w, {}, "int4", group_size=64)
    fixed, hashes = {}, {}
    for name, (kind, payload) in payloads.items():
        if kind == "raw":
            fixed[name] = (kind, payload)
            continue
        codes, scales = payload
        scales = np.asarray(scales, dtype=np.float32).astype(np.float16).astype(np.float32)
        fixed[name] = (kind, (codes, scales))
        hashes[name] = sha(np.asarray(codes).astype(np.uint8), scales)
    path = os.path.join(tmp, "tiny_moe.lumina")
    write_lumina(path, fixed, stats, "tiny_moe", "int4", group_size=64, moe_meta=meta)
    raw = open(path, "rb").read()
    hlen = struct.unpack("<IIQ", raw[:16])[2]
    hdr = json.loads(raw[16:16 + hlen])
    moe_map = {}
    for pfx, mm in (hdr.get("virtual_moe") or {}).items():  # serve.py:1357-1366
        mt = re.search(r"layers\.(\d+)\.", str(pfx))
        if mt:
            moe_map[int(mt.group(1))] = mm
    lm = load_model(path)
    model = ChatModel.from_tensors(lm.tensors.tensors, synthetic.hf_cfg(cfg), StubTok(),
                                   theta=cfg["rope_theta"], moe_map=moe_map)
    assert sorted(model.moe) == list(range(cfg["num_hidden_layers"]))

    gaps = []
    orig = qwen_next.moe_grouped_forward

    def probe(h, gate_up, down, router_w, top_k, **kw):
        lg = h @ router_w.T
        if kw.get("router_b") is not None:
            lg = lg + np.asarray(kw["router_b"], dtype=np.float32)
        sc = np.sort(qwen_next._sigmoid(lg), axis=1)[:, ::-1]
        gaps.append(float((sc[:, top_k - 1] - sc[:, top_k]).min()))
        return orig(h, gate_up, down, router_w, top_k, **kw)

    qwen_next.moe_grouped_forward = probe
    try:
        prompt = synthetic.prompt_ids(cfg, 24, seed=0)
        emb = model.t["model.embed_tokens.weight"].astype(np.float32)
        head_t = model.head.T.astype(np.float32)
        cache = {}
        h = emb[np.array(prompt)]
        for lyr in range(model.n_layer):
            h = model._layer(h, lyr, cache, 0)
        out = {"prompt": np.array(prompt), "logits_prefill_last": (h[-1:] @ head_t)[0].astype(np.float32)}
        pos = len(prompt)
        forced = [int(t) for t in np.random.default_rng(9).integers(0, cfg["vocab_size"], 8)]
        for s, tk in enumerate(forced):
            hh = emb[[tk]]
            for lyr in range(model.n_layer):
                hh = model._layer(hh, lyr, cache, pos)
            pos += 1
            if s in (0, 7):
                out[f"logits_step{s}"] = (hh @ head_t)[0].astype(np.float32)
        r = generate(model, prompt, max_tokens=16, rng=np.random.default_rng(0))
    finally:
        qwen_next.moe_grouped_forward = orig
    out.update({"forced": np.array(forced), "tokens": np.array(r["tokens"]),
                "min_route_gap": np.array(min(gaps)),
                "moe": np.array([MOE["experts"], MOE["top_k"]]), "router_std": np.array(MOE["router_std"]),
                "quant_sha_names": np.array(sorted(hashes)),
                "quant_sha": np.array([hashes[k] for k in sorted(hashes)])})
    np.savez_compressed(os.path.join(HERE, "tiny_moe.npz"), **out)
    print("moe tokens[:8]", r["tokens"][:8], "min route gap %.3g" % min(gaps))


def make_spec(ref, tmp):
    """Prompt-lookup speculative decoding (chat.generate_spec, chat.py:
    572-648) on the tiny model: a prompt whose tail repeats an earlier span
    (so the first drafts come from the prompt), 48 tokens, drafts of 4.
    Records the tokens and the SpecStats counters."""
    from lumina_framework.chat import ChatModel, generate_spec

    cfg = synthetic.TINY
    tensors, _, _ = tiny_lumina(tmp)
    model = ChatModel.from_tensors(tensors, synthetic.hf_cfg(cfg), StubTok(), theta=cfg["rope_theta"])
    p = synthetic.prompt_ids(cfg, 64, seed=0)
    prompt = p[:40] + p[8:20]
    r = generate_spec(model, prompt, max_tokens=48, draft_n=4, rng=np.random.default_rng(0))
    sp = r["spec"]
    out = {"prompt": np.array(prompt), "tokens": np.array(r["tokens"]),
           "counts": np.array([sp["drafted"], sp["accepted"], sp["target_forwards"], sp["tokens_out"]])}
    np.savez_compressed(os.path.join(HERE, "tiny_spec.npz"), **out)
    print("spec tokens[:8]", r["tokens"][:8], "drafted/accepted/forwards/out", out["counts"].tolist())


WIDE = {"seed": 0, "prompt": 17, "forced": 2, "greedy": 6}


def make_wide(ref, tmp):
    """The 7B decode shape (d 4096, 32 heads x 128, ffn 11008, vocab 32000)
    cut to two layers, int4 g64 (synthetic.random_int4_payloads: uniform
    codes, fp16-valued scales), written by the reference's writer, read by
    its loader and decoded by its ChatModel (theta 1e4). Records the hidden
    rows after each layer of a 17-row prefill, the last row's logits over the
    32000-row head, two teacher-forced decode steps' logits and six greedy
    tokens, plus hashes of every stored record."""
    from lumina_convert import write_lumina
    from lumina_framework.adapters import load_model
    from lumina_framework.chat import ChatModel, generate

    cfg = synthetic.LLAMA7B_2L
    payloads = synthetic.random_int4_payloads(cfg, seed=WIDE["seed"])
    hashes = {}
    for name, (kind, payload) in payloads.items():
        hashes[name] = sha(payload) if kind == "raw" else sha(payload[0], payload[1])
    path = os.path.join(tmp, "wide.lumina")
    write_lumina(path, payloads, [], "llama7b_2l", "int4", group_size=64)
    del payloads
    lm = load_model(path)
    model = ChatModel.from_tensors(lm.tensors.tensors, synthetic.hf_cfg(cfg), StubTok(), theta=cfg["rope_theta"])
    del lm
    prompt = synthetic.prompt_ids(cfg, WIDE["prompt"], seed=WIDE["seed"])
    emb = model.t["model.embed_tokens.weight"].astype(np.float32)
    head_t = model.head.T.astype(np.float32)
    cache = {}
    h = emb[np.array(prompt)]
    out = {"prompt": np.array(prompt)}
    for lyr in range(model.n_layer):
        h = model._layer(h, lyr, cache, 0)
        out[f"hidden_prefill_l{lyr}"] = h.astype(np.float32)
    out["logits_prefill_last"] = (h[-1:] @ head_t)[0].astype(np.float32)
    pos = len(prompt)
    forced = [int(t) for t in np.random.default_rng(9).integers(0, cfg["vocab_size"], WIDE["forced"])]
    for s, tk in enumerate(forced):
        hh = emb[[tk]]
        for lyr in range(model.n_layer):
            hh = model._layer(hh, lyr, cache, pos)
        pos += 1
        out[f"logits_step{s}"] = (hh @ head_t)[0].astype(np.float32)
    r = generate(model, prompt, max_tokens=WIDE["greedy"], rng=np.random.default_rng(0))
    out.update({"forced": np.array(forced), "tokens": np.array(r["tokens"]),
                "sha_names": np.array(sorted(hashes)),
                "sha": np.array([hashes[k] for k in sorted(hashes)])})
    np.savez_compressed(os.path.join(HERE, "wide_decode.npz"), **out)
    print("wide tokens", r["tokens"])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    ap.add_argument("--only", choices=("format", "tiny", "tops", "moe", "wide", "spec"), default=None,
                    help="regenerate one fixture family (tiny includes the EAGLE fixture)")
    args = ap.parse_args()
    ref = args.reference
    os.environ.setdefault("NUMBA_CACHE_DIR", tempfile.mkdtemp(prefix="numba_"))
    sys.path.insert(0, os.path.join(ref, "src"))
    sys.path.insert(0, os.path.join(ref, "scripts"))
    want = (lambda k: args.only in (None, k))  # noqa: E731
    with tempfile.TemporaryDirectory() as tmp:
        if want("format"):
            make_format(ref, tmp)
        if want("tiny"):
            model, prompt = make_tiny(ref, tmp)
            make_eagle(ref, model, prompt)
        if want("tops"):
            make_tops(ref)
        if want("moe"):
            make_moe(ref, tmp)
        if want("wide"):
            make_wide(ref, tmp)
        if want("spec"):
            make_spec(ref, tmp)


if __name__ == "__main__":
    main()
