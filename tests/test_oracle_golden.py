"""Pin the CPU oracle against golden vectors produced by the reference itself
(tests/golden/make_golden.py). CPU only."""
import hashlib
import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import lumina_format as lf
from oracle import quant, tops
from oracle.decode import (OracleModel, build_tree_mask, commit_rows, generate,
                           generate_cached, generate_spec, verify_tree)
from lumina_b200 import synthetic


def _sha(*arrs):
    h = hashlib.sha256()
    for a in arrs:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode() + str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


CASES = {
    "model.layers.0.a.weight": (37, 96, "int4", 64),
    "model.layers.0.b.weight": (16, 200, "int4", 64),
    "model.layers.0.c.weight": (17, 33, "int4", 64),
    "model.layers.0.d.weight": (20, 130, "int3", 64),
    "model.layers.1.e.weight": (24, 256, "int2", 128),
    "model.layers.1.f.weight": (19, 70, "int2", 128),
    "model.layers.1.g.weight": (24, 256, "binary", 128),
    "model.layers.1.h.weight": (21, 384, "binary", 128),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_quantizer_matches_reference(golden, name):
    g = golden("format_cases.npz")
    o, i, kind, gs = CASES[name]
    W = g[name + "|W"]
    if kind == "binary":
        codes, scales = quant.quantize_binary(W, gs)
    else:
        codes, scales = quant.quantize_int(W, int(kind[-1]), gs)
    assert np.array_equal(codes, g[name + "|codes"])
    assert np.array_equal(scales, g[name + "|scales"])


@pytest.mark.parametrize("group", [64, 128])
def test_writer_is_byte_identical(golden, tmp_path, group):
    g = golden("format_cases.npz")
    payloads = {}
    for name, (o, i, kind, gs) in CASES.items():
        if gs == group:
            payloads[name] = (kind, (g[name + "|codes"], g[name + "|scales"]))
    path = tmp_path / "w.lumina"
    lf.write_lumina(str(path), payloads, name="golden", rung="mixed", group_size=group)
    ref = open(os.path.join(GOLDEN, f"small_g{group}.lumina"), "rb").read()
    assert open(path, "rb").read() == ref


@pytest.mark.parametrize("group", [64, 128])
def test_loader_dequant_bit_exact(golden, group):
    g = golden("format_cases.npz")
    got = lf.load_dequant(os.path.join(GOLDEN, f"small_g{group}.lumina"))
    for name, (o, i, kind, gs) in CASES.items():
        if gs != group:
            continue
        ref = g[name + "|dequant"]
        assert got[name].dtype == np.float32 and got[name].shape == ref.shape
        assert np.array_equal(got[name].view(np.uint32), ref.view(np.uint32)), name


def test_pack_unpack_roundtrip():
    rng = np.random.default_rng(1)
    for (o, i) in [(1, 1), (3, 7), (5, 64), (2, 131)]:
        c4 = rng.integers(0, 16, (o, i))
        assert np.array_equal(lf.unpack_codes(lf.pack_codes_nibble(c4).tobytes(), (o, i), "nibble"), c4)
        c2 = rng.integers(0, 4, (o, i))
        assert np.array_equal(lf.unpack_codes(lf.pack_codes_2bit(c2).tobytes(), (o, i), "2bit"), c2)
        s = np.where(rng.standard_normal((o, i)) >= 0, 1.0, -1.0)
        assert np.array_equal(lf.unpack_signs(lf.pack_signs(s), i), s)
    with pytest.raises(ValueError):
        lf.unpack_codes(b"\x00" * 5, (2, 4), "nibble")


def test_tiny_quantization_matches_reference(golden):
    g = golden("tiny_decode.npz")
    w = synthetic.host_weights(synthetic.TINY, seed=0)
    payloads = quant.convert_arrays(w, "int4", group_size=64, fp16_scales=True)
    names = [str(n) for n in g["quant_sha_names"]]
    assert names == sorted(n for n, (k, _) in payloads.items() if k != "raw")
    for n, h in zip(names, g["quant_sha"]):
        codes, scales = payloads[n][1]
        assert _sha(codes.astype(np.uint8), scales) == str(h), n


def test_tiny_file_matches_reference(golden, tiny_file):
    g = golden("tiny_decode.npz")
    import json
    import struct
    raw = open(tiny_file, "rb").read()
    hlen = struct.unpack("<IIQ", raw[:16])[2]
    hdr = json.loads(raw[16:16 + hlen])
    digest = hashlib.sha256(json.dumps(hdr["tensors"]).encode() + raw[16 + hlen:]).hexdigest()
    assert digest == str(g["file_sha"])


@pytest.fixture(scope="module")
def tiny_model(tiny_file):
    return OracleModel(lf.load_dequant(tiny_file), synthetic.hf_cfg(synthetic.TINY),
                       theta=synthetic.TINY["rope_theta"])


def test_tiny_generate_matches_reference(golden, tiny_model):
    g = golden("tiny_decode.npz")
    prompt = [int(t) for t in g["prompt"]]
    toks, logits, _ = generate(tiny_model, prompt, 8, return_logits=True)
    assert toks == [int(t) for t in g["tokens"][:8]]
    np.testing.assert_allclose(logits[0], g["logits_prefill_last"], rtol=1e-5, atol=1e-7)


def test_tiny_teacher_forced_logits(golden, tiny_model):
    g = golden("tiny_decode.npz")
    m = tiny_model
    emb, head = m.embed(), m.head_t()
    cache = {}
    h = emb[np.array([int(t) for t in g["prompt"]])]
    for lyr in range(m.n_layer):
        h = m.layer(h, lyr, cache, 0)
    pos = h.shape[0]
    for s, tk in enumerate(int(t) for t in g["forced"]):
        hh = emb[[tk]]
        for lyr in range(m.n_layer):
            hh = m.layer(hh, lyr, cache, pos)
        pos += 1
        if f"logits_step{s}" in g:
            np.testing.assert_allclose((hh @ head)[0], g[f"logits_step{s}"], rtol=1e-5, atol=1e-7)


def test_prefix_cache_scenarios(golden, tiny_model):
    g = golden("tiny_decode.npz")
    P = {k: [int(t) for t in g[k]] for k in ("p1", "p2", "p3", "p4")}
    for k, n in (("r1", "p1"), ("r2", "p2"), ("r3", "p3"), ("r4", "p4")):
        nt = 6 if k == "r3" else 8
        assert generate(tiny_model, P[n], nt) == [int(t) for t in g[k]]
    st = {"ids": [], "kv": {}, "pos": 0}
    for j, (p, n) in enumerate(((P["p1"], 8), (P["p2"], 8), (P["p3"], 6), (P["p3"], 6), (P["p4"], 8))):
        toks, stats, st = generate_cached(tiny_model, p, n, state=st)
        assert toks == [int(t) for t in g[f"cached{j}_tokens"]]
        assert [stats["prefill_reused"], stats["prefill_computed"]] == list(g[f"cached{j}_stats"])


def test_spec_decode_matches_reference(golden, tiny_model):
    g = golden("tiny_spec.npz")
    toks, counts = generate_spec(tiny_model, [int(t) for t in g["prompt"]], 48, draft_n=4)
    assert toks == [int(t) for t in g["tokens"]]
    assert counts == [int(c) for c in g["counts"]]


def test_tree_mask_and_verify(golden, tiny_model):
    e = golden("tiny_eagle.npz")
    parents = [int(p) for p in e["parents"]]
    depths = [int(d) for d in e["depths"]]
    toks = [int(t) for t in e["toks"]]
    tm = build_tree_mask(parents)
    assert tm.shape == (len(parents), len(parents)) and (np.diag(tm) == 0).all()
    m = tiny_model
    emb = m.embed()
    cache = {}
    h = emb[np.array([int(t) for t in e["ids"]])]
    for lyr in range(m.n_layer):
        h = m.layer(h, lyr, cache, 0)
    pos = h.shape[0]
    lg, tc, _ = verify_tree(m, cache, pos, toks, parents, depths)
    assert np.array_equal(lg.argmax(axis=1), e["verify_argmax"])
    np.testing.assert_allclose(lg[:3], e["verify_logits_rows"], rtol=1e-5, atol=1e-7)
    # commit the greedy path rows and check the KV the reference committed
    order = [i for i in range(len(parents)) if depths[i] >= 1]
    gidx = {o: n for n, o in enumerate(order)}
    root = (h[-1:] @ m.head_t())[0]
    path, cur = [], 0
    while True:
        top = int(np.argmax(root if cur == 0 else lg[gidx[cur]]))
        kids = [i for i in range(1, len(toks)) if parents[i] == cur]
        nxt = next((i for i in kids if toks[i] == top), None)
        if nxt is None:
            break
        path.append(nxt)
        cur = nxt
    commit_rows(cache, tc, [gidx[i] for i in path])
    assert cache[0][0].shape[0] == int(e["kv_len"]) - 1  # bonus row appended by the next forward
    emb_b = emb[[int(e["accepted"][-1])]]
    hh = emb_b
    for lyr in range(m.n_layer):
        hh = m.layer(hh, lyr, cache, pos + len(path))
    np.testing.assert_allclose(hh, e["hidden_after"], rtol=1e-5, atol=1e-7)
    for lyr in range(m.n_layer):
        assert _sha(cache[lyr][0].astype(np.float32), cache[lyr][1].astype(np.float32)) == str(e["kv_sha"][lyr])


def test_tops_known_answers(golden):
    k = golden("tops_kat.npz")
    np.testing.assert_allclose(tops.ref_int8(k["xq"], k["xs"], k["wq"], k["ws"]), k["ref_int8"], rtol=1e-12)
    np.testing.assert_allclose(tops.ref_q4_0(k["xq"], k["xs"], k["q4"], k["q4s"]), k["ref_q4_0"], rtol=1e-12)
    xq, xs = tops.q8_repack(k["repack_x"])
    assert np.array_equal(xq, k["repack_xq"]) and np.array_equal(xs, k["repack_xs"])
    S, s, x = k["bin_S"], k["bin_s"], k["bin_x"]
    np.testing.assert_allclose(x @ (S.astype(np.float32) * s[:, None]).T, k["bin_y"], rtol=1e-6)


# ---------------------------------------------------------------------------
# virtual MoE (chat.py:285-299 -> qwen_next.py:31-78), tests/golden/tiny_moe.npz
# ---------------------------------------------------------------------------
def test_moe_quantization_matches_reference(golden):
    from conftest import MOE_GOLDEN
    g = golden("tiny_moe.npz")
    assert [int(v) for v in g["moe"]] == [MOE_GOLDEN["experts"], MOE_GOLDEN["top_k"]]
    assert float(g["router_std"]) == MOE_GOLDEN["router_std"]
    w, _ = synthetic.virtual_moe_weights(synthetic.TINY, MOE_GOLDEN["experts"], MOE_GOLDEN["top_k"], seed=0,
                                         router_std=MOE_GOLDEN["router_std"])
    payloads = quant.convert_arrays(w, "int4", group_size=64, fp16_scales=True)
    names = [str(n) for n in g["quant_sha_names"]]
    assert names == sorted(n for n, (k, _) in payloads.items() if k != "raw")
    assert "model.layers.0.mlp.experts.gate_up_proj" in names and "model.layers.0.mlp.gate.weight" not in names
    for n, h in zip(names, g["quant_sha"]):
        codes, scales = payloads[n][1]
        assert _sha(codes.astype(np.uint8), scales) == str(h), n


@pytest.fixture(scope="module")
def tiny_moe_model(tiny_moe_file):
    from lumina_b200.engine import moe_map_from_header
    hdr, _ = lf.read_header(tiny_moe_file)
    return OracleModel(lf.load_dequant(tiny_moe_file), synthetic.hf_cfg(synthetic.TINY),
                       theta=synthetic.TINY["rope_theta"], moe_map=moe_map_from_header(hdr))


def test_moe_oracle_matches_reference(golden, tiny_moe_model):
    g = golden("tiny_moe.npz")
    m = tiny_moe_model
    assert sorted(m.moe) == list(range(synthetic.TINY["num_hidden_layers"]))
    prompt = [int(t) for t in g["prompt"]]
    toks, logits, _ = generate(m, prompt, 16, return_logits=True)
    assert toks == [int(t) for t in g["tokens"]]
    np.testing.assert_allclose(logits[0], g["logits_prefill_last"], rtol=1e-5, atol=1e-7)
    emb, head = m.embed(), m.head_t()
    cache = {}
    h = emb[np.array(prompt)]
    for lyr in range(m.n_layer):
        h = m.layer(h, lyr, cache, 0)
    pos = h.shape[0]
    for s, tk in enumerate(int(t) for t in g["forced"]):
        hh = emb[[tk]]
        for lyr in range(m.n_layer):
            hh = m.layer(hh, lyr, cache, pos)
        pos += 1
        if f"logits_step{s}" in g:
            np.testing.assert_allclose((hh @ head)[0], g[f"logits_step{s}"], rtol=1e-5, atol=1e-7)


# ---------------------------------------------------------------------------
# the 7B decode width (head_dim 128, ffn 11008, vocab 32000), two layers:
# tests/golden/wide_decode.npz
# ---------------------------------------------------------------------------
def test_wide_records_match_reference(golden, wide_payloads):
    g = golden("wide_decode.npz")
    names = [str(n) for n in g["sha_names"]]
    assert names == sorted(wide_payloads)
    for n, h in zip(names, g["sha"]):
        kind, payload = wide_payloads[n]
        got = _sha(payload) if kind == "raw" else _sha(payload[0], payload[1])
        assert got == str(h), n


def test_wide_oracle_matches_reference(golden, wide_oracle):
    """The oracle's layer, head and greedy driver at 7B width agree with the
    reference's outputs (BLAS summation order may differ between hosts, so
    the bar is 1e-5 relative, not bit equality)."""
    g = golden("wide_decode.npz")
    m = wide_oracle
    emb, head = m.embed(), m.head_t()
    prompt = [int(t) for t in g["prompt"]]
    cache = {}
    h = emb[np.array(prompt)]

    def rel(a, b):
        return float(np.linalg.norm(np.float64(a) - b) / np.linalg.norm(np.float64(b)))

    for lyr in range(m.n_layer):
        h = m.layer(h, lyr, cache, 0)
        assert rel(h, g[f"hidden_prefill_l{lyr}"]) < 1e-5, lyr
    assert rel((h[-1:] @ head)[0], g["logits_prefill_last"]) < 1e-5
    pos = len(prompt)
    for s, tk in enumerate(int(t) for t in g["forced"]):
        hh = emb[[tk]]
        for lyr in range(m.n_layer):
            hh = m.layer(hh, lyr, cache, pos)
        pos += 1
        assert rel((hh @ head)[0], g[f"logits_step{s}"]) < 1e-5, s
    assert generate(m, prompt, len(g["tokens"])) == [int(t) for t in g["tokens"]]


def test_numba_gemv_int8_port_matches_reference_kernel():
    """The numba restatement of fused._gemv_int8 (the GEMV the CPU baseline
    times): bit-equal to the reference's own kernel on the KAT inputs, and
    within fp32 rounding of the int-exact ref_int8."""
    gemv = tops.numba_gemv_int8()
    if gemv is None:
        pytest.skip("numba not importable")
    g = np.load(os.path.join(GOLDEN, "tops_kat.npz"))
    out = np.empty(g["wq"].shape[0], np.float32)
    gemv(g["xq"], g["xs"], g["wq"], g["ws"], out)
    assert np.array_equal(out, g["numba_gemv_int8"])
    ref = g["ref_int8"]
    assert np.allclose(out, ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())
