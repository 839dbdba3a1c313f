"""GPU parity of the decode path on the tiny Llama config (4 layers, d 256,
int4 g64, fp32 KV, theta 1e4) against the reference's own outputs (golden
vectors from tests/golden/make_golden.py) and the pinned oracle."""
import numpy as np
import pytest

from oracle import lumina_format as lf
from oracle.decode import OracleModel, commit_rows, verify_tree as oracle_verify
from lumina_b200 import synthetic

pytestmark = pytest.mark.gpu

REL_L2 = 2e-3


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


class StubTok:
    def encode(self, p):
        return [int(t) for t in p]

    def decode(self, ids):
        return " ".join(str(i) for i in ids)


@pytest.fixture(scope="module")
def model(tiny_file):
    import torch
    assert torch.cuda.is_available()
    from lumina_b200.engine import CudaChatModel
    m = CudaChatModel.from_lumina(tiny_file, synthetic.hf_cfg(synthetic.TINY), StubTok(),
                                  theta=synthetic.TINY["rope_theta"], max_seq=512, max_rows=128)
    yield m
    m.close()


@pytest.fixture(scope="module")
def oracle(tiny_file):
    return OracleModel(lf.load_dequant(tiny_file), synthetic.hf_cfg(synthetic.TINY),
                       theta=synthetic.TINY["rope_theta"])


def test_prefill_and_teacher_forced_logits(model, golden):
    g = golden("tiny_decode.npz")
    prompt = [int(t) for t in g["prompt"]]
    model.kv_truncate(0)
    lg = model.forward(prompt, 0)[0]
    assert rel_l2(lg, g["logits_prefill_last"]) < REL_L2
    assert model.kv_length() == len(prompt)
    for s, tk in enumerate(int(t) for t in g["forced"]):
        lg, am = model.decode_step(tk)
        assert am == int(np.argmax(lg))
        if f"logits_step{s}" in g:
            assert rel_l2(lg, g[f"logits_step{s}"]) < REL_L2, s
    assert model.kv_length() == len(prompt) + len(g["forced"])


def test_greedy_tokens_match_reference(model, golden, oracle):
    from lumina_b200.engine import generate
    g = golden("tiny_decode.npz")
    prompt = [int(t) for t in g["prompt"]]
    r = generate(model, prompt, max_tokens=128)
    ref = [int(t) for t in g["tokens"]]
    if r["tokens"] != ref:
        # tokens must match wherever the reference top-1 margin exceeds the tolerance
        k = next(i for i, (a, b) in enumerate(zip(r["tokens"], ref)) if a != b)
        from oracle.decode import generate as ogen
        _, logits, _ = ogen(oracle, prompt, k + 1, return_logits=True)
        lg = np.sort(logits[k].astype(np.float64))
        margin = (lg[-1] - lg[-2]) / np.linalg.norm(logits[k])
        assert margin < REL_L2, f"token {k} differs with reference margin {margin:.3g}"
    assert len(r["tokens"]) == 128


def test_prefix_cache_scenarios(model, golden):
    from lumina_b200.engine import generate, generate_cached
    g = golden("tiny_decode.npz")
    P = {k: [int(t) for t in g[k]] for k in ("p1", "p2", "p3", "p4")}
    for k, n in (("r1", "p1"), ("r2", "p2"), ("r3", "p3"), ("r4", "p4")):
        nt = 6 if k == "r3" else 8
        assert generate(model, P[n], nt)["tokens"] == [int(t) for t in g[k]]
    st = None
    for j, (p, n) in enumerate(((P["p1"], 8), (P["p2"], 8), (P["p3"], 6), (P["p3"], 6), (P["p4"], 8))):
        c = generate_cached(model, p, max_tokens=n, state=st)
        st = c["cache_state"]
        assert c["tokens"] == [int(t) for t in g[f"cached{j}_tokens"]], j
        assert [c["stats"]["prefill_reused"], c["stats"]["prefill_computed"]] == list(g[f"cached{j}_stats"]), j
        assert len(st["ids"]) == model.kv_length()


def test_generate_spec_matches_reference(model, golden):
    """Prompt-lookup speculative decoding (chat.generate_spec) on the device:
    the reference's tokens and its drafted / accepted / forward counts; the
    rollbacks are KV truncations, and the KV ends one row past the last
    accepted token as in the reference."""
    from lumina_b200.engine import generate_spec
    g = golden("tiny_spec.npz")
    prompt = [int(t) for t in g["prompt"]]
    r = generate_spec(model, prompt, max_tokens=48, draft_n=4)
    assert r["tokens"] == [int(t) for t in g["tokens"]]
    sp = r["spec"]
    assert [sp["drafted"], sp["accepted"], sp["target_forwards"], sp["tokens_out"]] == [int(c) for c in g["counts"]]
    assert sp["drafted"] > 0 and sp["accepted"] > 0


def test_kv_block_indexing_bit_exact(model):
    """Truncation and re-append land rows at the same page slots: decode
    steps repeated after a truncation (mid-page and on a page boundary)
    reproduce every KV row bit for bit (deterministic kernels)."""
    rng = np.random.default_rng(5)
    toks = [int(t) for t in rng.integers(0, 4096, 40)]
    model.kv_truncate(0)
    for t in toks:
        model.decode_step(t, want_logits=False)
    ref = [model.kv_read(l, 0, 40) for l in range(model.n_layer)]
    for cut in (13, 16, 0):
        model.kv_truncate(cut)
        for t in toks[cut:]:
            model.decode_step(t, want_logits=False)
        for l in range(model.n_layer):
            k, v = model.kv_read(l, 0, 40)
            assert np.array_equal(k, ref[l][0]) and np.array_equal(v, ref[l][1]), (cut, l)
    # chunked prefill across page boundaries agrees with one-row steps
    model.kv_truncate(0)
    for a, b in ((0, 1), (1, 17), (17, 32), (32, 40)):
        model.forward(toks[a:b], a)
    for l in range(model.n_layer):
        k, v = model.kv_read(l, 0, 40)
        # a row in the wrong page slot differs at O(1); chunked and one-row
        # forwards differ only in float summation order
        assert rel_l2(k, ref[l][0]) < 1e-3 and rel_l2(v, ref[l][1]) < 1e-3
    # commit gather: rows base+src[i] -> base+i
    before = [model.kv_read(l, 0, 40) for l in range(model.n_layer)]
    src = [3, 5, 9, 10]
    model.kv_commit_rows(20, src)
    assert model.kv_length() == 24
    for l in range(model.n_layer):
        k, v = model.kv_read(l, 0, 24)
        assert np.array_equal(k[:20], before[l][0][:20])
        for i, s in enumerate(src):
            assert np.array_equal(k[20 + i], before[l][0][20 + s])
            assert np.array_equal(v[20 + i], before[l][1][20 + s])


def test_layer_dropin_matches_oracle(model, oracle):
    rng = np.random.default_rng(8)
    x = (rng.standard_normal((5, 256)) * 0.02).astype(np.float32)
    model.kv_truncate(0)
    cache = {}
    want = x
    got = x
    for lyr in range(model.n_layer):
        want = oracle.layer(want, lyr, cache, 0)
        got = model._layer(got, lyr, model.kv, 0)
        assert rel_l2(got, want) < REL_L2, lyr
        k, v = model.kv[lyr]
        assert k.shape == cache[lyr][0].shape
        assert rel_l2(np.asarray(k), cache[lyr][0]) < REL_L2
    # one more row at pos 5, then the dict-style truncation of chat.py:442-445
    x1 = (rng.standard_normal((1, 256)) * 0.02).astype(np.float32)
    for lyr in range(model.n_layer):
        want = oracle.layer(x1 if lyr == 0 else want, lyr, cache, 5)
        got = model._layer(x1 if lyr == 0 else got, lyr, model.kv, 5)
    assert rel_l2(got, want) < REL_L2
    for lyr, (k, v) in list(model.kv.items()):
        model.kv[lyr] = (k[:3], v[:3])
    assert model.kv_length() == 3


def test_tree_verify_and_commit(model, golden, oracle):
    from lumina_b200.engine import commit_verified, verify_tree
    e = golden("tiny_eagle.npz")
    ids = [int(t) for t in e["ids"]]
    parents = [int(p) for p in e["parents"]]
    depths = [int(d) for d in e["depths"]]
    toks = [int(t) for t in e["toks"]]
    model.kv_truncate(0)
    root_lg = model.forward(ids, 0)[0]
    pos = len(ids)
    lg, order = verify_tree(model, pos, toks, parents, depths)
    assert np.array_equal(lg.argmax(axis=1), e["verify_argmax"])
    assert rel_l2(lg[:3], e["verify_logits_rows"]) < REL_L2
    gidx = {o: n for n, o in enumerate(order)}
    out = []
    done, pos2, lg2, last = commit_verified(model, pos, toks, parents, depths,
                                            lambda i: root_lg if i == 0 else lg[gidx[i]], 64, out)
    assert out == [int(t) for t in e["accepted"]]
    assert pos2 == int(e["pos_after"]) and not done
    assert model.kv_length() == int(e["kv_len"])
    want = (e["hidden_after"] @ oracle.head_t())[0]
    assert rel_l2(lg2, want) < REL_L2


def test_decode_greedy_chain_matches_steps(model):
    """The device-chained greedy loop (argmax fed back on the GPU) yields the
    same tokens and the same KV rows as host-driven decode steps, across the
    attention split boundaries (every 64 rows) and page boundaries."""
    rng = np.random.default_rng(12)
    prompt = [int(t) for t in rng.integers(0, 4096, 50)]
    n = 90
    model.kv_truncate(0)
    model.forward(prompt, 0)
    tok, ref = prompt[-1], []
    model.kv_truncate(len(prompt) - 1)
    for _ in range(n):
        _, tok = model.decode_step(tok, want_logits=False)
        ref.append(tok)
    kv_ref = [model.kv_read(l, 0, len(prompt) - 1 + n) for l in range(model.n_layer)]
    model.kv_truncate(len(prompt) - 1)
    got = model.decode_greedy(prompt[-1], n)
    assert got == ref
    assert model.kv_length() == len(prompt) - 1 + n
    for l in range(model.n_layer):
        k, v = model.kv_read(l, 0, len(prompt) - 1 + n)
        assert np.array_equal(k, kv_ref[l][0]) and np.array_equal(v, kv_ref[l][1]), l
    # a second chain continues from where the first stopped
    more = model.decode_greedy(got[-1], 5)
    model.kv_truncate(len(prompt) - 1 + n)
    tok, ref2 = got[-1], []
    for _ in range(5):
        _, tok = model.decode_step(tok, want_logits=False)
        ref2.append(tok)
    assert more == ref2
    from lumina_b200.cuda import LuminaError
    model.kv_truncate(0)
    with pytest.raises(LuminaError, match="capacity"):
        model.decode_greedy(1, 513)
    with pytest.raises(LuminaError):
        model.decode_greedy(1, 0)


def test_profile_gemv(model):
    ms, launches, nbytes = model.profile_gemv(2)
    assert launches == 4 * model.n_layer
    assert ms > 0
    # tiny config: 4 layers, d 256, ffn 688, int4 codes (half a byte per
    # weight) plus group scales, activations and outputs
    params = 4 * (4 * 256 * 256 + 3 * 688 * 256)
    assert 0.5 * params < nbytes < 0.75 * params


def test_model_errors(model):
    from lumina_b200.cuda import LuminaError
    with pytest.raises(LuminaError, match="out of range"):
        model.decode_step(10 ** 6)
    with pytest.raises(LuminaError):
        model.kv_truncate(10 ** 6)
    model.kv_truncate(0)
    with pytest.raises(LuminaError, match="capacity"):
        model.forward(list(range(513)), 0)
    model.kv_truncate(0)
