"""GPU parity at the 7B decode width: d 4096, 32 heads x 128, ffn 11008,
vocab 32000, int4 g64, fp16 KV in 16-row pages -- the instantiations the 7B
decode bench runs (attnc_kernel<128, half>, the fp16 RoPE + paged-KV append
epilogue of the fused q/k/v GEMV, the hd-128 fp16 prefill attention, the
32000-row fp16 head with its fused argmax, the in-model q/k row permutation),
cut to two layers so that the oracle runs in seconds. The reference's own
outputs for this model are tests/golden/wide_decode.npz (the oracle is pinned
to them by test_oracle_golden.py); longer contexts are checked against the
oracle. Bar: 2e-3 relative L2 (chat.py:232-304 fp32 math against the device's
int16-activation integer dot)."""
import numpy as np
import pytest

from lumina_b200 import synthetic

pytestmark = pytest.mark.gpu

REL_L2 = 2e-3
CFG = synthetic.LLAMA7B_2L
D = CFG["hidden_size"]


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


class StubTok:
    def encode(self, p):
        return [int(t) for t in p]

    def decode(self, ids):
        return " ".join(str(i) for i in ids)


@pytest.fixture(scope="module")
def wide(wide_payloads, tmp_path_factory):
    """The model through the file path a user takes: the records written as
    a .lumina file (the oracle writer, byte-identical to the reference's),
    memory-mapped and uploaded packed by CudaChatModel.from_lumina."""
    import time
    import torch
    assert torch.cuda.is_available()
    from oracle.lumina_format import write_lumina
    from lumina_b200.engine import CudaChatModel
    path = str(tmp_path_factory.mktemp("wide") / "wide.lumina")
    write_lumina(path, wide_payloads, name="llama7b_2l", rung="int4", group_size=64)
    t0 = time.perf_counter()
    m = CudaChatModel.from_lumina(path, synthetic.hf_cfg(CFG), StubTok(), theta=CFG["rope_theta"],
                                  kv_fp16=True, max_seq=4160, max_rows=128, block_size=16)
    print("from_lumina of a 7B-width 2-layer file: %.2f s" % (time.perf_counter() - t0))
    yield m
    m.close()


def test_wide_logits_match_reference(wide, golden):
    g = golden("wide_decode.npz")
    prompt = [int(t) for t in g["prompt"]]
    wide.kv_truncate(0)
    lg = wide.forward(prompt, 0)[0]
    assert lg.shape == (CFG["vocab_size"],)
    assert rel_l2(lg, g["logits_prefill_last"]) < REL_L2
    for s, tk in enumerate(int(t) for t in g["forced"]):
        lg, am = wide.decode_step(tk)
        assert am == int(np.argmax(lg))
        assert rel_l2(lg, g[f"logits_step{s}"]) < REL_L2, s
    assert wide.kv_length() == len(prompt) + len(g["forced"])


def test_wide_greedy_tokens_match_reference(wide, golden, wide_oracle):
    from lumina_b200.engine import generate
    g = golden("wide_decode.npz")
    prompt = [int(t) for t in g["prompt"]]
    ref = [int(t) for t in g["tokens"]]
    got = generate(wide, prompt, max_tokens=len(ref))["tokens"]
    if got != ref:
        # tokens must match wherever the reference top-1 margin exceeds the tolerance
        k = next(i for i, (a, b) in enumerate(zip(got, ref)) if a != b)
        from oracle.decode import generate as ogen
        _, logits, _ = ogen(wide_oracle, prompt, k + 1, return_logits=True)
        lg = np.sort(logits[k].astype(np.float64))
        margin = (lg[-1] - lg[-2]) / np.linalg.norm(logits[k])
        assert margin < REL_L2, f"token {k} differs with reference margin {margin:.3g}"
    # the device-chained greedy loop gives the host-driven tokens
    wide.kv_truncate(0)
    wide.forward(prompt[:-1], 0)
    assert wide.decode_greedy(prompt[-1], len(ref)) == got


def _layer_chunked(model, x, lyr, pos0, chunk=128):
    out = np.empty_like(x)
    for c0 in range(0, x.shape[0], chunk):
        out[c0:c0 + chunk] = model._layer(x[c0:c0 + chunk], lyr, model.kv, pos0 + c0)
    return out


def test_wide_layer_dropin_matches_oracle(wide, wide_oracle):
    """_layer against the oracle's layer over appends that start at KV length
    0, 1, 18 and 512: a one-row decode on an empty cache (seven of the eight
    cluster CTAs own no key), a 17-row prefill across a page boundary, a
    494-row prefill in 128-row chunks, and a decode row at length 512 (eight
    64-key splits); then every fp16 K/V row against the oracle's fp32 rows."""
    rng = np.random.default_rng(21)
    wide.kv_truncate(0)
    cache = {}
    pos = 0
    for n in (1, 17, 494, 1):
        x = (rng.standard_normal((n, D)) * 0.5).astype(np.float32)
        want, got = x, x
        for lyr in range(wide.n_layer):
            want = wide_oracle.layer(want, lyr, cache, pos)
            got = _layer_chunked(wide, got, lyr, pos)
            assert rel_l2(got, want) < REL_L2, (n, pos, lyr)
        pos += n
    assert wide.kv_length() == pos == 513
    for lyr in range(wide.n_layer):
        k, v = wide.kv_read(lyr, 0, pos)
        ok, ov = cache[lyr]
        assert k.shape == ok.shape == (pos, 32, 128)
        # device rows are fp16: compare with the oracle's rows rounded to fp16
        assert rel_l2(k, ok.astype(np.float16)) < REL_L2, lyr
        assert rel_l2(v, ov.astype(np.float16)) < REL_L2, lyr
        assert np.array_equal(k, k.astype(np.float16).astype(np.float32))


@pytest.fixture(scope="module")
def long_context(wide):
    """4096 random prompt tokens prefilled on the device (32 chunks of 128)."""
    rng = np.random.default_rng(33)
    toks = [int(t) for t in rng.integers(0, CFG["vocab_size"], 4096)]
    return toks


def _prefill(wide, toks):
    if wide.kv_length() != len(toks):
        wide.kv_truncate(0)
        wide.forward(toks, 0)
    return len(toks)


def test_wide_decode_step_at_4096(wide, wide_oracle, long_context):
    """One graph-replayed decode step after a 4096-token prefill (the
    context length of the tree-speculation workload) against the oracle run
    on the device's own cached rows: the step's logits over the 32000-row
    head, its argmax, and the appended K/V rows."""
    T = _prefill(wide, long_context)
    cache = {}
    for lyr in range(wide.n_layer):
        cache[lyr] = wide.kv_read(lyr, 0, T)
    tok = 1234
    lg, am = wide.decode_step(tok)
    h = wide_oracle.embed()[[tok]]
    for lyr in range(wide.n_layer):
        h = wide_oracle.layer(h, lyr, cache, T)
    want = (h @ wide_oracle.head_t())[0]
    assert rel_l2(lg, want) < REL_L2
    assert am == int(np.argmax(lg))
    for lyr in range(wide.n_layer):
        k, v = wide.kv_read(lyr, T, 1)
        assert rel_l2(k, cache[lyr][0][T:].astype(np.float16)) < REL_L2, lyr
        assert rel_l2(v, cache[lyr][1][T:].astype(np.float16)) < REL_L2, lyr
    wide.kv_truncate(T)


def _tree_4x2():
    """A depth-5, 32-node draft tree: the root's 4 children, 2 children
    each, then single chains, plus 3 nodes at depth 5."""
    parents, depths, frontier = [-1], [0], [0]
    for b in (4, 2, 1, 1):
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


def test_wide_tree_verify_at_4096(wide, wide_oracle, long_context):
    """The tree verification forward of the tree-speculation workload (31
    child rows, ancestry bias, positions Lp - 1 + depth) over a 4096-token
    context: the projections split K over CTAs (31 rows fill too few tiles)
    and the attention splits its 65 key tiles; logits of every row and the
    children's K/V rows against the oracle's verify_tree on the device's own
    cached rows."""
    from lumina_b200.engine import verify_tree
    from oracle.decode import verify_tree as overify
    T = _prefill(wide, long_context)
    cache = {}
    for lyr in range(wide.n_layer):
        cache[lyr] = wide.kv_read(lyr, 0, T)
    parents, depths = _tree_4x2()
    rng = np.random.default_rng(8)
    ids = [long_context[-1]] + [int(t) for t in rng.integers(0, CFG["vocab_size"], len(parents) - 1)]
    try:
        lg, order = verify_tree(wide, T, ids, parents, depths)
        want, tc, _ = overify(wide_oracle, cache, T, ids, parents, depths)
        assert lg.shape == want.shape == (31, CFG["vocab_size"])
        for r in range(31):
            assert rel_l2(lg[r], want[r]) < REL_L2, r
        for lyr in range(wide.n_layer):
            k, v = wide.kv_read(lyr, T, 31)
            assert rel_l2(k, tc[lyr][0][T:].astype(np.float16)) < REL_L2, lyr
            assert rel_l2(v, tc[lyr][1][T:].astype(np.float16)) < REL_L2, lyr
        # a second verification gives the same bits (fixed split order)
        wide.kv_truncate(T)
        lg2, _ = verify_tree(wide, T, ids, parents, depths)
        assert np.array_equal(lg2.view(np.uint32), lg.view(np.uint32))
    finally:
        wide.kv_truncate(T)


@pytest.mark.parametrize("T", [4096, 4000, 512, 17, 1])
def test_wide_attention_kernel(wide, long_context, T):
    """attnc_kernel<128, half> alone (lumina_kv_attend) against numpy
    softmax(q K^T / sqrt(128)) V over the same paged fp16 rows, at key counts
    that split evenly and unevenly over the eight cluster CTAs."""
    _prefill(wide, long_context)
    wide.kv_truncate(T)
    try:
        rng = np.random.default_rng(T)
        for lyr in range(wide.n_layer):
            k, v = wide.kv_read(lyr, 0, T)
            q = rng.standard_normal((32, 128)).astype(np.float32)
            got = wide.kv_attend(lyr, q)
            s = np.einsum("hd,thd->ht", q.astype(np.float64), k.astype(np.float64)) / np.sqrt(128.0)
            p = np.exp(s - s.max(axis=1, keepdims=True))
            p /= p.sum(axis=1, keepdims=True)
            want = np.einsum("ht,thd->hd", p, v.astype(np.float64))
            assert rel_l2(got, want) < 1e-4, (T, lyr)
    finally:
        wide.kv_truncate(0)
