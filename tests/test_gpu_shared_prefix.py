"""Several sequences over one shared prefix (engine.generate_shared_prefix):
the prefix is prefilled once, the sequences' rows sit side by side in one KV
cache, and each decode step is one forward of all live sequences with an
attention bias that keeps every row to the prefix and its own sequence.
Every sequence must reproduce what the single-sequence path gives for its
own prompt: the logits after the prompt and the greedy tokens. The dense
tiny model and its virtual-MoE variant (routed layers at several rows)."""
import numpy as np
import pytest

from lumina_b200 import synthetic

pytestmark = pytest.mark.gpu

# the logits bar of the parity tests against the reference: a single prompt
# of 33+ rows runs its projections on the tcgen05 GEMM (fp16 activations,
# about 3e-4), the shared path's few suffix rows on the int16-activation
# batched GEMV (about 5e-5)
LOGITS_BAR = 2e-3


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


class StubTok:
    def encode(self, p):
        return [int(t) for t in p]

    def decode(self, ids):
        return " ".join(map(str, ids))


def _check(path, n_seq, max_tokens):
    import torch
    assert torch.cuda.is_available()
    from lumina_b200.engine import CudaChatModel, generate_shared_prefix
    rng = np.random.default_rng(11)
    vocab = synthetic.TINY["vocab_size"]
    prefix = [int(t) for t in rng.integers(0, vocab, 40)]
    suffixes = [[int(t) for t in rng.integers(0, vocab, L)] for L in (3, 5, 1, 2, 4, 1, 6, 2)[:n_seq]]
    m = CudaChatModel.from_lumina(path, synthetic.hf_cfg(synthetic.TINY), StubTok(),
                                  theta=synthetic.TINY["rope_theta"], max_seq=512, max_rows=128)
    try:
        res = generate_shared_prefix(m, prefix, suffixes, max_tokens=max_tokens)
        for b, s in enumerate(suffixes):
            m.kv_truncate(0)
            lg = m.forward(prefix + s, 0)[0]
            assert rel_l2(res["first_logits"][b], lg) < LOGITS_BAR, b
            first = int(np.argmax(lg))
            want = [first] + m.decode_greedy(first, max_tokens - 1)
            assert res["tokens"][b] == want, b
    finally:
        m.close()


def test_shared_prefix_dense_matches_single_sequences(tiny_file):
    _check(tiny_file, 8, 10)


def test_shared_prefix_moe_matches_single_sequences(tiny_moe_file):
    _check(tiny_moe_file, 3, 8)
