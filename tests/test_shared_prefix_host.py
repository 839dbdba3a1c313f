"""Host logic of engine.generate_shared_prefix on the CPU, against a fake
model that records every forward: the prefix is prefilled once at position
0; each row of a later forward sits at its own sequence's next position and
its bias admits the prefix (0), its sequence's cached rows (+1, whatever
their cache index), its sequence's rows of the same forward up to itself
(0), and nothing else (-inf); suffix forwards hold at most 64 rows; each
sequence's tokens are the argmaxes of its own rows."""
import numpy as np
import pytest

from lumina_b200.engine import generate_shared_prefix

V = 97


class FakeModel:
    max_rows = 128

    def __init__(self):
        self.len = 0
        self.calls = []

    def kv_length(self):
        return self.len

    def kv_truncate(self, n):
        self.len = n

    def forward(self, tokens, pos0, all_rows=False, pos_override=None, attn_bias=None):
        tokens = list(tokens)
        assert pos0 == self.len
        self.calls.append((tokens, pos0, None if pos_override is None else np.array(pos_override),
                           None if attn_bias is None else np.array(attn_bias)))
        self.len += len(tokens)
        rows = len(tokens) if all_rows else 1
        out = np.zeros((rows, V), np.float32)
        src = tokens if all_rows else tokens[-1:]
        for i, t in enumerate(src):
            out[i, (7 * t + 3) % V] = 1.0  # next token = (7t + 3) mod V
        return out


def _expect(first_tok, n):
    out, t = [], first_tok
    for _ in range(n):
        t = (7 * t + 3) % V
        out.append(t)
    return out


@pytest.mark.parametrize("lens", [(3, 5, 1), (16,) * 8, (1, 2)])
def test_bias_positions_and_tokens(lens):
    rng = np.random.default_rng(len(lens))
    prefix = [int(t) for t in rng.integers(0, V, 11)]
    sfx = [[int(t) for t in rng.integers(0, V, L)] for L in lens]
    steps = 5
    m = FakeModel()
    res = generate_shared_prefix(m, prefix, sfx, max_tokens=steps)
    P, B = len(prefix), len(sfx)
    # prefix once, plain
    toks0, pos0, po0, b0 = m.calls[0]
    assert toks0 == prefix and pos0 == 0 and po0 is None and b0 is None
    # the rows' sequences in the driver's order: the suffixes in sequence
    # order (forwards of at most 64 rows), then one row per sequence a step
    order = [b for b in range(B) for _ in sfx[b]]
    forwards = [order[c:c + 64] for c in range(0, len(order), 64)] + [list(range(B))] * (steps - 1)
    assert len(m.calls) == 1 + len(forwards)
    owner, nxt_pos = [], [P] * B
    for (toks, start, po, bias), seqs in zip(m.calls[1:], forwards):
        n = len(seqs)
        assert len(toks) == n and start == P + len(owner) and bias.shape == (n, start + n)
        for i, b in enumerate(seqs):
            row = bias[i]
            assert np.all(row[:P] == 0.0)                      # the prefix
            for k, ob in enumerate(owner):                      # cached rows: +1 own, -inf others
                assert row[P + k] == (1.0 if ob == b else -np.inf), (i, k)
            for j, sb in enumerate(seqs):                       # this forward: own rows up to itself
                assert row[start + j] == (0.0 if j <= i and sb == b else -np.inf), (i, j)
            assert po[i] == nxt_pos[b]
            nxt_pos[b] += 1
        owner += seqs
    for b, s in enumerate(sfx):
        assert res["tokens"][b] == _expect(s[-1], steps)
        assert int(np.argmax(res["first_logits"][b])) == (7 * s[-1] + 3) % V


def test_rejects_empty_and_too_many():
    m = FakeModel()
    with pytest.raises(Exception):
        generate_shared_prefix(m, [1, 2], [[3], []])
    with pytest.raises(Exception):
        generate_shared_prefix(m, [1, 2], [[3]] * 65)
    with pytest.raises(Exception):
        generate_shared_prefix(m, [1, 2], [[3]], max_tokens=0)
