"""The persistent decode step (one kernel per token, LUMINA_MEGAKERNEL=1):
same logits as the reference (2e-3 relative L2) on the recorded
teacher-forced steps, the same greedy tokens and KV rows as the multi-kernel
decode path of the same model."""
import numpy as np
import pytest

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
        return " ".join(map(str, ids))


def _model(tiny_file):
    from lumina_b200.engine import CudaChatModel
    return CudaChatModel.from_lumina(tiny_file, synthetic.hf_cfg(synthetic.TINY), StubTok(),
                                     theta=synthetic.TINY["rope_theta"], max_seq=512, max_rows=128)


def test_megakernel_step_and_chain(tiny_file, golden, monkeypatch):
    import torch
    assert torch.cuda.is_available()
    g = golden("tiny_decode.npz")
    prompt = [int(t) for t in g["prompt"]]
    ref = _model(tiny_file)  # the multi-kernel decode path
    monkeypatch.setenv("LUMINA_MEGAKERNEL", "1")
    mk = _model(tiny_file)
    try:
        # teacher-forced steps against the reference's own logits
        for m in (ref, mk):
            m.kv_truncate(0)
            m.forward(prompt, 0)
        for s, tk in enumerate(int(t) for t in g["forced"]):
            lg_mk, am = mk.decode_step(tk)
            lg_mk = lg_mk.copy()
            lg_ref, _ = ref.decode_step(tk)
            assert am == int(np.argmax(lg_mk))
            assert rel_l2(lg_mk, lg_ref) < 1e-4, s
            if f"logits_step{s}" in g:
                assert rel_l2(lg_mk, g[f"logits_step{s}"]) < REL_L2, s
        # device-chained greedy run from the prompt: tokens and KV rows
        n = 80
        for m in (ref, mk):
            m.kv_truncate(len(prompt) - 1)
        want = []
        tok = prompt[-1]
        for _ in range(n):
            _, tok = ref.decode_step(tok, want_logits=False)
            want.append(tok)
        got = mk.decode_greedy(prompt[-1], n)
        assert got == want
        T = len(prompt) - 1 + n
        assert mk.kv_length() == T
        for lyr in range(mk.n_layer):
            k1, v1 = mk.kv_read(lyr, 0, T)
            k0, v0 = ref.kv_read(lyr, 0, T)
            assert rel_l2(k1, k0) < 1e-4 and rel_l2(v1, v0) < 1e-4, lyr
        # the step is repeatable bit for bit
        mk.kv_truncate(len(prompt) - 1)
        again = mk.decode_greedy(prompt[-1], n)
        assert again == got
    finally:
        mk.close()
        ref.close()
