"""The host sampler (engine.make_pick, the reference's pick closure of
chat.py:330-378) on the CPU: the greedy-only fast path returns the index the
float64 path returns, ties included (the first maximum), and the repeat
penalty still goes through the full path."""
import numpy as np

from lumina_b200.engine import make_pick


def test_greedy_fast_path_matches_float64_argmax():
    rng = np.random.default_rng(0)
    pick = make_pick()
    assert pick.greedy
    for i in range(300):
        lg = rng.standard_normal(4096).astype(np.float32)
        if i % 3 == 0:  # exact ties at the maximum
            lg[rng.integers(0, lg.size, 4)] = lg.max()
        assert pick(lg, []) == int(np.argmax(np.asarray(lg, np.float64)))


def test_repeat_penalty_uses_the_full_path():
    lg = np.zeros(16, np.float32)
    lg[3], lg[7] = 2.0, 1.5
    assert make_pick()(lg, [3]) == 3
    # 2.0 / 1.5 < 1.5: the penalized token loses the argmax
    pick = make_pick(repeat_penalty=1.5)
    assert not pick.greedy
    assert pick(lg, [3]) == 7
