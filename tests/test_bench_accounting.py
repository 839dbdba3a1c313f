"""bench.py's byte accounting and argument rules (CPU): the GEMV sweep's
bytes per call (7B shapes x int4/int3/int2/binary x batch 1/4/16), the
virtual-MoE records' shapes and map, the refusal of invalid timing
arguments, and the CPU baseline's whole-token sample."""
import numpy as np
import pytest

import bench
from lumina_b200 import synthetic


def test_sweep_bytes_formula():
    # N*K*b/8 codes + N*ceil(K/g)*2 fp16 scales + batch*K*4 in + batch*N*4 out
    assert bench.sweep_bytes(4096, 4096, 4, 64, 1) == 4096 * 2048 + 4096 * 64 * 2 + 4096 * 4 + 4096 * 4
    assert bench.sweep_bytes(4096, 11008, 3, 64, 4) == 4096 * 4128 + 4096 * 172 * 2 + 4 * 11008 * 4 + 4 * 4096 * 4
    assert bench.sweep_bytes(32000, 4096, 1, 128, 16) == 32000 * 512 + 32000 * 32 * 2 + 16 * 4096 * 4 + 16 * 32000 * 4


def test_sweep_covers_7b_shapes_kinds_and_batches():
    assert set(bench.SWEEP_SHAPES) == {(4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)}
    assert [k for k, _, _ in bench.SWEEP_KINDS] == ["int4", "int3", "int2", "binary"]
    assert bench.SWEEP_BATCHES == (1, 4, 16)


def test_moe_records_layout():
    cfg = dict(synthetic.LLAMA7B, num_hidden_layers=2)
    recs = synthetic.QuantizedRecords(cfg, moe=(bench.MOE_EXPERTS, bench.MOE_TOP_K))
    assert recs.moe_map == {0: {"experts": 8, "ie": 1376, "top_k": 2}, 1: {"experts": 8, "ie": 1376, "top_k": 2}}
    shapes = {n: s for n, (_, s) in recs.order.items()}
    assert shapes["model.layers.1.mlp.experts.gate_up_proj"] == (8 * 2 * 1376, 4096)
    assert shapes["model.layers.1.mlp.experts.down_proj"] == (8 * 1376, 4096)
    assert shapes["model.layers.1.mlp.gate.weight"] == (8, 4096)
    assert shapes["model.layers.1.mlp.gate_bias"] == (8,)
    assert not any(".mlp.gate_proj." in n or ".mlp.down_proj." in n for n in shapes)
    # the routed MLP moves a quarter of the dense one's packed bytes at top-2 of 8
    dense = 3 * 11008 * 4096
    touched = bench.MOE_TOP_K * 3 * 1376 * 4096
    assert touched * 4 == dense


def test_warmup_floor():
    with pytest.raises(SystemExit):
        bench.main(["--warmup", "2", "--impl", "reference"])
    with pytest.raises(SystemExit):
        bench.main(["--moe", "--gpus", "2"])


def test_cpu_gemv_leg_times_and_memoises():
    cache = {}
    t = bench.cpu_gemv_us(256, 512, 4, cache)
    assert t > 0 and cache == {(256, 512, 4): t}
    assert bench.cpu_gemv_us(256, 512, 4, cache) == t


def test_cpu_sample_runs_every_layer_over_distinct_weight_sets():
    """The CPU baseline's step is one whole token: every layer and the head.
    Layers l and l + 4 share one fp32 weight set, neighbouring layers do
    not, so a set is re-read from DRAM only after the other sets' bytes
    have streamed through the caches; the step's token is the argmax of the
    head over the last layer's output."""
    cfg = dict(synthetic.TINY, num_hidden_layers=6)
    s = bench.CpuDecodeSample(cfg, weight_sets=4)
    w = s.m._wcache
    q = [w[f"model.layers.{l}.self_attn.q_proj.weight"] for l in range(6)]
    assert q[0] is q[4] and q[1] is q[5]
    assert len({id(a) for a in q[:4]}) == 4
    assert not any(np.shares_memory(a, b) for a in q[:4] for b in q[:4] if a is not b)
    assert np.array_equal(q[0], q[1])  # equal values, distinct memory
    tok0, pos0 = s.tok, s.pos
    cache = {l: tuple(np.array(a, copy=True) for a in s.cache[l]) for l in range(6)}
    h = s.emb[[tok0]]
    for l in range(6):
        h = s.m.layer(h, l, cache, pos0)
    want = int(np.argmax((h[-1:] @ s.head_t)[0].astype(np.float64)))
    dt = s.step()
    assert dt > 0 and s.pos == pos0 + 1 and s.tok == want
    assert "all 6" in s.describe(1) and "4 distinct weight sets" in s.describe(1)


def test_numba_leg_reports_failure_as_unavailable(monkeypatch):
    """The numba GEMV leg sits beside the decode baseline: an error inside it
    (numba missing or failing on the host) becomes an "unavailable" entry,
    never an exception that would lose the bench line."""
    def broken():
        raise RuntimeError("no jit here")
    monkeypatch.setattr(bench, "cpu_numba_gemv", broken)
    got = bench.numba_leg()
    assert got == {"unavailable": "RuntimeError: no jit here"}
