"""Host-side logic of the virtual-MoE path (CPU): the header map, the
layer detection rule, and the synthetic expert layout, which with every
expert picked reproduces the dense SwiGLU it was split from
(virtual_moe.py:140-147; qwen_next.py:31-78 with unit weights)."""
import numpy as np
import pytest

from lumina_b200 import synthetic
from lumina_b200.engine import moe_layers, moe_map_from_header
from oracle.decode import moe_grouped_forward


def test_header_map_is_keyed_by_layer():
    hdr = {"virtual_moe": {"model.layers.2.mlp.": {"experts": 8, "ie": 86, "top_k": 2},
                           "no_layer_here": {"experts": 1, "ie": 1, "top_k": 1}}}
    assert moe_map_from_header(hdr) == {2: {"experts": 8, "ie": 86, "top_k": 2}}
    assert moe_map_from_header({}) == {}


def test_experts_without_a_map_entry_are_an_error():
    recs = {"model.layers.1.mlp.experts.gate_up_proj": object()}
    with pytest.raises(KeyError, match="layer 1"):
        moe_layers(recs, 2, {})
    got = moe_layers(recs, 2, {"1": {"experts": 4, "ie": 10, "top_k": 2, "router_feat": "abs"}})
    assert got == {1: {"experts": 4, "ie": 10, "top_k": 2}}  # router_feat is dropped, as chat.py:181-183


def test_all_experts_reproduce_the_dense_mlp():
    cfg = dict(synthetic.TINY, num_hidden_layers=1)
    dense = synthetic.host_weights(cfg, seed=3)
    w, meta = synthetic.virtual_moe_weights(cfg, experts=8, top_k=8, seed=3)
    p = "model.layers.0.mlp."
    assert meta[p] == {"experts": 8, "ie": 86, "top_k": 8, "router_feat": "raw", "layer": "0"}
    assert w[p + "experts.gate_up_proj"].shape == (8 * 2 * 86, 256)
    assert w[p + "experts.down_proj"].shape == (8 * 86, 256)
    h = np.random.default_rng(0).standard_normal((3, 256)).astype(np.float32)
    g = h @ dense[p + "gate_proj.weight"].T
    u = h @ dense[p + "up_proj.weight"].T
    ref = ((g / (1.0 + np.exp(-np.clip(g, -40, 40)))) * u) @ dense[p + "down_proj.weight"].T
    out, info = moe_grouped_forward(h, w[p + "experts.gate_up_proj"].reshape(8, 172, 256),
                                    w[p + "experts.down_proj"].reshape(8, 86, 256), w[p + "gate.weight"], 8,
                                    router_b=w[p + "gate_bias"])
    assert sorted(info["experts"][0].tolist()) == list(range(8))
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-6)


def _device_topk(sc, k):
    """The device rule (moe.cu topk_row): descending score, ties to the
    lower expert index."""
    out, taken = [], set()
    for _ in range(k):
        best = None
        for e, v in enumerate(sc):
            if e not in taken and (best is None or v > sc[best]):
                best = e
        taken.add(best)
        out.append(best)
    return out


@pytest.mark.parametrize("E", [2, 4, 8, 16, 64])
def test_topk_rule_matches_numpy_argsort(E):
    """qwen_next.py:63 picks np.argsort(-scores)[:, :k]. Without ties the
    device rule gives the same experts in the same order. numpy's sort is not
    stable, so on exact score ties the reference's order is its sort
    algorithm's; the device takes the lower index, and both pick the same
    score values."""
    rng = np.random.default_rng(E)
    for _ in range(200):
        sc = rng.standard_normal(E).astype(np.float32)
        k = int(rng.integers(1, E + 1))
        assert _device_topk(sc.tolist(), k) == np.argsort(-sc[None], axis=1)[0, :k].tolist()
        tied = rng.choice(np.float32([0.25, 0.5, 0.75, 1.0]), size=E).astype(np.float32)
        dev = _device_topk(tied.tolist(), k)
        ref = np.argsort(-tied[None], axis=1)[0, :k]
        assert sorted(tied[dev].tolist()) == sorted(tied[ref].tolist())


def test_device_moe_arithmetic_equals_dequant_math():
    """The routed kernels never dequantize: gate/up use
    s/15 * (2 sum h c - 15 sum h) per 32-column chunk and down uses
    a * s * (2c - 15) / 15. Both equal the reference's dequant-then-multiply
    (adapters/lumina.py:135-139, qwen_next.py:69-75) up to fp32 rounding."""
    import kernel_model
    from oracle import lumina_format as lf
    rng = np.random.default_rng(11)
    Ie, D = 86, 256
    codes = rng.integers(0, 16, (2 * Ie, D))
    scales = (np.abs(rng.standard_normal((2 * Ie, D // 64))) * 0.02 + 1e-3).astype(np.float32)
    h = rng.standard_normal(D).astype(np.float32)
    W = lf.dequant("int4", codes.astype(np.uint8), scales, 64)
    np.testing.assert_allclose(kernel_model.moe_gate_up(codes, scales, h), W.astype(np.float64) @ h,
                               rtol=1e-5, atol=1e-6)
    dcodes = rng.integers(0, 16, (Ie, D))
    dscales = (np.abs(rng.standard_normal((Ie, D // 64))) * 0.02 + 1e-3).astype(np.float32)
    a = rng.standard_normal(Ie).astype(np.float32)
    Wd = lf.dequant("int4", dcodes.astype(np.uint8), dscales, 64)
    np.testing.assert_allclose(kernel_model.moe_down(dcodes, dscales, a), Wd.T.astype(np.float64) @ a,
                               rtol=1e-5, atol=1e-6)
