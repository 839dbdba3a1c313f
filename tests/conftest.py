import os
import sys

import numpy as np
import pytest

REPO = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
for p in (REPO, os.path.join(REPO, "lumina-studio_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 and the built CUDA library")


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return np.load(os.path.join(GOLDEN, name), allow_pickle=False)
    return load


@pytest.fixture(scope="session")
def tiny_file(tmp_path_factory):
    """The tiny int4 g64 model, quantized by the oracle and written by the
    oracle writer (byte-identical to the reference-written file; pinned by
    test_oracle_golden.py)."""
    from oracle.quant import convert_arrays
    from oracle.lumina_format import write_lumina
    from lumina_b200 import synthetic
    w = synthetic.host_weights(synthetic.TINY, seed=0)
    payloads = convert_arrays(w, "int4", group_size=64, fp16_scales=True)
    path = str(tmp_path_factory.mktemp("tiny") / "tiny.lumina")
    write_lumina(path, payloads, name="tiny", rung="int4", group_size=64)
    return path


MOE_GOLDEN = {"experts": 8, "top_k": 2, "router_std": 0.1}  # tests/golden/make_golden.py MOE


@pytest.fixture(scope="session")
def tiny_moe_file(tmp_path_factory):
    """The tiny model with every MLP split into 8 routed experts (top-2),
    quantized by the oracle and written by the oracle writer with the
    virtual_moe header entry the reference's writer stores."""
    from oracle.quant import convert_arrays
    from oracle.lumina_format import write_lumina
    from lumina_b200 import synthetic
    w, meta = synthetic.virtual_moe_weights(synthetic.TINY, MOE_GOLDEN["experts"], MOE_GOLDEN["top_k"], seed=0,
                                            router_std=MOE_GOLDEN["router_std"])
    payloads = convert_arrays(w, "int4", group_size=64, fp16_scales=True)
    path = str(tmp_path_factory.mktemp("tiny_moe") / "tiny_moe.lumina")
    write_lumina(path, payloads, name="tiny_moe", rung="int4", group_size=64,
                 extra_header={"virtual_moe": meta})
    return path


@pytest.fixture(scope="session")
def wide_payloads():
    """The 7B decode shape cut to two layers (synthetic.LLAMA7B_2L) as int4
    g64 payloads with uniform codes and fp16-valued scales; the reference
    decoded the same records for tests/golden/wide_decode.npz."""
    from lumina_b200 import synthetic
    return synthetic.random_int4_payloads(synthetic.LLAMA7B_2L, seed=0)


@pytest.fixture(scope="session")
def wide_oracle(wide_payloads):
    """OracleModel over the wide payloads, dequantized as the reference's
    loader does (fp64 product rounded to fp32, adapters/lumina.py:135-139)."""
    from oracle import lumina_format as lf
    from oracle.decode import OracleModel
    from lumina_b200 import synthetic
    t = {}
    for name, (kind, payload) in wide_payloads.items():
        t[name] = payload if kind == "raw" else lf.dequant(kind, payload[0], payload[1], 64)
    cfg = synthetic.LLAMA7B_2L
    return OracleModel(t, synthetic.hf_cfg(cfg), theta=cfg["rope_theta"])
