"""Bounded waits surface as errors, and the device stays usable.

The decode GEMVs stream weights into shared memory through bulk copies and
wait for them with bounded polls; a wait that gives up sets the device fault
word and the kernel returns (after letting its copies in flight land). This
file makes those waits give up without any fault: lumina_debug_wait_limit(0)
lets every wait poll zero times, so the first wait of each warp reports a
timeout while the copies themselves still complete. Each synchronous entry
must then return the timeout as an error, the asynchronous GEMV must leave it
in lumina_fault_status, and the next call with the default limit must succeed
with correct results (the word is cleared, not blamed on later calls)."""
import numpy as np
import pytest

from oracle import lumina_format as lf

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


@pytest.fixture
def zero_wait():
    from lumina_b200 import cuda
    cuda.ensure_device(0)
    cuda.fault_status(0, clear=True)
    cuda.debug_wait_limit(0)
    try:
        yield cuda
    finally:
        cuda.debug_wait_limit(-1)
        cuda.fault_status(0, clear=True)


@pytest.fixture(scope="module")
def tiny(tiny_file):
    import torch
    assert torch.cuda.is_available()
    from lumina_b200 import synthetic
    from lumina_b200.engine import CudaChatModel
    m = CudaChatModel.from_lumina(tiny_file, synthetic.hf_cfg(synthetic.TINY), StubTok(),
                                  theta=synthetic.TINY["rope_theta"], max_seq=256, max_rows=64)
    yield m
    m.close()


def test_forward_reports_timeout_then_recovers(tiny, golden, zero_wait):
    from lumina_b200.cuda import LuminaError
    g = golden("tiny_decode.npz")
    prompt = [int(t) for t in g["prompt"]]
    tiny.kv_truncate(0)
    # the prefill (tcgen05 projections) with waits that give up, then with
    # the default limit
    with pytest.raises(LuminaError, match="gemm_tc05_kernel"):
        tiny.forward(prompt[:-1], 0)
    zero_wait.debug_wait_limit(-1)
    tiny.kv_truncate(0)
    tiny.forward(prompt[:-1], 0)
    # one row: the tensor-pipe decode GEMV (gemv_tc_kernel) with waits that give up
    zero_wait.debug_wait_limit(0)
    with pytest.raises(LuminaError, match="gemv_tc_kernel"):
        tiny.forward(prompt[-1:], len(prompt) - 1)
    zero_wait.debug_wait_limit(-1)
    assert zero_wait.fault_status(0) == 0  # the failing call cleared the word
    tiny.kv_truncate(len(prompt) - 1)
    lg = tiny.forward(prompt[-1:], len(prompt) - 1)[0]
    assert rel_l2(lg, g["logits_prefill_last"]) < REL_L2


def test_layer_forward_reports_timeout(tiny, zero_wait):
    from lumina_b200.cuda import LuminaError
    tiny.kv_truncate(0)
    x = (np.random.default_rng(2).standard_normal((1, 256)) * 0.02).astype(np.float32)
    with pytest.raises(LuminaError, match="timed out"):
        tiny._layer(x, 0, tiny.kv, 0)
    zero_wait.debug_wait_limit(-1)
    tiny.kv_truncate(0)
    y = tiny._layer(x, 0, tiny.kv, 0)
    assert np.isfinite(y).all()
    tiny.kv_truncate(0)


@pytest.mark.parametrize("kind", ["int2", "binary"])
def test_async_gemv_leaves_fault_word(zero_wait, kind):
    """lumina_gemv (the CUDA-core decode GEMV, gemv_fused_kernel, at batch 1)
    is asynchronous: a timeout shows in lumina_fault_status; lumina_gemv_host
    returns it as its error; with the default limit both give the oracle's
    result and leave the word at zero."""
    import torch
    from lumina_b200.cuda import LuminaError, Weight
    cuda = zero_wait
    rows, cols, group = 512, 1024, 128
    rng = np.random.default_rng(4)
    if kind == "int2":
        codes = rng.integers(0, 4, (rows, cols)).astype(np.uint8)
        blob, pack = lf.pack_codes_2bit(codes), "2bit"
    else:
        blob, pack = lf.pack_signs(np.where(rng.standard_normal((rows, cols)) >= 0, 1.0, -1.0)), "none"
        codes = blob
    scales = (rng.random((rows, cols // group)) * 0.05 + 0.01).astype(np.float16).astype(np.float32)
    w = Weight.upload(kind, group, pack, blob, scales, rows, cols)
    Wd = lf.dequant(kind, codes, scales, group, cols)
    x = rng.standard_normal((1, cols)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty((1, rows), dtype=torch.float32, device="cuda")
    w.gemv(xd.data_ptr(), 1, cols, yd.data_ptr(), rows)
    torch.cuda.synchronize()
    assert cuda.fault_status(0, clear=False) & 1
    assert cuda.fault_status(0, clear=True) & 1
    assert cuda.fault_status(0) == 0
    with pytest.raises(LuminaError, match="timed out"):
        w.gemv_host(x)
    assert cuda.fault_status(0) == 0
    cuda.debug_wait_limit(-1)
    w.gemv(xd.data_ptr(), 1, cols, yd.data_ptr(), rows)
    torch.cuda.synchronize()
    assert cuda.fault_status(0) == 0
    assert rel_l2(yd.cpu().numpy(), x @ Wd.T) < REL_L2
    assert rel_l2(w.gemv_host(x), x @ Wd.T) < REL_L2


def test_gemm_rows_timeout(zero_wait, monkeypatch):
    """The tcgen05 multi-row projection: with waits that give up, bit 3 of
    the fault word is set and nothing hangs (the kernel still lets its TMA
    loads and MMAs land and frees its tensor memory); with the default limit
    the next call gives the reference math."""
    import torch
    from lumina_b200.cuda import Weight
    cuda = zero_wait
    monkeypatch.setenv("LUMINA_INT4_LAYOUT", "mma")
    rows, cols, group, M = 512, 1024, 64, 40
    rng = np.random.default_rng(6)
    codes = rng.integers(0, 16, (rows, cols)).astype(np.uint8)
    scales = (rng.random((rows, cols // group)) * 0.05 + 0.01).astype(np.float16).astype(np.float32)
    w = Weight.upload("int4", group, "nibble", lf.pack_codes_nibble(codes), scales, rows, cols)
    try:
        x = rng.standard_normal((M, cols)).astype(np.float32)
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty((M, rows), dtype=torch.float32, device="cuda")
        w.gemm_rows(xd.data_ptr(), M, cols, yd.data_ptr(), rows)
        torch.cuda.synchronize()
        assert cuda.fault_status(0) & 8
        cuda.debug_wait_limit(-1)
        w.gemm_rows(xd.data_ptr(), M, cols, yd.data_ptr(), rows)
        torch.cuda.synchronize()
        assert cuda.fault_status(0) == 0
        W16 = lf.dequant("int4", codes, scales, group).astype(np.float16).astype(np.float32)
        assert rel_l2(yd.cpu().numpy(), x @ W16.T) < REL_L2
    finally:
        w.free()
