"""GPU parity: packed-weight upload, bit-exact unpack / dequant gates, the
fused dequant GEMV of every kind, and the TOPS-semantics int8 family.
All calls go through the C ABI (ctypes)."""
import os

import numpy as np
import pytest

import kernel_model
from conftest import GOLDEN
from oracle import lumina_format as lf
from oracle import tops as otops

pytestmark = pytest.mark.gpu

REL_L2 = 2e-3     # GEMV / logits tolerance vs the reference math (fp32 accumulate)
TIGHT = 2e-6      # vs the exact model of the device arithmetic


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from lumina_b200 import cuda
    cuda.ensure_device(0)  # self-test must pass
    return torch


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def ref_gemv(x, W):
    """The reference's GEMV: fp32 x @ fp16-rounded dequantized W^T in fp32
    (adapters/lumina.py:135-150 -> chat.py:140 -> chat.py:239-243)."""
    W16 = np.asarray(W, np.float32).astype(np.float16).astype(np.float32)
    return np.asarray(x, np.float32) @ W16.T


def upload(kind, group, codes, scales, rows, cols):
    from lumina_b200.cuda import Weight
    if kind == "int4":
        blob, pack = lf.pack_codes_nibble(codes), "nibble"
    elif kind == "int2":
        blob, pack = lf.pack_codes_2bit(codes), "2bit"
    elif kind == "binary":
        blob, pack = lf.pack_signs(np.where(codes > 0, 1, -1)), "none"
    else:
        blob, pack = np.asarray(codes, np.uint8), "none"
    return Weight.upload(kind, group, pack, blob, scales, rows, cols)


def device_gemv(torch, w, x):
    xd = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
    yd = torch.empty((x.shape[0], w.rows), dtype=torch.float32, device="cuda")
    w.gemv(xd.data_ptr(), x.shape[0], x.shape[1], yd.data_ptr(), w.rows)
    torch.cuda.synchronize()
    return yd.cpu().numpy()


GOLD = {
    "model.layers.0.a.weight": 64, "model.layers.0.b.weight": 64, "model.layers.0.c.weight": 64,
    "model.layers.0.d.weight": 64, "model.layers.1.e.weight": 128, "model.layers.1.f.weight": 128,
    "model.layers.1.g.weight": 128, "model.layers.1.h.weight": 128,
}


def golden_record(name):
    from lumina_b200.loader import LuminaFile
    with LuminaFile(os.path.join(GOLDEN, "small_g%d.lumina" % GOLD[name])) as f:
        r = f.record(name)
        return r.kind, r.group, r.pack, r.codes.copy(), r.scales.copy(), r.shape


@pytest.mark.parametrize("name", sorted(GOLD))
def test_unpack_dequant_bit_exact(torch_cuda, golden, name):
    torch = torch_cuda
    from lumina_b200.cuda import Weight
    kind, group, pack, codes, scales, (rows, cols) = golden_record(name)
    w = Weight.upload(kind, group, pack, codes, scales, rows, cols)
    out = torch.empty(rows * cols, dtype=torch.uint8, device="cuda")
    w.unpack(out.data_ptr())
    deq = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    w.dequant(deq.data_ptr())
    torch.cuda.synchronize()
    if kind == "binary":
        want = lf.sign_bits(codes.reshape(rows, -1), cols)
    else:
        want = lf.unpack_codes(codes.tobytes(), (rows, cols), pack)
    assert np.array_equal(out.cpu().numpy().reshape(rows, cols), want)
    g = golden("format_cases.npz")[name + "|dequant"]
    got = deq.cpu().numpy().reshape(rows, cols)
    assert np.array_equal(got.view(np.uint32), g.view(np.uint32))


@pytest.mark.parametrize("name", sorted(GOLD))
@pytest.mark.parametrize("batch", [1, 3, 16])
def test_gemv_golden_records(torch_cuda, golden, name, batch):
    from lumina_b200.cuda import Weight
    kind, group, pack, codes, scales, (rows, cols) = golden_record(name)
    w = Weight.upload(kind, group, pack, codes, scales, rows, cols)
    x = np.random.default_rng(batch).standard_normal((batch, cols)).astype(np.float32)
    y = device_gemv(torch_cuda, w, x)
    W = golden("format_cases.npz")[name + "|dequant"]
    assert rel_l2(y, ref_gemv(x, W)) < REL_L2
    c = lf.sign_bits(codes.reshape(rows, -1), cols) if kind == "binary" else \
        lf.unpack_codes(codes.tobytes(), (rows, cols), pack)
    km = kernel_model.gemv(c, scales, group, lf.KIND_BITS[kind], x)
    np.testing.assert_allclose(y, km, rtol=TIGHT, atol=TIGHT * np.abs(km).max())


SHAPES = [  # (kind, group, N, K)
    ("int4", 64, 4096, 4096), ("int4", 64, 11008, 4096), ("int4", 64, 4096, 11008),
    ("int2", 128, 4096, 4096), ("int2", 128, 4096, 11008),
    ("binary", 128, 4096, 4096), ("binary", 128, 11008, 4096),
    ("int3", 64, 4096, 4096), ("int3", 64, 4096, 11008),
]


@pytest.mark.parametrize("kind,group,N,K", SHAPES)
@pytest.mark.parametrize("batch", [1, 4, 16])
def test_gemv_7b_shapes(torch_cuda, kind, group, N, K, batch):
    bits = lf.KIND_BITS[kind]
    rng = np.random.default_rng(N + K + bits)
    codes = rng.integers(0, 1 << bits, (N, K)).astype(np.uint8)
    ng = (K + group - 1) // group
    scales = (np.abs(rng.standard_normal((N, ng))) * 0.02 + 1e-3).astype(np.float16).astype(np.float32)
    w = upload(kind, group, codes, scales, N, K)
    assert w.info()["fp16_scales"]
    x = rng.standard_normal((batch, K)).astype(np.float32)
    y = device_gemv(torch_cuda, w, x)
    lv = lf.levels(bits).astype(np.float32)
    W = np.repeat(scales, group, axis=1)[:, :K] * lv[codes]
    assert rel_l2(y, ref_gemv(x, W)) < REL_L2
    rows = slice(0, 256)
    km = kernel_model.gemv(codes[rows], scales[rows], group, bits, x)
    np.testing.assert_allclose(y[:, rows], km, rtol=TIGHT, atol=TIGHT * np.abs(km).max())


@pytest.mark.parametrize("group,N,K", [(64, 4096, 4096), (64, 12288, 4096), (128, 4096, 11008), (64, 300, 640),
                                         (64, 4096, 11008)])
@pytest.mark.parametrize("batch", [1, 2, 3, 4, 5, 8, 9, 16])
def test_gemv_fragment_layout(torch_cuda, monkeypatch, group, N, K, batch):
    """int4 in the tensor-core fragment layout: the tensor-pipe decode GEMV
    (batch <= 4: units split over CTAs and warps, shared-tile combine) and
    the batched tensor-pipe GEMV (5..16: activation fragments in global
    memory, K split over CTAs with an ordered combine) give the exact-model
    results of their arithmetic (64-column activation blocks), and the same
    bits on a repeated call."""
    monkeypatch.setenv("LUMINA_INT4_LAYOUT", "mma")
    rng = np.random.default_rng(N + K + batch)
    codes = rng.integers(0, 16, (N, K)).astype(np.uint8)
    ng = (K + group - 1) // group
    scales = (np.abs(rng.standard_normal((N, ng))) * 0.02 + 1e-3).astype(np.float16).astype(np.float32)
    w = upload("int4", group, codes, scales, N, K)
    rows32, nbp = -(-N // 32) * 32, (-(-K // 32) + 1) // 2 * 2
    assert w.info()["device_bytes"] == rows32 * nbp * 16 + rows32 * ng * 2  # the fragment layout
    x = rng.standard_normal((batch, K)).astype(np.float32)
    y = device_gemv(torch_cuda, w, x)
    y2 = device_gemv(torch_cuda, w, x)
    assert np.array_equal(y.view(np.uint32), y2.view(np.uint32))
    W = np.repeat(scales, group, axis=1)[:, :K] * lf.levels(4).astype(np.float32)[codes]
    assert rel_l2(y, ref_gemv(x, W)) < REL_L2
    rows = np.r_[0:128, N - 128:N]
    km = kernel_model.gemv(codes[rows], scales[rows], group, 4, x, **kernel_model.TENSOR_PIPE)
    np.testing.assert_allclose(y[:, rows], km, rtol=TIGHT, atol=TIGHT * np.abs(km).max())


@pytest.mark.parametrize("kind,group,N,K", [("int3", 64, 4096, 4096), ("int2", 128, 11008, 4096),
                                            ("binary", 128, 4096, 11008), ("int2", 128, 300, 640)])
@pytest.mark.parametrize("batch", [1, 3, 4, 7, 16])
def test_gemv_narrow_fragment_layout(torch_cuda, monkeypatch, kind, group, N, K, batch):
    """int3 / int2 / binary codes stored one per nibble in the fragment
    layout (LUMINA_NARROW_LAYOUT=mma): the unpack gate returns the file's
    codes, and the tensor-pipe GEMVs (decode for batch <= 4, batched for
    5..16) give the exact-model results with the kind's own level count."""
    monkeypatch.setenv("LUMINA_NARROW_LAYOUT", "mma")
    torch = torch_cuda
    bits = lf.KIND_BITS[kind]
    rng = np.random.default_rng(N + K + batch + bits)
    codes = rng.integers(0, 1 << bits, (N, K)).astype(np.uint8)
    ng = (K + group - 1) // group
    scales = (np.abs(rng.standard_normal((N, ng))) * 0.02 + 1e-3).astype(np.float16).astype(np.float32)
    w = upload(kind, group, codes, scales, N, K)
    rows32, nbp = -(-N // 32) * 32, (-(-K // 32) + 1) // 2 * 2
    assert w.info()["device_bytes"] == rows32 * nbp * 16 + rows32 * ng * 2  # one code per nibble
    out = torch.empty(N * K, dtype=torch.uint8, device="cuda")
    w.unpack(out.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().reshape(N, K), codes)
    x = rng.standard_normal((batch, K)).astype(np.float32)
    y = device_gemv(torch, w, x)
    y2 = device_gemv(torch, w, x)
    assert np.array_equal(y.view(np.uint32), y2.view(np.uint32))
    W = np.repeat(scales, group, axis=1)[:, :K] * lf.levels(bits).astype(np.float32)[codes]
    assert rel_l2(y, ref_gemv(x, W)) < REL_L2
    rows = np.r_[0:128, N - 128:N]
    km = kernel_model.gemv(codes[rows], scales[rows], group, bits, x, **kernel_model.TENSOR_PIPE)
    np.testing.assert_allclose(y[:, rows], km, rtol=TIGHT, atol=TIGHT * np.abs(km).max())


def test_gemv_fragment_layout_two_devices(torch_cuda, monkeypatch):
    """One process, the tensor-pipe GEMV on device 0 and then on device 1:
    the kernel's raised shared-memory limit is a per-device setting, so the
    launch on the second device must raise it there too; both devices give
    the same bits."""
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    monkeypatch.setenv("LUMINA_INT4_LAYOUT", "mma")
    from lumina_b200.cuda import Weight
    rng = np.random.default_rng(11)
    N, K, group = 4096, 4096, 64
    codes = rng.integers(0, 16, (N, K)).astype(np.uint8)
    scales = (np.abs(rng.standard_normal((N, K // group))) * 0.02 + 1e-3).astype(np.float16).astype(np.float32)
    x = rng.standard_normal((1, K)).astype(np.float32)
    outs = []
    for dev in (0, 1):
        w = Weight.upload("int4", group, "nibble", lf.pack_codes_nibble(codes), scales, N, K, device=dev)
        with torch.cuda.device(dev):
            xd = torch.from_numpy(x).to(f"cuda:{dev}")
            yd = torch.empty((1, N), dtype=torch.float32, device=f"cuda:{dev}")
            w.gemv(xd.data_ptr(), 1, K, yd.data_ptr(), N)
            torch.cuda.synchronize(dev)
            outs.append(yd.cpu().numpy())
        w.free()
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    W = np.repeat(scales, group, axis=1) * lf.levels(4).astype(np.float32)[codes]
    assert rel_l2(outs[1], ref_gemv(x, W)) < REL_L2


def test_fp32_scales_path(torch_cuda):
    rng = np.random.default_rng(3)
    N, K = 300, 640
    codes = rng.integers(0, 16, (N, K)).astype(np.uint8)
    scales = (np.abs(rng.standard_normal((N, K // 64))) * 0.02 + 1e-3).astype(np.float32)
    w = upload("int4", 64, codes, scales, N, K)
    assert not w.info()["fp16_scales"]
    x = rng.standard_normal((2, K)).astype(np.float32)
    y = device_gemv(torch_cuda, w, x)
    km = kernel_model.gemv(codes, scales, 64, 4, x)
    np.testing.assert_allclose(y, km, rtol=TIGHT, atol=TIGHT * np.abs(km).max())


def test_gemv_host_entry(torch_cuda):
    rng = np.random.default_rng(4)
    codes = rng.integers(0, 16, (128, 256)).astype(np.uint8)
    scales = np.full((128, 4), 0.03125, np.float32)
    w = upload("int4", 64, codes, scales, 128, 256)
    x = rng.standard_normal((5, 256)).astype(np.float32)
    np.testing.assert_allclose(w.gemv_host(x), device_gemv(torch_cuda, w, x), rtol=0, atol=0)


def test_upload_errors(torch_cuda):
    from lumina_b200.cuda import LuminaError, Weight
    codes = np.zeros((4, 32), np.uint8)
    with pytest.raises(LuminaError, match="group_size"):
        Weight.upload("int4", 48, "nibble", codes, np.ones((4, 2), np.float32), 4, 64)
    with pytest.raises(LuminaError, match="scales"):
        Weight.upload("int4", 64, "nibble", codes, np.ones((4, 2), np.float32), 4, 64)
    with pytest.raises(LuminaError, match="packed flag"):
        Weight.upload("int4", 64, "2bit", codes, np.ones((4, 1), np.float32), 4, 64)
    with pytest.raises(LuminaError, match="out of range"):
        Weight.upload("int3", 64, "none", np.full((4, 64), 9, np.uint8), np.ones((4, 1), np.float32), 4, 64)


def test_tops_known_answers(torch_cuda, golden):
    from lumina_b200 import cuda
    k = golden("tops_kat.npz")
    r = cuda.gemv_int8(k["xq"], k["xs"], k["wq"], k["ws"])
    assert "out" in r, r
    assert float(np.abs(r["out"] - k["ref_int8"]).max()) <= 1e-3   # tops.py:168-170
    r = cuda.gemv_q4_0(k["xq"], k["xs"], k["q4"], k["q4s"])
    assert float(np.abs(r["out"] - k["ref_q4_0"]).max()) <= 1e-2   # tops.py:196-198
    rng = np.random.default_rng(11)
    xh = rng.standard_normal(256).astype(np.float16)
    wh = (rng.standard_normal((37, 256)) * 0.05).astype(np.float16)
    r = cuda.gemv_fp16(xh, wh)
    ref = xh.astype(np.float32) @ wh.astype(np.float32).T
    assert float(np.abs(r["out"] - ref).max() / np.abs(ref).max()) <= 1e-2   # tops.py:217-220
    xqm = rng.integers(-8, 8, (5, 256)).astype(np.int8)
    xsm = (np.abs(rng.standard_normal((5, 8))).astype(np.float32) + 0.01)
    r = cuda.gemm_int8(xqm, xsm, k["wq"], k["ws"])
    for m in range(5):
        assert float(np.abs(r["out"][m] - otops.ref_int8(xqm[m], xsm[m], k["wq"], k["ws"])).max()) <= 1e-2
    # edge shapes of tests/test_tops_kernel.py:223-239 (K = 32/96, N = 1/7)
    for N, K in ((1, 32), (7, 96), (3, 1024)):
        xq = rng.integers(-127, 128, K).astype(np.int8)
        xs = (np.abs(rng.standard_normal(K // 32)) + 0.01).astype(np.float32)
        wq = rng.integers(-127, 128, (N, K)).astype(np.int8)
        ws = (np.abs(rng.standard_normal(N)) + 0.1).astype(np.float32)
        r = cuda.gemv_int8(xq, xs, wq, ws)
        ref = otops.ref_int8(xq, xs, wq, ws)
        assert float(np.abs(r["out"] - ref).max()) <= 1e-3 * max(1.0, float(np.abs(ref).max()))


def test_tops_error_convention():
    from lumina_b200 import cuda
    r = cuda.gemv_int8(np.zeros(16, np.int8), np.ones(1, np.float32), np.zeros((2, 32), np.int8),
                       np.ones(2, np.float32))
    assert "error" in r
