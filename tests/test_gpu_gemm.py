"""The tcgen05 multi-row projection (lumina_gemm_rows, the prefill / tree
verification path): int4 codes turned into fp16 weights in shared memory,
the fp32 activation rows as fp16 hi and lo planes by TMA, fp32 accumulation
in tensor memory.

Two bars against the reference's math (fp32 x @ fp16-rounded dequantized
W, chat.py:140 + 239-243): the 2e-3 relative L2 of the decode path, and
5e-5 against the float64 product (fp32 accumulation over up to 11008
terms; a single fp16 plane of x would already miss it at about 2e-4) -- a
wrong swizzle, descriptor, plane offset or tile placement shows up as an
O(1) error there, not a rounding-sized one."""
import numpy as np
import pytest

from oracle import lumina_format as lf

pytestmark = pytest.mark.gpu

REL_L2 = 2e-3
EXACT = 5e-5


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from lumina_b200 import cuda
    cuda.ensure_device(0)
    return torch


@pytest.mark.parametrize("group,N,K", [(64, 4096, 4096), (64, 12288, 4096), (64, 4096, 11008), (128, 4096, 11008),
                                         (64, 300, 640), (64, 22016, 4096)])
@pytest.mark.parametrize("M", [8, 31, 64, 100, 256, 300])
def test_gemm_rows(torch_cuda, monkeypatch, group, N, K, M):
    torch = torch_cuda
    from lumina_b200.cuda import Weight
    monkeypatch.setenv("LUMINA_INT4_LAYOUT", "mma")
    rng = np.random.default_rng(N + K + M + group)
    codes = rng.integers(0, 16, (N, K)).astype(np.uint8)
    ng = (K + group - 1) // group
    scales = (np.abs(rng.standard_normal((N, ng))) * 0.02 + 1e-3).astype(np.float16).astype(np.float32)
    w = Weight.upload("int4", group, "nibble", lf.pack_codes_nibble(codes), scales, N, K)
    try:
        x = rng.standard_normal((M, K)).astype(np.float32)
        xd = torch.from_numpy(x).cuda()
        yd = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        w.gemm_rows(xd.data_ptr(), M, K, yd.data_ptr(), N)
        torch.cuda.synchronize()
        y = yd.cpu().numpy()
        W16 = lf.dequant("int4", codes, scales, group).astype(np.float16).astype(np.float32)
        assert rel_l2(y, x @ W16.T) < REL_L2
        assert rel_l2(y, x.astype(np.float64) @ W16.astype(np.float64).T) < EXACT
        # a second call gives the same bits (fixed accumulation order)
        w.gemm_rows(xd.data_ptr(), M, K, yd.data_ptr(), N)
        torch.cuda.synchronize()
        assert np.array_equal(yd.cpu().numpy().view(np.uint32), y.view(np.uint32))
    finally:
        w.free()
