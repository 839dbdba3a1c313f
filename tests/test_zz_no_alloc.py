"""lumina_gemv_noalloc: the packed GEMV for callers that cannot allocate
device memory (a runtime that owns every allocation through its own pool, or
one that must not trigger a cudaFree's device-wide synchronisation).

It must give lumina_gemv's results (same tolerance as the other GEMV tests)
on back-to-back calls that share its fixed scratch array, and refuse sizes
beyond that array. This file is collected last so that a first-failure stop
has already run every other test; it also passes alone in a fresh process
(the first call on the device does the scratch set-up)."""
import numpy as np
import pytest

from oracle import lumina_format as lf

pytestmark = pytest.mark.gpu

TIGHT = 2e-6  # the GEMV tests' tolerance between two device paths of the same arithmetic


def _weight(kind, rows, cols, group, seed):
    from lumina_b200.cuda import Weight
    rng = np.random.default_rng(seed)
    bits = {"int4": 4, "int3": 3, "int2": 2, "binary": 1}[kind]
    codes = rng.integers(0, 1 << bits, (rows, cols)).astype(np.uint8)
    ng = -(-cols // group)
    scales = (rng.random((rows, ng)) * 0.02 + 0.001).astype(np.float16).astype(np.float32)
    if kind == "int4":
        blob, pack = lf.pack_codes_nibble(codes), "nibble"
    elif kind == "int2":
        blob, pack = lf.pack_codes_2bit(codes), "2bit"
    elif kind == "binary":
        blob, pack = lf.pack_signs(np.where(codes > 0, 1.0, -1.0)), "none"
    else:
        blob, pack = codes, "none"
    return Weight.upload(kind, group, pack, blob, scales, rows, cols)


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from lumina_b200 import cuda
    cuda.ensure_device(0)
    return torch


@pytest.mark.parametrize("kind,rows,cols,group,batch", [
    ("int4", 4096, 4096, 64, 1),
    ("int4", 11008, 4096, 64, 3),
    ("int3", 1000, 2048, 64, 16),
    ("int2", 4096, 11008, 128, 4),
    ("binary", 4096, 4096, 128, 2),
])
def test_noalloc_matches_gemv_twice(torch_cuda, kind, rows, cols, group, batch):
    torch = torch_cuda
    w = _weight(kind, rows, cols, group, seed=rows + cols + batch)
    try:
        rng = np.random.default_rng(batch)
        outs = []
        for call in range(2):  # two calls in a row share (and overwrite) the fixed scratch
            x = torch.from_numpy((rng.standard_normal((batch, cols)) * (1 + call)).astype(np.float32)).cuda()
            y_ref = torch.empty((batch, rows), dtype=torch.float32, device="cuda")
            y = torch.full((batch, rows), float("nan"), dtype=torch.float32, device="cuda")
            w.gemv(x.data_ptr(), batch, cols, y_ref.data_ptr(), rows)
            w.gemv_noalloc(x.data_ptr(), batch, cols, y.data_ptr(), rows)
            torch.cuda.synchronize()
            a, b = y.cpu().numpy(), y_ref.cpu().numpy()
            np.testing.assert_allclose(a, b, rtol=TIGHT, atol=TIGHT * np.abs(b).max())
            outs.append(a)
        assert not np.array_equal(outs[0], outs[1])
    finally:
        w.free()


def test_noalloc_rejects_oversize(torch_cuda):
    from lumina_b200.cuda import LuminaError
    torch = torch_cuda
    cols = 32768  # 16 rows x 1024 blocks x 72 bytes > 1 MiB
    w = _weight("int4", 64, cols, 64, seed=1)
    try:
        x = torch.zeros((16, cols), dtype=torch.float32, device="cuda")
        y = torch.zeros((16, 64), dtype=torch.float32, device="cuda")
        with pytest.raises(LuminaError, match="scratch"):
            w.gemv_noalloc(x.data_ptr(), 16, cols, y.data_ptr(), 64)
        # the largest batch that fits still runs and matches
        w.gemv_noalloc(x.data_ptr(), 8, cols, y.data_ptr(), 64)
        torch.cuda.synchronize()
        assert float(y[:8].abs().max()) == 0.0
    finally:
        w.free()


_NO_ALLOC_CHILD = r"""
import sys
import numpy as np
import torch
sys.path[:0] = sys.argv[1:4]
from lumina_b200 import cuda
import test_zz_no_alloc as t

cuda.ensure_device(0)
cases = [("int4", 4096, 4096, 64, 1), ("int3", 1000, 2048, 64, 16), ("int2", 2048, 4096, 128, 4),
         ("binary", 2048, 4096, 128, 2)]
ws, bufs = [], []
for i, (kind, rows, cols, group, batch) in enumerate(cases):
    ws.append(t._weight(kind, rows, cols, group, seed=i))
    bufs.append((torch.randn(batch, cols, device="cuda"), torch.empty(batch, rows, device="cuda")))
torch.cuda.synchronize()

def run_all():
    for w, (x, y), (kind, rows, cols, group, batch) in zip(ws, bufs, cases):
        w.gemv_noalloc(x.data_ptr(), batch, cols, y.data_ptr(), rows)
    torch.cuda.synchronize()

run_all()  # the first calls load the kernels and look up the scratch array's address
free0 = torch.cuda.mem_get_info()[0]
for _ in range(5):
    run_all()
free1 = torch.cuda.mem_get_info()[0]
print("FREE", free0, free1)
assert free1 == free0, (free0, free1)
"""


def test_noalloc_allocates_nothing(torch_cuda, tmp_path):
    """In a fresh process whose first GEMV call is lumina_gemv_noalloc (so the
    library has not made its lumina_gemv scratch yet), with every kernel
    loaded at start-up (CUDA_MODULE_LOADING=EAGER), repeated calls of every
    kind leave the device's free memory unchanged to the byte."""
    import os
    import subprocess
    import sys
    from conftest import REPO
    script = tmp_path / "child.py"
    script.write_text(_NO_ALLOC_CHILD)
    env = dict(os.environ, CUDA_MODULE_LOADING="EAGER")
    r = subprocess.run([sys.executable, str(script), os.path.join(REPO, "tests"),
                        os.path.join(REPO, "lumina-studio_b200"), REPO],
                       capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "FREE" in r.stdout
