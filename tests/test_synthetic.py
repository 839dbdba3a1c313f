"""The benchmark's GPU-side input generator restates the reference quantizer
(ptq_ladder.py:215-249, 370-399) and the file packing (adapters/lumina.py:
20-40); checked here on the CPU against the oracle."""
import numpy as np
import torch

from oracle import lumina_format as lf
from oracle.quant import group_scales, quantize_int
from lumina_b200 import synthetic


def test_quantizer_matches_oracle():
    rng = np.random.default_rng(4)
    W = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    for bits in (4, 3, 2):
        c, s = synthetic._quantize_gpu(torch.from_numpy(W), bits, 64)
        s_ref = group_scales(W, 64, bits)
        # same multiplier chosen (fp32 vs fp64 MSE ties aside), fp16-rounded
        assert np.mean(np.isclose(s.numpy(), s_ref.astype(np.float16).astype(np.float32), rtol=0)) > 0.97
        codes_ref, _ = quantize_int(W, bits, 64)
        assert np.mean(c.numpy() == codes_ref) > 0.97


def test_packing_matches_file_layout():
    rng = np.random.default_rng(5)
    for bits, pack in ((4, lf.pack_codes_nibble), (2, lf.pack_codes_2bit)):
        c = rng.integers(0, 1 << bits, (8, 128), dtype=np.uint8)
        got = synthetic._pack_gpu(torch.from_numpy(c), bits).numpy()
        assert np.array_equal(got.reshape(-1), np.asarray(pack(c)).reshape(-1))


def test_quantizer_ragged_last_group_matches_oracle():
    """A width that is not a multiple of the group (the tiny model's
    down_proj, 688 columns at g64): the last group is scored over its own
    columns, as ptq_ladder.py:229-247 does."""
    rng = np.random.default_rng(6)
    W = (rng.standard_normal((64, 688)) * 0.02).astype(np.float32)
    c, s = synthetic._quantize_gpu(torch.from_numpy(W), 4, 64)
    assert c.shape == (64, 688) and s.shape == (64, 11)
    s_ref = group_scales(W, 64, 4)
    assert np.mean(np.isclose(s.numpy(), s_ref.astype(np.float16).astype(np.float32), rtol=0)) > 0.97
    assert np.mean(np.isclose(s.numpy()[:, -1], s_ref[:, -1].astype(np.float16).astype(np.float32), rtol=0)) > 0.95
    codes_ref, _ = quantize_int(W, 4, 64)
    assert np.mean(c.numpy() == codes_ref) > 0.97
