"""The benchmark's GPU-side input generator restates the reference quantizer
(ptq_ladder.py:215-249, 370-399) and the file packing (adapters/lumina.py:
20-40); checked here on the CPU against the oracle: codes and stored
(fp16-rounded) scales are bit-identical, so the GPU run and the reference
see the same packed model."""
import numpy as np
import pytest
import torch

from oracle import lumina_format as lf
from oracle.quant import quantize_int
from lumina_b200 import synthetic


def _oracle(W, bits):
    codes, sc = quantize_int(W, bits, 64)
    # the file writer: fp64 -> fp32 -> fp16 (quant.py convert_arrays)
    return codes, sc.astype(np.float32).astype(np.float16).astype(np.float32)


@pytest.mark.parametrize("seed", [4, 7])
@pytest.mark.parametrize("bits", [4, 3, 2])
def test_quantizer_matches_oracle(seed, bits):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((128, 1024)) * 0.02).astype(np.float32)
    c, s = synthetic._quantize_gpu(torch.from_numpy(W), bits, 64)
    codes_ref, s_ref = _oracle(W, bits)
    assert np.array_equal(s.numpy(), s_ref)
    assert np.array_equal(c.numpy(), codes_ref)


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
    codes_ref, s_ref = _oracle(W, 4)
    assert np.array_equal(s.numpy(), s_ref)
    assert np.array_equal(c.numpy(), codes_ref)
