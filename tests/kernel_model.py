"""Exact numpy model of the device GEMV arithmetic (not the reference).

The parity oracle for the GEMV is the reference's own math (x @ fp16(dequant)
.T in fp32, ``oracle``). This module restates *our* kernel's arithmetic —
int16 activation blocks, exact integer dot, per-block fp32 scale-up — so a
test can also hold the device result to ~1e-6 and catch indexing mistakes
that the 2e-3 reference tolerance would hide.
"""
import numpy as np


def act_quant(x):
    """Per-32-column int16 quantization: q = rint(x * fp32(32767/amax))."""
    x = np.asarray(x, dtype=np.float32)
    B, K = x.shape
    nblk = (K + 31) // 32
    xp = np.zeros((B, nblk * 32), np.float32)
    xp[:, :K] = x
    blk = xp.reshape(B, nblk, 32)
    amax = np.abs(blk).max(axis=2)
    with np.errstate(divide="ignore", invalid="ignore"):
        f = np.where(amax > 0, np.float32(32767.0) / amax, np.float32(0)).astype(np.float32)
        sx = np.where(amax > 0, amax / np.float32(32767.0), np.float32(0)).astype(np.float32)
    q = np.rint((blk * f[:, :, None]).astype(np.float32)).clip(-32767, 32767).astype(np.int64)
    return q, sx


def gemv(codes, scales, group, bits, x):
    """y (B, N) float64 for unpacked codes (N, K) and fp32 scales (N, ng)."""
    codes = np.asarray(codes, dtype=np.int64)
    N, K = codes.shape
    L = (1 << bits) - 1
    q, sx = act_quant(x)
    B, nblk, _ = q.shape
    cp = np.zeros((N, nblk * 32), np.int64)
    cp[:, :K] = codes
    cb = cp.reshape(N, nblk, 32)
    d = np.einsum("bkj,nkj->bnk", q, cb)                    # exact integer dots
    t = 2 * d - L * q.sum(axis=2)[:, None, :]
    s = np.asarray(scales, dtype=np.float64)[:, (np.arange(nblk) * 32) // group]  # (N, nblk)
    return (t * sx[:, None, :].astype(np.float64) * s[None]).sum(axis=2) / L
