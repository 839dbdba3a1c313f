"""Exact numpy model of the device GEMV arithmetic (not the reference).

The parity oracle for the GEMV is the reference's own math (x @ fp16(dequant)
.T in fp32, ``oracle``). This module restates *our* kernel's arithmetic —
int16 activation blocks, exact integer dot, per-block fp32 scale-up — so a
test can also hold the device result to ~1e-6 and catch indexing mistakes
that the 2e-3 reference tolerance would hide.
"""
import numpy as np


# The CUDA-core GEMVs quantize per 32 columns to +-32767; the tensor-pipe
# decode GEMV (gemv_tc.cu) per 64 columns to +-32639, so that each value
# splits into two signed bytes (q = 256 * qh + ql).
CUDA_CORE = dict(block=32, qmax=32767)
TENSOR_PIPE = dict(block=64, qmax=32639)


def act_quant(x, block=32, qmax=32767):
    """Per-block int16 quantization: q = rint(x * fp32(qmax/amax))."""
    x = np.asarray(x, dtype=np.float32)
    B, K = x.shape
    nblk = (K + block - 1) // block
    xp = np.zeros((B, nblk * block), np.float32)
    xp[:, :K] = x
    blk = xp.reshape(B, nblk, block)
    amax = np.abs(blk).max(axis=2)
    with np.errstate(divide="ignore", invalid="ignore"):
        f = np.where(amax > 0, np.float32(qmax) / amax, np.float32(0)).astype(np.float32)
        sx = np.where(amax > 0, amax / np.float32(qmax), np.float32(0)).astype(np.float32)
    q = np.rint((blk * f[:, :, None]).astype(np.float32)).clip(-qmax, qmax).astype(np.int64)
    return q, sx


def gemv(codes, scales, group, bits, x, block=32, qmax=32767):
    """y (B, N) float64 for unpacked codes (N, K) and fp32 scales (N, ng)."""
    codes = np.asarray(codes, dtype=np.int64)
    N, K = codes.shape
    L = (1 << bits) - 1
    q, sx = act_quant(x, block, qmax)
    B, nblk, _ = q.shape
    cp = np.zeros((N, nblk * block), np.int64)
    cp[:, :K] = codes
    cb = cp.reshape(N, nblk, block)
    d = np.einsum("bkj,nkj->bnk", q, cb)                    # exact integer dots
    t = 2 * d - L * q.sum(axis=2)[:, None, :]
    s = np.asarray(scales, dtype=np.float64)[:, (np.arange(nblk) * block) // group]  # (N, nblk)
    return (t * sx[:, None, :].astype(np.float64) * s[None]).sum(axis=2) / L


def moe_gate_up(codes, scales, h, group=64):
    """The routed gate/up arithmetic of moe_gu_kernel for one row h:
    per 32-column chunk, s/15 * (2 * sum h*c - 15 * sum h), in float32."""
    codes = np.asarray(codes, np.float32)
    h = np.asarray(h, np.float32)
    N, K = codes.shape
    out = np.zeros(N, np.float32)
    for c0 in range(0, K, 32):
        hc = h[c0:c0 + 32]
        dot = (codes[:, c0:c0 + 32] * hc).sum(axis=1, dtype=np.float32)
        s = np.asarray(scales, np.float32)[:, c0 // group]
        out += s * (np.float32(2) * dot - np.float32(15) * hc.sum(dtype=np.float32))
    return out / np.float32(15)


def moe_down(codes, scales, a, group=64):
    """The transposed down arithmetic of moe_down_kernel: y = sum_i a_i * s_i
    * (2 c_i - 15) / 15 over the rows of down (groups along the output)."""
    codes = np.asarray(codes, np.float32)
    s = np.repeat(np.asarray(scales, np.float32), group, axis=1)[:, :codes.shape[1]]
    coef = np.asarray(a, np.float32)[:, None] * s
    return (coef * (np.float32(2) * codes - np.float32(15))).sum(axis=0, dtype=np.float32) / np.float32(15)
