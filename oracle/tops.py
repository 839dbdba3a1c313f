"""Oracle: the int8 fused-GEMV semantics of the reference's TOPS kernels.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

  * ``q8_repack``  — src/lumina_framework/fused.py:91-102 (per-32 absmax,
    ``np.round`` half-even, clip ±127, scale amax/127)
  * ``ref_int8``   — src/lumina_framework/tops.py:115-127, the int32-exact
    reference of ``tops_gemv_int8`` (kernels/tops_int8.c:41-66):
    ``out[n] = ws[n] * sum_b xs[b] * dot32(xq_b, wq[n]_b)``
  * ``ref_q4_0``   — tops.py:130-149 (``tops_gemv_q4_0``, tops_int8.c:73-106):
    packed (N, K/2) nibbles, value = code - 8, scales (N, K/32)
  * ``quantize_int8_per_row`` — src/lumina_framework/memory.py:158-163 (the
    ``TensorContainer`` payload that feeds ``fused_gemv_int8``)
  * ``self_test_inputs`` — the known-answer inputs of ``tops._self_test``
    (tops.py:152-238, seed 11, N=37, K=256)
  * ``numba_gemv_int8`` — ``fused._gemv_int8`` (fused.py:163-184), the
    numba kernel that serves ``fused_gemv_int8`` when the compiled tops
    kernel is absent, restated with its loop order and fp32 rounding so that
    the CPU baseline can time the reference's own GEMV path
"""
from __future__ import annotations

import functools

import numpy as np


def q8_repack(x, block=32):
    x = np.asarray(x, dtype=np.float32)
    flat = x.reshape(-1)
    pad = (-flat.size) % block
    if pad:
        flat = np.concatenate([flat, np.zeros(pad, np.float32)])
    blk = flat.reshape(-1, block)
    amax = np.abs(blk).max(axis=1, keepdims=True).clip(1e-12)
    q = np.round(blk * (127.0 / amax)).clip(-127, 127).astype(np.int8)
    q = q.reshape(-1)[:x.size].reshape(x.shape)
    return q, (amax[:, 0] / 127.0).astype(np.float32)


def ref_int8(xq, xs, wq, ws):
    N, K = wq.shape
    nb = K // 32
    xb = xq[:nb * 32].astype(np.int64).reshape(nb, 32)
    wb = wq[:, :nb * 32].astype(np.int64).reshape(N, nb, 32)
    seg = np.einsum("nbj,bj->nb", wb, xb).astype(np.float64)
    acc = (seg * xs[:nb].astype(np.float64)).sum(axis=1)
    return acc * ws.reshape(-1).astype(np.float64)


def ref_q4_0(xq, xs, wq, ws):
    N = wq.shape[0]
    K = wq.shape[1] * 2
    nb = K // 32
    inter = np.empty((N, K), dtype=np.int64)
    inter[:, 0::2] = (wq & 15).astype(np.int64) - 8
    inter[:, 1::2] = (wq >> 4).astype(np.int64) - 8
    seg = np.einsum("nbj,bj->nb", inter.reshape(N, nb, 32),
                    xq[:K].astype(np.int64).reshape(nb, 32)).astype(np.float64)
    return (seg * xs[:nb].astype(np.float64) * ws.astype(np.float64)).sum(axis=1)


def quantize_int8_per_row(x):
    x = np.atleast_2d(x)
    amax = np.abs(x).max(axis=1, keepdims=True).clip(1e-12)
    q = np.round(x * (127.0 / amax)).clip(-127, 127).astype(np.int8)
    return q, (amax / 127.0).astype(np.float32)


def self_test_inputs():
    """The first draws of tops._self_test (tops.py:154-159,185-187)."""
    rng = np.random.default_rng(11)
    N, K = 37, 256
    xq = rng.integers(-8, 8, K).astype(np.int8)
    xs = (np.abs(rng.standard_normal(K // 32)).astype(np.float32) + 0.01)
    wq = rng.integers(-8, 8, (N, K)).astype(np.int8)
    ws = (np.abs(rng.standard_normal(N)).astype(np.float32) + 0.1)
    codes = rng.integers(0, 16, (N, K)).astype(np.uint8)
    q4 = ((codes[:, 0::2] & 15) | ((codes[:, 1::2] & 15) << 4)).astype(np.uint8)
    q4s = (np.abs(rng.standard_normal((N, K // 32))).astype(np.float32) + 0.01)
    return {"xq": xq, "xs": xs, "wq": wq, "ws": ws, "q4": q4, "q4s": q4s}


@functools.lru_cache(maxsize=1)
def numba_gemv_int8():
    """The compiled ``gemv(xq, xs, wq, ws, out)`` of fused.py:163-184: one
    core, rows in order; per row an int32 dot per 32-element block, and
    ``acc += f32(dot) * f32(xs[b]) * f32(ws[n])`` in block order, all in
    fp32. None when numba is not importable."""
    try:
        import numba
    except ImportError:
        return None

    @numba.njit(cache=False)
    def gemv(xq, xs, wq, ws, out):
        nrows, k = wq.shape
        for n in range(nrows):
            s = np.float32(ws[n])
            acc = np.float32(0.0)
            for b in range(k // 32):
                dot = np.int32(0)
                for j in range(b * 32, b * 32 + 32):
                    dot += np.int32(xq[j]) * np.int32(wq[n, j])
                acc += np.float32(dot) * np.float32(xs[b]) * s
            out[n] = acc

    return gemv
