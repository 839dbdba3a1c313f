"""Oracle: the Lumina quantizer with no calibration data (H = I).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

With no calibration activations (``_collect_acts`` returns ``{}``,
scripts/lumina_convert.py:219-226) the GPTQ inverse Hessian is the identity,
so the error feedback ``W[:, j+1:] -= err * Hinv[j, j+1:]`` adds exact zeros
(ptq_ladder.py:317-324) and each code is ``argmin |W/s - level|`` with ``s``
from the MSE scale search. This module is that computation, vectorised:

  * ``group_scales``  — ptq_ladder.py:215-249 (7 absmax multipliers, first
    minimum of the mean squared error wins, ties keep the earlier candidate)
  * ``quantize_int``  — ptq_ladder.py:252-329 + 370-399 with Hinv = None
  * ``quantize_binary`` — ptq_ladder.py:402-455 with Hinv = None: sign
    (``>= 0`` is +1) then a least-squares scale per group over the original W
  * ``convert_arrays`` — scripts/lumina_convert.py:48-97 (2-D tensors whose
    name contains embed/head/lm_head/output/router/norm stay raw fp32, as do
    tensors with a side < 16)
"""
from __future__ import annotations

import numpy as np

from .lumina_format import levels, pack_signs

_MULTIPLIERS = (1.0, 0.8, 0.65, 0.5, 0.4, 0.3, 0.2)  # ptq_ladder.py:235
SENSITIVE_SUBSTR = ("embed", "head", "lm_head", "output", "router", "norm", "norm_")


def _nearest(wn: np.ndarray, lv: np.ndarray) -> np.ndarray:
    """argmin over levels of |wn - lv| with the first index winning ties,
    as ``np.argmin`` in ptq_ladder.py:238-239,314."""
    return np.abs(wn[..., None] - lv).argmin(axis=-1)


def group_scales(W: np.ndarray, group_size: int, nbits: int) -> np.ndarray:
    """ptq_ladder.py:215-249, identical arithmetic (fp64)."""
    W = np.asarray(W, dtype=np.float64)
    o, i = W.shape
    ng = (i + group_size - 1) // group_size
    lv = levels(nbits)
    out = np.zeros((o, ng))
    for g in range(ng):
        Wg = W[:, g * group_size:min(i, (g + 1) * group_size)]
        amax = np.abs(Wg).max(axis=1).clip(1e-12)
        best_e = best_s = None
        for f in _MULTIPLIERS:
            s = np.clip(amax * f, 1e-12, None)
            wn = Wg / s[:, None]
            e = ((wn - lv[_nearest(wn, lv)]) ** 2).mean(axis=1)
            if best_e is None:
                best_e, best_s = e, s
            else:
                take = e < best_e
                best_e = np.where(take, e, best_e)
                best_s = np.where(take, s, best_s)
        out[:, g] = best_s
    return out


def quantize_int(W: np.ndarray, nbits: int, group_size: int = 64) -> tuple[np.ndarray, np.ndarray]:
    """(codes int32 (o,i), scales fp64 (o, ng)) — ptq_ladder.py:370-399 with
    Hinv = None. Columns are visited in ``argsort(-diag)`` order in the
    reference, which with H = I only permutes identical independent work."""
    W = np.asarray(W, dtype=np.float64)
    s = group_scales(W, group_size, nbits)
    se = np.repeat(s, group_size, axis=1)[:, :W.shape[1]]
    codes = _nearest(W / se, levels(nbits)).astype(np.int32)
    return codes, s


def quantize_binary(W: np.ndarray, group_size: int = 64) -> tuple[np.ndarray, np.ndarray]:
    """(packed sign bytes (o, ceil(i/8)), fp32 scales (o, ng)) —
    ptq_ladder.py:402-455 with Hinv = None."""
    W = np.asarray(W, dtype=np.float64)
    o, i = W.shape
    ng = (i + group_size - 1) // group_size
    sign = np.where(W >= 0, 1.0, -1.0)
    scales = np.empty((o, ng))
    for g in range(ng):
        sl = slice(g * group_size, min(i, (g + 1) * group_size))
        num = np.einsum("oj,oj->o", W[:, sl], sign[:, sl])
        den = np.einsum("oj,oj->o", sign[:, sl], sign[:, sl]).clip(1e-12)
        scales[:, g] = num / den
    return pack_signs(sign), scales.astype(np.float32)


def is_sensitive(name: str) -> bool:
    """scripts/lumina_convert.py:48-52."""
    return any(s in name.lower() for s in SENSITIVE_SUBSTR)


def convert_arrays(arrays: dict, rung: str, group_size: int = 64,
                   fp16_scales: bool = False) -> dict:
    """``{name: ("raw", fp32) | (kind, (codes, scales))}`` as
    scripts/lumina_convert.py:55-97 returns (without its stats list).

    ``fp16_scales`` rounds every stored scale to the nearest fp16 value (the
    F32 field then holds fp16-exact numbers) — the synthetic workloads are
    specified with an fp16 scale per group.
    """
    bits = {"int4": 4, "int3": 3, "int2": 2, "binary": 1}[rung]
    out = {}
    for name, W in arrays.items():
        W = np.asarray(W, dtype=np.float64)
        if W.ndim != 2 or min(W.shape) < 16 or is_sensitive(name):
            out[name] = ("raw", W.astype(np.float32))
            continue
        if bits == 1:
            codes, scales = quantize_binary(W, group_size)
        else:
            codes, scales = quantize_int(W, bits, group_size)
        scales = np.asarray(scales, dtype=np.float32)
        if fp16_scales:
            scales = scales.astype(np.float16).astype(np.float32)
        out[name] = (rung, (codes, scales))
    return out
