"""Codes -> the `.lumina` file layout (what lumina_weight_upload takes).

Same packing as the reference writer (adapters/lumina.py:20-40 for int4 /
int2, ptq_ladder.py:37-47 for sign bits; int3 stays one byte per code,
scripts/lumina_convert.py:146-147).
"""
from __future__ import annotations

import numpy as np


def to_file_layout(kind: str, codes: np.ndarray):
    """(blob uint8, packed flag, logical (rows, cols)). For ``binary`` the
    codes are already the packed sign bytes (quantize_binary's payload)."""
    codes = np.asarray(codes)
    if kind == "binary":
        rows = codes.shape[0]
        return np.ascontiguousarray(codes, np.uint8), "none", (rows, codes.shape[1] * 8)
    o, i = codes.shape
    if kind == "int4":
        c = codes.astype(np.uint8)
        if i % 2:
            c = np.concatenate([c, np.zeros((o, 1), np.uint8)], axis=1)
        c = c.reshape(o, -1, 2)
        return ((c[..., 0] & 0xF) | ((c[..., 1] & 0xF) << 4)).astype(np.uint8), "nibble", (o, i)
    if kind == "int2":
        c = codes.astype(np.uint8)
        pad = (-i) % 4
        if pad:
            c = np.concatenate([c, np.zeros((o, pad), np.uint8)], axis=1)
        c = c.reshape(o, -1, 4) & 0x3
        return (c[..., 0] | (c[..., 1] << 2) | (c[..., 2] << 4) | (c[..., 3] << 6)).astype(np.uint8), "2bit", (o, i)
    if kind == "int3":
        return np.ascontiguousarray(codes, np.uint8), "none", (o, i)
    raise ValueError("unknown kind " + kind)
