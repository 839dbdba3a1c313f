"""Oracle: the `.lumina` container, code packing and dequantization.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates:
  * ``pack_codes_nibble`` / ``pack_codes_2bit`` / ``unpack_codes`` —
    src/lumina_framework/adapters/lumina.py:20-76
  * ``pack_signs`` / ``unpack_signs`` / ``_levels`` —
    src/lumina_format/codecs/ptq_ladder.py:37-59
  * dequant at load — src/lumina_framework/adapters/lumina.py:135-150
  * the on-disk container written by ``write_lumina`` —
    scripts/lumina_convert.py:100-165 (magic ``<IIQ``, JSON header, blobs)
"""
from __future__ import annotations

import json
import struct

import numpy as np

LUMINA_MAGIC = 0x4E494D4C  # "LMIN"  (adapters/lumina.py:16)
LUMINA_VERSION = 1         # (adapters/lumina.py:17)

KIND_BITS = {"int4": 4, "int3": 3, "int2": 2, "binary": 1}


def levels(nbits: int) -> np.ndarray:
    """``np.linspace(-1, 1, 2**b)`` in float64 (ptq_ladder.py:58-59)."""
    return np.linspace(-1.0, 1.0, 2 ** nbits)


def pack_codes_nibble(codes: np.ndarray) -> np.ndarray:
    """Two int4 codes per byte, low nibble = even column; odd widths padded
    with a zero code (adapters/lumina.py:20-27)."""
    codes = np.asarray(codes)
    o, i = codes.shape
    if i % 2:
        codes = np.concatenate([codes, np.zeros((o, 1), codes.dtype)], axis=1)
    c = codes.astype(np.uint8).reshape(o, -1, 2)
    return ((c[..., 0] & 0xF) | ((c[..., 1] & 0xF) << 4)).astype(np.uint8)


def pack_codes_2bit(codes: np.ndarray) -> np.ndarray:
    """Four int2 codes per byte, column 4j+t in bits 2t..2t+1; widths padded to
    a multiple of 4 (adapters/lumina.py:30-40)."""
    codes = np.asarray(codes)
    o, i = codes.shape
    pad = (-i) % 4
    if pad:
        codes = np.concatenate([codes, np.zeros((o, pad), codes.dtype)], axis=1)
    c = codes.astype(np.uint8).reshape(o, -1, 4) & 0x3
    return (c[..., 0] | (c[..., 1] << 2) | (c[..., 2] << 4) | (c[..., 3] << 6)).astype(np.uint8)


def pack_signs(sign: np.ndarray) -> np.ndarray:
    """1 bit per weight, bit t of byte j = column 8j+t, 1 means +1; widths
    padded to a multiple of 8 (ptq_ladder.py:37-47)."""
    pos = (np.asarray(sign) > 0).astype(np.uint8)
    o, i = pos.shape
    pad = (-i) % 8
    if pad:
        pos = np.concatenate([pos, np.zeros((o, pad), np.uint8)], axis=1)
    w = (1 << np.arange(8)).astype(np.uint8)
    return (pos.reshape(o, -1, 8) * w).sum(axis=2).astype(np.uint8)


def unpack_codes(buf: bytes | np.ndarray, shape: tuple[int, int], flag: str) -> np.ndarray:
    """Inverse of the packers. The packed row stride comes from the blob size,
    never from the matrix width (adapters/lumina.py:50-76)."""
    o, i = shape
    raw = np.frombuffer(bytes(buf), dtype=np.uint8) if not isinstance(buf, np.ndarray) \
        else np.ascontiguousarray(buf, dtype=np.uint8).reshape(-1)
    if flag == "nibble":
        per = 2
        parts = (raw & 0xF, raw >> 4)
    elif flag == "2bit":
        per = 4
        parts = tuple((raw >> (2 * t)) & 0x3 for t in range(4))
    else:
        return raw.reshape(o, i)
    wp = raw.size * per // o
    if wp * o != raw.size * per or wp < i:
        raise ValueError("bad %s blob: %d bytes for shape %s" % (flag, raw.size, shape))
    flat = np.stack([p.reshape(o, -1) for p in parts], axis=2).reshape(o, wp)
    return flat[:, :i]


def unpack_signs(packed: np.ndarray, m: int) -> np.ndarray:
    """Sign bits to {-1,+1} float32 (ptq_ladder.py:50-55)."""
    packed = np.asarray(packed, dtype=np.uint8)
    bits = (packed[:, :, None] >> np.arange(8, dtype=np.uint8)) & 1
    return np.where(bits == 1, 1, -1).astype(np.float32).reshape(packed.shape[0], -1)[:, :m]


def sign_bits(packed: np.ndarray, m: int) -> np.ndarray:
    """Sign bits as 0/1 codes (the binary kind's code value)."""
    packed = np.asarray(packed, dtype=np.uint8)
    bits = (packed[:, :, None] >> np.arange(8, dtype=np.uint8)) & 1
    return bits.reshape(packed.shape[0], -1)[:, :m].astype(np.uint8)


def dequant(kind: str, codes: np.ndarray, scales: np.ndarray, group: int,
            cols: int | None = None) -> np.ndarray:
    """Load-time dequant, fp64 product rounded once to fp32
    (adapters/lumina.py:135-150).

    ``codes`` are unpacked codes (o, i) for int kinds; for ``binary`` they are
    the packed sign bytes (o, ceil(i/8)) and the width is
    ``scales.shape[1] * group`` exactly as the reference computes it (:143).
    """
    scales = np.asarray(scales, dtype=np.float32)
    if kind in ("int4", "int3", "int2"):
        lv = levels(KIND_BITS[kind])
        s = np.repeat(scales, group, axis=1)[:, :codes.shape[1]]
        return (s * lv[codes.astype(np.int64)]).astype(np.float32)
    if kind == "binary":
        K = scales.shape[1] * group if cols is None else cols
        bits = (codes[:, :, None] >> np.arange(8, dtype=np.uint8)) & 1
        signs = np.where(bits == 1, 1.0, -1.0).astype(np.float32).reshape(codes.shape[0], -1)[:, :K]
        s = np.repeat(scales, group, axis=1)[:, :K]
        return (signs * s).astype(np.float32)
    raise ValueError("unknown kind " + kind)


# ---------------------------------------------------------------------------
# container (scripts/lumina_convert.py:100-165; adapters/lumina.py:95-159)
# ---------------------------------------------------------------------------

def write_lumina(path: str, payloads: dict, name: str = "lumina", rung: str = "int4",
                 group_size: int = 64, group_sizes: dict | None = None,
                 extra_header: dict | None = None) -> None:
    """Serialise ``{name: ("raw", fp32) | (kind, (codes, scales))}``.

    Same record fields and byte layout as ``write_lumina``
    (lumina_convert.py:121-165): raw tensors as F32 blobs; int4 nibble-packed,
    int2 2-bit packed, int3 and binary (already sign-packed codes) one byte
    per stored code with ``packed: none``; F32 scales after the codes.
    ``group_sizes`` lets a file mix group sizes per tensor (the reader honours
    the per-tensor ``group_size`` field, adapters/lumina.py:126).
    """
    header = {"format": "lumina", "version": LUMINA_VERSION, "name": name,
              "rung": rung, "matrices": []}
    if extra_header:
        header.update(extra_header)
    blobs, idx, off = [], {}, 0
    for tname, (kind, payload) in payloads.items():
        if kind == "raw":
            a = np.ascontiguousarray(payload, dtype=np.float32)
            raw = a.tobytes()
            idx[tname] = {"kind": "raw", "dtype": "F32", "shape": list(a.shape),
                          "offset": off, "length": len(raw)}
            blobs.append(raw)
            off += len(raw)
            continue
        codes, scales = payload
        codes = np.ascontiguousarray(codes).astype(np.uint8)
        scales = np.ascontiguousarray(scales, dtype=np.float32)
        flag, shape = "none", list(codes.shape)
        if kind == "int4":
            cb, flag = pack_codes_nibble(codes).tobytes(), "nibble"
        elif kind == "int2":
            cb, flag = pack_codes_2bit(codes).tobytes(), "2bit"
        else:
            cb = codes.tobytes()
        sb = scales.tobytes()
        gs = int((group_sizes or {}).get(tname, group_size))
        idx[tname] = {"kind": kind, "codes_dtype": "uint8", "codes_shape": list(codes.shape),
                      "scales_dtype": "F32", "scales_shape": list(scales.shape),
                      "shape": shape, "packed": flag, "group_size": gs,
                      "offset": off, "codes_len": len(cb), "scales_len": len(sb)}
        blobs += [cb, sb]
        off += len(cb) + len(sb)
    header["tensors"] = idx
    hb = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<IIQ", LUMINA_MAGIC, LUMINA_VERSION, len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)


def read_header(path: str) -> tuple[dict, int]:
    """(header, offset of the blob area) — adapters/lumina.py:43-47,96-99."""
    with open(path, "rb") as f:
        magic, ver, hlen = struct.unpack("<IIQ", f.read(16))
        if magic != LUMINA_MAGIC:
            raise ValueError("not a .lumina file")
        return json.loads(f.read(hlen)), 16 + hlen


def load_dequant(path: str) -> dict[str, np.ndarray]:
    """Reference loader semantics: every tensor to fp32
    (adapters/lumina.py:95-159)."""
    hdr, base = read_header(path)
    with open(path, "rb") as f:
        f.seek(base)
        buf = f.read()
    out = {}
    for tname, info in hdr["tensors"].items():
        if info.get("kind") == "raw" or "kind" not in info:
            s, e = info["offset"], info["offset"] + info["length"]
            out[tname] = np.frombuffer(buf[s:e], dtype=np.float32).reshape(info["shape"])
            continue
        kind, gs = info["kind"], int(info.get("group_size", 64))
        s = info["offset"]
        e = s + info["codes_len"]
        scales = np.frombuffer(buf[e:e + info["scales_len"]], dtype=np.float32).reshape(info["scales_shape"])
        shape = [int(x) for x in info.get("shape", info["codes_shape"])]
        codes = unpack_codes(buf[s:e], (shape[0], shape[1]), info.get("packed", "none"))
        out[tname] = dequant(kind, codes, scales, gs)
    return out
