"""`.lumina` records straight to device memory.

Reads the container the reference writes (scripts/lumina_convert.py:100-165;
header ``<IIQ`` magic/version/length, JSON header, blobs) with the record
semantics of ``LuminaAdapter.load`` (src/lumina_framework/adapters/lumina.py:
95-159) — but quantized records are handed to the device packed, never
dequantized to fp32 on the host (the reference materialises fp32 at
lumina.py:135-150 and then fp16 at chat.py:140).
"""
from __future__ import annotations

import json
import mmap
import struct
from dataclasses import dataclass

import numpy as np

LUMINA_MAGIC = 0x4E494D4C  # adapters/lumina.py:16


@dataclass
class Record:
    name: str
    kind: str             # raw | int4 | int3 | int2 | binary
    shape: tuple          # logical (rows, cols) (raw: the array shape)
    group: int = 0
    pack: str = "none"
    codes: np.ndarray | None = None   # uint8 view of the codes blob
    scales: np.ndarray | None = None  # fp32 (rows, n_groups)
    data: np.ndarray | None = None    # raw fp32 tensor


class LuminaFile:
    """Memory-mapped `.lumina` file; records are zero-copy numpy views."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        head = self._f.read(16)
        if len(head) < 16:
            raise ValueError("not a .lumina file (short header): " + path)
        magic, self.version, hlen = struct.unpack("<IIQ", head)
        if magic != LUMINA_MAGIC:
            raise ValueError("not a .lumina file (magic %#x): %s" % (magic, path))
        self.header = json.loads(self._f.read(hlen))
        self.base = 16 + hlen
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self._buf = np.frombuffer(self._mm, dtype=np.uint8)
        self.tensors = self.header.get("tensors", {})

    def close(self):
        try:
            del self._buf
            self._mm.close()
            self._f.close()
        except Exception:  # noqa: BLE001
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def names(self):
        return list(self.tensors.keys())

    def _slice(self, off, n):
        s = self.base + int(off)
        return self._buf[s:s + int(n)]

    def record(self, name: str) -> Record:
        info = self.tensors[name]
        if ("codec" in info and info["codec"] == "f32-reference") or info.get("kind") == "raw" \
                or "kind" not in info:
            # raw fp32 (adapters/lumina.py:106-120, 153-158)
            arr = self._slice(info["offset"], info["length"]).view(np.float32).reshape(info["shape"])
            return Record(name, "raw", tuple(arr.shape), data=arr)
        kind = info.get("kind", "int4")
        gs = int(info.get("group_size", 64))
        codes = self._slice(info["offset"], info["codes_len"])
        scales = self._slice(int(info["offset"]) + int(info["codes_len"]), info["scales_len"]) \
            .view(np.float32).reshape(info["scales_shape"])
        shape = [int(x) for x in info.get("shape", info["codes_shape"])]
        rows = shape[0]
        if kind == "binary":
            # the stored shape is the packed sign-byte shape; the reader takes
            # the width from the scales (adapters/lumina.py:142-148), which only
            # loads when it equals 8 * packed bytes rounded to whole bytes
            cols = int(info["scales_shape"][1]) * gs
            if (cols + 7) // 8 != shape[1]:
                raise ValueError("%s: binary record of %d sign bytes per row with %d-column scale groups "
                                 "is not loadable (the reference loader rejects it too)" % (name, shape[1], cols))
        else:
            cols = shape[1]
        return Record(name, kind, (rows, cols), group=gs, pack=info.get("packed", "none"),
                      codes=codes, scales=scales)


def upload_record(rec: Record, device: int = 0):
    """A packed record to a device ``cuda.Weight``."""
    from .cuda import Weight
    if rec.kind == "raw":
        raise ValueError(rec.name + " is a raw tensor")
    return Weight.upload(rec.kind, rec.group, rec.pack, rec.codes, rec.scales, rec.shape[0],
                         rec.shape[1], device=device)
