"""Tensor-parallel shard files: one `.lumina` file per rank.

``write_tp_shards`` reads a `.lumina` model once and writes, for each of
``tp`` ranks, a `.lumina` file holding only that rank's slice of every
projection (the column / row split of ``sharding.shard_record``, packed codes
copied as stored, never dequantized), its experts of every virtual-MoE layer
(``sharding.expert_shard``), its vocab slice of ``lm_head``, and the
replicated raw tensors (embedding, norms, routers). The header carries
``"tp_shard": {"rank": r, "size": tp}``; ``CudaChatModel.from_lumina`` then
loads the file as that rank's shard without slicing again, so each rank reads
about 1/tp of the projection bytes. The reference has no multi-device path;
the container is the reference's (scripts/lumina_convert.py:100-165): magic,
JSON header, then each record's codes blob followed by its F32 scales.
"""
from __future__ import annotations

import json
import os
import re
import struct

import numpy as np

from .loader import LUMINA_MAGIC, LuminaFile, Record
from . import sharding

_SHARDED = ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
            "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight")


def _layer_part(name: str) -> str | None:
    m = re.match(r"model\.layers\.\d+\.(.+)$", name)
    return m.group(1) if m else None


def _entry(rec: Record, info: dict, off: int) -> tuple[dict, list]:
    """Header entry and blobs of one record at blob offset ``off``."""
    if rec.kind == "raw":
        a = np.ascontiguousarray(rec.data, dtype=np.float32)
        return ({"kind": "raw", "dtype": "F32", "shape": list(a.shape), "offset": off,
                 "length": a.nbytes}, [a.tobytes()])
    rows, cols = rec.shape
    codes = np.ascontiguousarray(rec.codes, dtype=np.uint8)
    scales = np.ascontiguousarray(rec.scales, dtype=np.float32)
    if rec.kind == "binary":
        stored = [rows, codes.size // rows]  # the packed sign-byte shape the reader expects
    else:
        stored = [rows, cols]
    e = {"kind": rec.kind, "codes_dtype": "uint8", "codes_shape": stored, "scales_dtype": "F32",
         "scales_shape": list(scales.shape), "shape": stored, "packed": rec.pack,
         "group_size": int(rec.group), "offset": off, "codes_len": codes.nbytes, "scales_len": scales.nbytes}
    return e, [codes.tobytes(), scales.tobytes()]


def write_tp_shards(path: str, tp: int, head_dim: int, out_dir: str) -> list[str]:
    """Write ``tp`` shard files of the model at ``path`` into ``out_dir``;
    returns their paths in rank order."""
    if tp < 1:
        raise ValueError("tp must be >= 1")
    os.makedirs(out_dir, exist_ok=True)
    base = os.path.splitext(os.path.basename(path))[0]
    out = []
    with LuminaFile(path) as f:
        names = f.names()
        from .engine import moe_map_from_header
        moe = moe_map_from_header(f.header)  # virtual-MoE layers split by experts
        for r in range(tp):
            header = {k: v for k, v in f.header.items() if k not in ("tensors", "matrices")}
            header["matrices"] = []
            header["tp_shard"] = {"rank": r, "size": tp}
            idx, blobs, off = {}, [], 0
            for n in names:
                rec = f.record(n)
                part = _layer_part(n)
                if rec.kind != "raw" and part in _SHARDED:
                    rec = sharding.shard_record(rec, part, r, tp, head_dim)
                elif rec.kind != "raw" and part in ("mlp.experts.gate_up_proj", "mlp.experts.down_proj"):
                    layer = int(n.split(".")[2])
                    rec = sharding.expert_shard(rec, moe[layer]["experts"], r, tp)
                elif rec.kind == "raw" and n == "lm_head.weight":
                    rec = Record(n, "raw", rec.shape, data=sharding.vocab_shard(np.asarray(rec.data), r, tp))
                e, b = _entry(rec, f.tensors[n], off)
                idx[n] = e
                blobs += b
                off += sum(len(x) for x in b)
            header["tensors"] = idx
            hb = json.dumps(header).encode()
            p = os.path.join(out_dir, f"{base}.tp{tp}.rank{r}.lumina")
            with open(p, "wb") as fo:
                fo.write(struct.pack("<IIQ", LUMINA_MAGIC, int(f.version), len(hb)))
                fo.write(hb)
                for x in blobs:
                    fo.write(x)
            out.append(p)
    return out
