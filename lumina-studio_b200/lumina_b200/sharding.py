"""Tensor-parallel shards of `.lumina` records (no reference counterpart:
the reference has no multi-device code).

Column-parallel (rows split): q/k/v by heads, gate/up by group-aligned FFN
slices, lm_head by vocab. Row-parallel (columns split at scale-group
boundaries, so no group is ever cut): o by heads, down by the same FFN
slices as gate/up. When the FFN group count does not divide by the TP size
(11008 / 64 = 172 groups at TP 8) the first ranks take one group more.
Virtual-MoE layers split by experts (expert parallelism): each rank keeps
E/tp whole experts of gate_up and down and the whole router.
"""
from __future__ import annotations

import numpy as np

from .loader import Record

BITS = {"int4": 4, "int3": 8, "int2": 2, "binary": 1}  # stored bits per code in the file


def ffn_bounds(ffn: int, group: int, rank: int, tp: int) -> tuple[int, int]:
    ng = (ffn + group - 1) // group
    base, extra = divmod(ng, tp)
    g0 = rank * base + min(rank, extra)
    g1 = g0 + base + (1 if rank < extra else 0)
    return min(g0 * group, ffn), min(g1 * group, ffn)


def _rows(rec: Record, r0: int, r1: int) -> Record:
    rows = rec.shape[0]
    stride = rec.codes.size // rows
    codes = np.ascontiguousarray(rec.codes.reshape(rows, stride)[r0:r1])
    return Record(rec.name, rec.kind, (r1 - r0, rec.shape[1]), rec.group, rec.pack,
                  codes.reshape(-1), np.ascontiguousarray(rec.scales[r0:r1]))


def _cols(rec: Record, c0: int, c1: int) -> Record:
    if c0 % rec.group:
        raise ValueError(f"{rec.name}: column shard at {c0} is not group aligned")
    rows = rec.shape[0]
    stride = rec.codes.size // rows
    bits = BITS[rec.kind]
    b0 = c0 * bits // 8
    b1 = min(stride, (c1 * bits + 7) // 8)
    codes = np.ascontiguousarray(rec.codes.reshape(rows, stride)[:, b0:b1])
    g0, g1 = c0 // rec.group, (c1 + rec.group - 1) // rec.group
    return Record(rec.name, rec.kind, (rows, c1 - c0), rec.group, rec.pack, codes.reshape(-1),
                  np.ascontiguousarray(rec.scales[:, g0:g1]))


def shard_record(rec: Record, what: str, rank: int, tp: int, head_dim: int) -> Record:
    if tp <= 1:
        return rec
    rows, cols = rec.shape
    if what in ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight"):
        per = rows // tp
        if per * tp != rows or per % head_dim:
            raise ValueError(f"{rec.name}: {rows} rows do not split into whole heads over {tp} ranks")
        return _rows(rec, rank * per, (rank + 1) * per)
    if what in ("mlp.gate_proj.weight", "mlp.up_proj.weight"):
        r0, r1 = ffn_bounds(rows, rec.group, rank, tp)
        return _rows(rec, r0, r1)
    if what == "self_attn.o_proj.weight":
        per = cols // tp
        return _cols(rec, rank * per, (rank + 1) * per)
    if what == "mlp.down_proj.weight":
        c0, c1 = ffn_bounds(cols, rec.group, rank, tp)
        return _cols(rec, c0, c1)
    raise ValueError("no shard rule for " + what)


def expert_shard(rec: Record, experts: int, rank: int, tp: int) -> Record:
    """Expert parallelism for a virtual-MoE layer: rank r keeps the rows of
    experts [r E/tp, (r+1) E/tp) of the flat experts.gate_up_proj (E*2Ie
    rows) or experts.down_proj (E*Ie rows); the router stays whole."""
    if tp <= 1:
        return rec
    if experts % tp:
        raise ValueError(f"{rec.name}: {experts} experts do not split over {tp} ranks")
    rows = rec.shape[0]
    if rows % experts:
        raise ValueError(f"{rec.name}: {rows} rows are not {experts} experts")
    per = rows // experts * (experts // tp)
    return _rows(rec, rank * per, (rank + 1) * per)


def vocab_shard(head: np.ndarray, rank: int, tp: int) -> np.ndarray:
    if tp <= 1:
        return head
    V = head.shape[0]
    if V % tp:
        raise ValueError(f"vocab {V} does not split over {tp} ranks")
    per = V // tp
    return np.ascontiguousarray(head[rank * per:(rank + 1) * per])
