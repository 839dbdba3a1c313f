"""Tensor-parallel shard rules and the exchange step, on the CPU.

Two gloo ranks (world size 2, 127.0.0.1) each take their shard of the tiny
int4 model's projections with ``sharding.shard_record`` and dequantize it
with the oracle. Column-parallel shards (q/k/v by heads, gate/up by
group-aligned FFN rows, lm_head by vocab) concatenate to the full output;
row-parallel shards (o_proj, down by group-aligned K ranges) give partial
products whose all-reduce (sum, the same step the library runs through
NCCL after o_proj and down_proj) equals the full product. Uneven splits
(FFN 688 = 10.75 groups of 64) are covered, and at TP 8 the 7B FFN split
(172 groups) is checked for group alignment and coverage.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import lumina_format as lf
from lumina_b200 import sharding
from lumina_b200.loader import LuminaFile

HD = 64


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _deq(rec):
    if rec.kind == "binary":
        codes = rec.codes.reshape(rec.shape[0], -1)
    else:
        codes = lf.unpack_codes(rec.codes, rec.shape, rec.pack)
    return lf.dequant(rec.kind, codes, rec.scales, rec.group, rec.shape[1])


def _worker(rank, world, port, path, out):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        f = LuminaFile(path)
        rng = np.random.default_rng(0)
        x = rng.standard_normal((2, 688)).astype(np.float32)
        h = rng.standard_normal((2, 256)).astype(np.float32)
        res = {}
        p = "model.layers.1."
        for nm, inp in (("self_attn.o_proj.weight", h), ("mlp.down_proj.weight", x)):
            rec = f.record(p + nm)
            sh = sharding.shard_record(rec, nm, rank, world, HD)
            c0 = (rank * rec.shape[1] // world) if "o_proj" in nm else \
                sharding.ffn_bounds(rec.shape[1], rec.group, rank, world)[0]
            part = torch.from_numpy(inp[:, c0:c0 + sh.shape[1]] @ _deq(sh).T)
            dist.all_reduce(part)  # the row-parallel exchange step
            res[nm] = part.numpy()
        for nm in ("self_attn.q_proj.weight", "mlp.gate_proj.weight"):
            sh = sharding.shard_record(f.record(p + nm), nm, rank, world, HD)
            y = torch.from_numpy(h @ _deq(sh).T)
            parts = [None] * world
            dist.all_gather_object(parts, y.numpy())
            res[nm] = np.concatenate(parts, axis=1)
        head = f.record("lm_head.weight").data
        parts = [None] * world
        dist.all_gather_object(parts, h @ sharding.vocab_shard(head, rank, world).T)
        res["lm_head.weight"] = np.concatenate(parts, axis=1)
        if rank == 0:
            np.savez(out, **res)
    finally:
        dist.destroy_process_group()


def test_tp2_shards_reassemble_full_products(tiny_file, tmp_path):
    out = str(tmp_path / "tp.npz")
    mp.start_processes(_worker, args=(2, _free_port(), tiny_file, out), nprocs=2, start_method="spawn")
    got = np.load(out)
    full = lf.load_dequant(tiny_file)
    rng = np.random.default_rng(0)
    x = rng.standard_normal((2, 688)).astype(np.float32)
    h = rng.standard_normal((2, 256)).astype(np.float32)
    p = "model.layers.1."
    np.testing.assert_allclose(got["self_attn.o_proj.weight"], h @ full[p + "self_attn.o_proj.weight"].T,
                               rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(got["mlp.down_proj.weight"], x @ full[p + "mlp.down_proj.weight"].T,
                               rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(got["self_attn.q_proj.weight"], h @ full[p + "self_attn.q_proj.weight"].T,
                               rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(got["mlp.gate_proj.weight"], h @ full[p + "mlp.gate_proj.weight"].T,
                               rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(got["lm_head.weight"], h @ full["lm_head.weight"].T, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("ffn,group,tp", [(11008, 64, 8), (11008, 64, 4), (11008, 128, 2), (688, 64, 2),
                                          (11008, 128, 8)])
def test_ffn_bounds_cover_group_aligned(ffn, group, tp):
    b = [sharding.ffn_bounds(ffn, group, r, tp) for r in range(tp)]
    assert b[0][0] == 0 and b[-1][1] == ffn
    for (a0, a1), (c0, _) in zip(b, b[1:]):
        assert a1 == c0 and a0 % group == 0 and c0 % group == 0
    sizes = [e - s for s, e in b]
    # one whole group apart at most (plus the short last group)
    assert max(sizes) - min(sizes) <= group + (-ffn % group)


def test_shard_files_hold_each_ranks_slice(tiny_file, tmp_path):
    """write_tp_shards: every rank's file holds exactly shard_record's slice
    of each projection (codes as stored, scales), the vocab slice of the
    head, the replicated raw tensors, and the tp_shard marker the loader
    checks."""
    from lumina_b200 import sharding
    from lumina_b200.loader import LuminaFile
    from lumina_b200.shards import _SHARDED, _layer_part, write_tp_shards
    for tp in (2, 4):
        paths = write_tp_shards(tiny_file, tp, 64, str(tmp_path / f"tp{tp}"))
        assert len(paths) == tp
        with LuminaFile(tiny_file) as full:
            for r, p in enumerate(paths):
                with LuminaFile(p) as f:
                    assert f.header["tp_shard"] == {"rank": r, "size": tp}
                    assert sorted(f.names()) == sorted(full.names())
                    for n in full.names():
                        a, b = full.record(n), f.record(n)
                        if a.kind == "raw":
                            want = sharding.vocab_shard(a.data, r, tp) if n == "lm_head.weight" else a.data
                            assert b.kind == "raw" and np.array_equal(b.data, want), n
                            continue
                        part = _layer_part(n)
                        w = sharding.shard_record(a, part, r, tp, 64) if part in _SHARDED else a
                        assert (b.kind, b.shape, b.group, b.pack) == (w.kind, w.shape, w.group, w.pack), n
                        assert np.array_equal(b.codes, w.codes) and np.array_equal(b.scales, w.scales), n


def test_expert_shards_sum_to_the_routed_mlp(tiny_moe_file):
    """Expert parallelism (sharding.expert_shard): at TP 2 and 4 each rank
    keeps E/tp whole experts of gate_up and down; the ranks' shares of the
    routed MLP (the top-k experts a rank holds, others contributing zero)
    add up to the full routed MLP of the oracle for a random normalized
    row, and the shard rows concatenate to the full records."""
    from lumina_b200.engine import moe_map_from_header
    rng = np.random.default_rng(7)
    with LuminaFile(tiny_moe_file) as f:
        mm = moe_map_from_header(f.header)[0]
        E, ie, K = mm["experts"], mm["ie"], mm["top_k"]
        gu = f.record("model.layers.0.mlp.experts.gate_up_proj")
        dn = f.record("model.layers.0.mlp.experts.down_proj")
        router = np.asarray(f.record("model.layers.0.mlp.gate.weight").data, np.float64)
    h = rng.standard_normal(gu.shape[1])
    score = 1.0 / (1.0 + np.exp(-(router @ h)))
    picks = np.argsort(-score)[:K]

    def mlp_share(gu_w, dn_w, experts):
        y = np.zeros(dn_w.shape[1])
        for j, e in enumerate(experts):
            if e not in picks:
                continue
            g = gu_w[2 * ie * j:2 * ie * j + ie] @ h
            u = gu_w[2 * ie * j + ie:2 * ie * (j + 1)] @ h
            a = g / (1.0 + np.exp(-np.clip(g, -40, 40))) * u
            y += dn_w[ie * j:ie * (j + 1)].T @ a
        return y

    full = mlp_share(_deq(gu).astype(np.float64), _deq(dn).astype(np.float64), list(range(E)))
    for tp in (2, 4):
        parts, rows_gu, rows_dn = [], [], []
        for r in range(tp):
            g_r = sharding.expert_shard(gu, E, r, tp)
            d_r = sharding.expert_shard(dn, E, r, tp)
            assert g_r.shape == (E // tp * 2 * ie, gu.shape[1]) and d_r.shape == (E // tp * ie, dn.shape[1])
            rows_gu.append(_deq(g_r))
            rows_dn.append(_deq(d_r))
            parts.append(mlp_share(rows_gu[-1].astype(np.float64), rows_dn[-1].astype(np.float64),
                                   list(range(r * E // tp, (r + 1) * E // tp))))
        assert np.array_equal(np.concatenate(rows_gu), _deq(gu))
        assert np.array_equal(np.concatenate(rows_dn), _deq(dn))
        np.testing.assert_allclose(sum(parts), full, rtol=1e-12, atol=1e-12)
    with pytest.raises(ValueError, match="do not split"):
        sharding.expert_shard(gu, E, 0, 3)


def test_shard_files_hold_each_ranks_experts(tiny_moe_file, tmp_path):
    """write_tp_shards on a virtual-MoE model: each rank's file holds its
    experts' rows of gate_up and down (expert_shard), the whole router, and
    the virtual_moe header map the loader reads."""
    from lumina_b200.engine import moe_map_from_header
    from lumina_b200.shards import write_tp_shards
    paths = write_tp_shards(tiny_moe_file, 2, HD, str(tmp_path / "moe_tp2"))
    with LuminaFile(tiny_moe_file) as full:
        moe = moe_map_from_header(full.header)
        for r, p in enumerate(paths):
            with LuminaFile(p) as f:
                assert moe_map_from_header(f.header) == moe
                for l, mm in moe.items():
                    for nm in ("mlp.experts.gate_up_proj", "mlp.experts.down_proj"):
                        n = f"model.layers.{l}.{nm}"
                        w = sharding.expert_shard(full.record(n), mm["experts"], r, 2)
                        b = f.record(n)
                        assert b.shape == w.shape and np.array_equal(b.codes, w.codes), n
                        assert np.array_equal(b.scales, w.scales), n
                    n = f"model.layers.{l}.mlp.gate.weight"
                    assert np.array_equal(f.record(n).data, full.record(n).data)
