"""One rank of the tensor-parallel decode check (run under torchrun by
tests/test_gpu_tp.py): builds its shard of the tiny int4 model, maps the
other rank's exchange region, runs prefill, teacher-forced steps and a
device-chained greedy run, and writes its results to <out>.rank<r>.npz."""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path[:0] = [REPO, os.path.join(REPO, "lumina-studio_b200")]


class StubTok:
    def encode(self, p):
        return [int(t) for t in p]

    def decode(self, ids):
        return " ".join(map(str, ids))


def main(path, golden, out, shard_dir=None):
    """With ``shard_dir`` every rank loads its own shard file written there by
    shards.write_tp_shards (instead of slicing the full file at load)."""
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    from lumina_b200 import synthetic
    from lumina_b200.engine import CudaChatModel
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=torch.device(f"cuda:{local}"))
    g = np.load(golden)
    if shard_dir:
        base = os.path.splitext(os.path.basename(path))[0]
        path = os.path.join(shard_dir, f"{base}.tp{world}.rank{rank}.lumina")
    m = CudaChatModel.from_lumina(path, synthetic.hf_cfg(synthetic.TINY), StubTok(),
                                  theta=synthetic.TINY["rope_theta"], max_seq=512, max_rows=128, device=local,
                                  tp_rank=rank, tp_size=world)
    try:
        m.init_tp()
        prompt = [int(t) for t in g["prompt"]]
        res = {"prefill": m.forward(prompt, 0)[0].copy()}
        for s, tk in enumerate(int(t) for t in g["forced"][:4]):
            lg, am = m.decode_step(tk)
            res[f"step{s}"] = lg.copy()
            res[f"am{s}"] = np.int64(am)
        res["kv0_k"], res["kv0_v"] = m.kv_read(0, 0, m.kv_length())
        m.kv_truncate(len(prompt))
        res["greedy"] = np.asarray(m.decode_greedy(int(g["forced"][0]), 24), np.int64)
        np.savez(f"{out}.rank{rank}.npz", **res)
    finally:
        m.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main(*sys.argv[1:5])
