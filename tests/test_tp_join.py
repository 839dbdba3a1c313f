"""Failure detection of the tensor-parallel join, on the CPU (gloo ranks,
no GPU): the exchange of peer-memory handles that ``CudaChatModel.init_tp``
runs hands every rank's handle to every rank in rank order, and a rank
whose peer never arrives gets an error within the group's timeout instead
of waiting forever."""
import os
import socket
import time
from datetime import timedelta

import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, out, rank0_leaves):
    import torch.distributed as dist
    from lumina_b200.engine import gather_peer_handles
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    if rank0_leaves and rank == 0:
        return  # leaves before the exchange, without a word to the others
    t0 = time.time()
    try:
        got = gather_peer_handles(bytes([rank + 7]) * 64)
        msg = "ok " + "".join(h[:1].hex() for h in got)
    except Exception as e:  # noqa: BLE001
        msg = "error " + type(e).__name__
    with open(f"{out}.{rank}", "w") as f:
        f.write(f"{msg} {time.time() - t0:.1f}")
    try:
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        pass


def _run(tmp_path, rank0_leaves):
    out = str(tmp_path / "join")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out, rank0_leaves)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung in the handle exchange"
    return out


def test_handles_reach_every_rank(tmp_path):
    out = _run(tmp_path, rank0_leaves=False)
    for r in range(2):
        assert open(f"{out}.{r}").read().startswith("ok 0708"), r  # both handles, rank order


def test_missing_rank_raises_instead_of_hanging(tmp_path):
    out = _run(tmp_path, rank0_leaves=True)
    msg = open(f"{out}.1").read()
    assert msg.startswith("error"), msg
    assert float(msg.split()[-1]) < 60
