"""Multi-process host logic of the batch-sharded job on CPU (gloo, world size 2): the shard
ranges, the rank-ordered gather of the output latents, and failure detection when a rank dies
before the gather (the survivor gets an error within the process-group timeout, not a hang)."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch

    from mtorch_b200 import parallel

    try:
        dist = parallel.init("gloo", timeout_s=10.0)
        lo, hi = parallel.shard(8, world, rank)
        # each rank's "latents": the sample indices it owns, as bytes
        local = torch.from_numpy(np.arange(lo, hi, dtype=np.int64).view(np.uint8).copy())
        if mode == "die" and rank == 1:
            os._exit(0)  # leaves between steps, with nothing in flight
        out = parallel.gather_shards(local)
        q.put((rank, "ok", out.numpy().view(np.int64).tolist()))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", type(e).__name__))


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    for p in procs:
        p.join(timeout=120)
    while not q.empty():
        results.append(q.get())
    for p in procs:
        if p.is_alive():
            p.kill()
    return sorted(results)


def test_shard_ranges():
    from mtorch_b200 import parallel

    assert [parallel.shard(64, 8, r) for r in (0, 7)] == [(0, 8), (56, 64)]
    with pytest.raises(ValueError):
        parallel.shard(64, 3, 0)


def test_gather_is_rank_ordered():
    res = _run("ok")
    assert [r[1] for r in res] == ["ok", "ok"]
    for _, _, vals in res:
        assert vals == list(range(8))


def test_dead_rank_is_an_error_not_a_hang():
    res = _run("die")
    assert len(res) == 1 and res[0][0] == 0
    assert res[0][1] == "error"
