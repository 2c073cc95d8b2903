"""Multi-rank host logic on CPU (gloo, world size 2): shard planning,
max-over-ranks timing, the all-gather assembly, and failure detection when a
rank dies (the survivors' next collective ends with an error within the
process-group timeout instead of hanging)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from mlk2_b200 import dist as mdist


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shards_partition_exactly():
    for units in (0, 1, 7, 65536, 2**28 + 3):
        for world in (1, 2, 3, 4, 8):
            spans = [mdist.shard(units, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == units
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c and a <= b
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        mdist.shard(10, 2, 2)


def _worker(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import torch

    try:
        dist = mdist.init("gloo", rank, timeout_s=10.0)
        if mode == "ok":
            t = mdist.max_over_ranks(float(rank) + 0.5, dist)
            b, e = mdist.shard(10, world, rank)
            local = torch.arange(b, e, dtype=torch.float32)
            full = mdist.all_gather_shards(local, dist)
            q.put((rank, t, full.tolist()))
        else:
            if rank == 1:
                raise RuntimeError("rank 1 fails before its collective")
            mdist.max_over_ranks(1.0, dist)  # waits for the dead rank
            q.put((rank, "no-error"))
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent, never swallowed
        q.put((rank, "error", type(exc).__name__))


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=90) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda t: t[0])


def test_two_rank_max_and_gather():
    out = _run("ok")
    assert [o[1] for o in out] == [1.5, 1.5]
    for o in out:
        assert o[2] == list(np.arange(10, dtype=np.float32))


def test_dead_rank_is_detected_not_hung():
    out = _run("fail")
    assert out[1][1] == "error"                 # the failing rank reports itself
    assert out[0][1] == "error"                 # the survivor's collective errors out
