"""Multi-rank host logic with 2 gloo ranks on CPU: map sharding, the stats gather and the
max-over-ranks timing used by bench.py under torchrun (no GPU)."""
import os
import socket

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import datetime

    import torch
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from scenemap_b200 import dist
        maps = list(dist.rank_maps(rank, world, 3))
        stats = np.array([[m * 100 + k for k in range(16)] for m in maps], np.int64)
        allst = dist.gather_stats(stats, world)
        t = dist.max_over_ranks([1.0 + rank, 5.0 - rank], world)
        q.put((rank, maps, allst.tolist(), t))
    finally:
        torch.distributed.destroy_process_group()


def test_two_rank_shard_gather_and_max():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(2):
        r = q.get(timeout=120)
        res[r[0]] = r
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][1] == [0, 1, 2] and res[1][1] == [3, 4, 5]
    want = [[m * 100 + k for k in range(16)] for m in range(6)]
    assert res[0][2] == want and res[1][2] == want        # every rank sees all maps, rank order
    assert res[0][3] == [2.0, 5.0] and res[1][3] == [2.0, 5.0]


def test_rank_maps_rejects_bad_input():
    from scenemap_b200 import dist
    with pytest.raises(ValueError):
        dist.rank_maps(2, 2, 4)
