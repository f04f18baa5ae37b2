"""Multi-rank host logic on CPU: world_size-2 gloo process groups run the same
shard -> per-rank work -> ordered gather -> max-over-ranks path that the
multi-GPU bench and engine use, with a CPU stand-in for the per-rank device
session (units are independent, so there is no data-path collective)."""
import os
import socket

import numpy as np
import pytest

from qppocr_b200.shard import gather_shards, local_shard, max_over_ranks, shard_bounds


def test_shard_bounds_cover_exactly_once():
    for n in (0, 1, 2, 7, 64, 4096, 4097):
        for world in (1, 2, 3, 8):
            seen = []
            sizes = []
            for r in range(world):
                a, b = shard_bounds(n, world, r)
                seen.extend(range(a, b))
                sizes.append(b - a)
            assert seen == list(range(n))
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_units, q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        units = np.arange(n_units, dtype=np.int64)
        mine = local_shard(units, world, rank)
        # stand-in for this rank's device session: a per-unit result
        results = [int(u) * 3 + 1 for u in mine]
        gathered = gather_shards(results, world, rank)
        t = max_over_ranks(float(rank + 1) * 0.5, world)
        q.put((rank, gathered, t, len(mine)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_units", [10, 7, 1])
def test_gloo_world2_shard_gather(n_units):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n_units, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in procs:
        rank, gathered, t, n_local = q.get(timeout=120)
        out[rank] = (gathered, t, n_local)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert out[0][0] == [u * 3 + 1 for u in range(n_units)]
    assert out[1][0] is None
    assert out[0][1] == out[1][1] == 1.0  # max over ranks of 0.5, 1.0
    assert out[0][2] + out[1][2] == n_units
