"""Host-side logic of the N>1 path, as world_size-2 gloo ranks on the CPU:
request shards are disjoint and cover the global set, and the reported step
time is the max over ranks."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from specdec_b200.shard import max_over_ranks, request_range, shard
from specdec_b200.synth import make_prompts


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    per = 4
    glob = make_prompts(per * world, 5, 100, seed=1)
    mine = shard(glob, per, rank, world)
    import torch

    got = [torch.zeros_like(torch.from_numpy(mine)) for _ in range(world)]
    dist.all_gather(got, torch.from_numpy(mine))
    step_ms = [10.0 + rank, 5.0 * (world - rank)]
    mx = max_over_ranks(step_ms, dist)
    if rank == 0:
        q.put((np.concatenate([g.numpy() for g in got]), glob, mx))
    dist.barrier()
    dist.destroy_process_group()


def test_request_shards_and_max_timing():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    gathered, glob, mx = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert np.array_equal(gathered, glob)
    assert mx == [11.0, 10.0]


def test_request_range_validation():
    assert request_range(8, 3, 4) == (24, 32)
    with pytest.raises(ValueError):
        request_range(8, 4, 4)
    with pytest.raises(ValueError):
        shard(np.zeros((7, 2)), 4, 1, 2)
