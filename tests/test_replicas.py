"""Replica helpers over two gloo ranks on CPU (the multi-GPU path has no data-path
collective; only the work split and the job timing are shared between ranks)."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from conftest import ROOT  # noqa: F401  (puts the package on sys.path)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, lens, q):
    import datetime
    import torch.distributed as dist
    from julia1 import replicas
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        share = replicas.rank_share(lens, 8, 2000, rank, world)
        units = sum(lens[i] for b in share for i in b)
        secs = 1.0 + rank  # rank 1 is the slow one
        slowest = replicas.max_over_ranks(secs)
        rate = replicas.aggregate_rate(units, secs)
        q.put((rank, share, units, slowest, rate))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_split_and_time():
    import numpy as np
    import julia1 as j1
    lens = np.random.default_rng(3).integers(1, 512, size=97).tolist()
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, lens, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, share, units, slowest, rate = q.get(timeout=120)
        out[r] = (share, units, slowest, rate)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # every row runs exactly once across the ranks, in Engine::batches micro-batches
    rows = sorted(i for r in out for b in out[r][0] for i in b)
    assert rows == list(range(len(lens)))
    batches, devices = j1.plan_batches(lens, 8, 2000, world)
    for r in range(world):
        assert out[r][0] == [b for b, d in zip(batches, devices) if d == r]
    # greedy balance keeps the two shares within one micro-batch of each other
    assert abs(out[0][1] - out[1][1]) <= 2000
    total = out[0][1] + out[1][1]
    for r in range(world):
        assert out[r][2] == 2.0
        assert out[r][3] == pytest.approx(total / 2.0)


def test_single_process_fallbacks():
    from julia1 import replicas
    assert replicas.max_over_ranks(3.5) == 3.5
    assert replicas.aggregate_rate(100, 4.0) == 25.0
