"""Multi-GPU host logic on CPU: sessions sharded across ranks with no data-path
collective, run as world-size-2 `gloo` process groups (no GPU)."""
import os
import socket

import numpy as np
import pytest

from rpgbarengine_b200 import dist as rdist
from rpgbarengine_b200 import synth


def test_shards_cover_every_session_once():
    for n in (0, 1, 2, 5, 64):
        for world in (1, 2, 4, 8):
            got = sorted(i for r in range(world) for i in rdist.shard_sessions(n, r, world))
            assert got == list(range(n))
            sizes = [len(rdist.shard_sessions(n, r, world)) for r in range(world)]
            assert max(sizes) - min(sizes) <= 1


def test_shard_arguments_checked():
    with pytest.raises(ValueError):
        rdist.shard_sessions(4, 2, 2)
    with pytest.raises(ValueError):
        rdist.shard_sessions(4, 0, 0)
    with pytest.raises(ValueError):
        rdist.shard_sessions(-1, 0, 1)


def test_job_throughput_uses_slowest_rank():
    assert rdist.job_throughput(512, 8, 1000.0) == pytest.approx(4096.0)
    with pytest.raises(ValueError):
        rdist.job_throughput(1, 1, 0.0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _session_digest(index):
    """What a session computes depends on its global index only: its prompt."""
    ids = synth.prompt_ids(rdist.session_seed(42, index), 64)
    return int(np.bitwise_xor.reduce(ids.astype(np.int64) * (np.arange(64) + 1)))


def _rank(rank, world, port, n_sessions, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = rdist.shard_sessions(n_sessions, rank, world)
        results = {i: _session_digest(i) for i in mine}
        gathered = [None] * world
        dist.all_gather_object(gathered, results)
        # per-rank device times: rank r reports r+1 ms etc.; the job time is the max
        t = rdist.max_over_ranks([1.0 + rank, 10.0 - rank, 3.0], dist)
        q.put((rank, gathered, t))
    finally:
        dist.destroy_process_group()


def test_two_rank_sessions_match_single_rank():
    import torch.multiprocessing as mp
    world, n = 2, 7
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    single = {i: _session_digest(i) for i in rdist.shard_sessions(n, 0, 1)}
    for rank, gathered, t in out:
        merged = {}
        for part in gathered:
            assert not set(part) & set(merged)
            merged.update(part)
        assert merged == single
        assert t == [2.0, 10.0, 3.0]
