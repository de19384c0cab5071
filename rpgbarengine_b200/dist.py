"""Independent sessions sharded across GPUs: the multi-GPU plan of the token loop
for single-model serving (one process per GPU, weights replicated per GPU).

The reference runs every session of a model in one process on the host cores
(src/engine.cc:349-515, one generate at a time per session); its sessions share
nothing but the read-only weights.  Here session i of a job runs on rank
i % world.  There is no data-path collective: a session's tokens depend only on
its own prompt, options and seed, never on the world size or on which GPU runs
it.  The one collective is the max-over-ranks reduction of the timings after
the timed region.
"""
from __future__ import annotations

from dataclasses import dataclass


def shard_sessions(n_sessions: int, rank: int, world: int) -> list[int]:
    """Global indices of the sessions that rank `rank` of `world` runs
    (round-robin, so ranks differ by at most one session)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if n_sessions < 0:
        raise ValueError("negative session count")
    return list(range(rank, n_sessions, world))


def session_seed(base: int, index: int) -> int:
    """Prompt seed of global session `index`: a function of the session alone, so
    a session's prompt (and hence its tokens) is the same at every world size."""
    return base + index


@dataclass
class RankTimes:
    """Device times of one rank's timed region, in milliseconds."""
    total_ms: float
    prefill_ms: float
    decode_ms: float

    def as_list(self) -> list[float]:
        return [self.total_ms, self.prefill_ms, self.decode_ms]


def max_over_ranks(values: list[float], dist=None, device=None) -> list[float]:
    """Element-wise max of `values` over all ranks (one all-reduce MAX); the
    values unchanged without a process group.  Every rank must call it."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return list(values)
    import torch
    t = torch.tensor(values, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


def job_throughput(units_per_session: int, n_sessions: int, max_ms: float) -> float:
    """Whole-job throughput: the units every session processed over the slowest
    rank's time (units per second)."""
    if max_ms <= 0:
        raise ValueError("non-positive time")
    return units_per_session * n_sessions / (max_ms / 1e3)
