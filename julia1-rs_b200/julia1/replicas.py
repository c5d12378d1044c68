"""Replica (one process per GPU) helpers.

The encoder forward has no cross-sequence exchange, so N GPUs run N independent
replicas: every rank owns whole micro-batches and nothing crosses NVLink on the
data path. The host-side pieces live here so that they can be tested with gloo
ranks on CPU:

* `rank_share` deals the micro-batches of Engine::batches (src/engine.rs:191-210)
  to ranks with the same greedy token balance the in-process pool uses
  (j1_plan_batches), so a multi-process job and a pool engine split work alike;
* `max_over_ranks` / `aggregate_rate` implement the timing rule for a job: the
  slowest rank's time, and units processed by all ranks over that time.
"""
import torch
import torch.distributed as dist

from . import plan_batches


def rank_share(row_lens, batch_size, max_batch_tokens, rank, world):
    """The micro-batches (lists of row indices, ascending length) rank `rank` runs."""
    batches, devices = plan_batches(row_lens, batch_size, max_batch_tokens, world)
    return [b for b, d in zip(batches, devices) if d == rank]


def max_over_ranks(x, device=None):
    """Largest `x` over the default process group (x itself without one)."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(x)
    v = torch.tensor([float(x)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(v, op=dist.ReduceOp.MAX)
    return float(v.item())


def aggregate_rate(units_this_rank, seconds_this_rank, device=None):
    """Whole-job throughput: units summed over ranks / the slowest rank's time."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(units_this_rank) / float(seconds_this_rank)
    v = torch.tensor([float(units_this_rank), float(seconds_this_rank)], dtype=torch.float64,
                     device=device or "cpu")
    u = v[:1].clone()
    s = v[1:].clone()
    dist.all_reduce(u, op=dist.ReduceOp.SUM)
    dist.all_reduce(s, op=dist.ReduceOp.MAX)
    return float(u.item()) / float(s.item())
