"""Statistics over env shards held by several processes (one GPU each), outside the control step.

The step itself has no collective: envs are independent and every rank steps its own shard (global env ids through
NRB200Engine.set_env_offset, as isaac_net/core/sharded.py:61-77).  What crosses ranks is bookkeeping, done between
steps or at the end of an episode, over torch.distributed (NCCL over NVLink on GPU ranks, gloo on CPU):

  global_counters(engine)       counters() of the whole batch: one all_reduce of the summed counter words and the
                                PRBs offered
  gather_env_rows(t)            a per-env tensor [E_shard, ...] of every rank, concatenated in global env order on
                                every rank (one all_gather; shards must be equal-sized, as bench.py makes them)

The reference's ShardedEngine concatenates every step's outputs on its first device (sharded.py:130-140); these
helpers are the opt-in, per-episode form of that and are never part of a timed step.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def global_counters(engine, group=None):
    """engine.counters() summed over every rank of the process group (every rank gets the result)."""
    c = engine.ctr.sum(0).to(torch.float64)
    v = torch.cat([c, torch.tensor([float(engine.prb_avail)], dtype=torch.float64, device=c.device)])
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(v, op=dist.ReduceOp.SUM, group=group)
    return engine.fold_counters(v[:-1].round().long(), float(v[-1]))


def gather_env_rows(t, group=None):
    """[E_shard, ...] on every rank -> [world * E_shard, ...] in rank (global env id) order, on every rank."""
    if not (dist.is_available() and dist.is_initialized()):
        return t.clone()
    world = dist.get_world_size(group)
    out = torch.empty((world * t.shape[0], *t.shape[1:]), dtype=t.dtype, device=t.device)
    dist.all_gather_into_tensor(out, t.contiguous(), group=group)
    return out


__all__ = ["global_counters", "gather_env_rows"]
