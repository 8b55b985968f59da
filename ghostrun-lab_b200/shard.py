"""Data-parallel sharding of the env step: one process per GPU, every rank steps its own envs, and the only exchange
is one all-reduce of scalar episode counters per rollout (rl/train.py:331-450: per-rank seed seed * 7919 + rank,
`dist.all_reduce` of the rollout statistics). The env step itself has no collective: envs are independent.

    ctr = EpisodeCounters(device)
    for t in range(T):
        env.step(); ctr.account(env)
    ctr.rollout_end()         # sum over ranks into ctr.total (no collective with one process)
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

FIELDS = ('finished', 'deaths', 'return_sum', 'level_events')


def rank_seed(seed: int, rank: int) -> int:
    """The env run seed of a rank (rl/train.py:356): envs of different ranks draw different episodes."""
    return int(seed) * 7919 + int(rank)


class EpisodeCounters:
    """Per-rollout episode statistics of this rank's envs, accumulated on the env's device without host syncs:
    finished episodes, deaths of finished episodes, summed returns of finished episodes, level events. float64, so
    integer counts stay exact. `rollout_end` sums the rollout's counters over the ranks into the job totals."""

    def __init__(self, device):
        self.v = torch.zeros(len(FIELDS), dtype=torch.float64, device=device)       # this rollout, this rank
        self.total = torch.zeros(len(FIELDS), dtype=torch.float64, device=device)   # all finished rollouts, all ranks
        self._attached = None

    def attach(self, env) -> bool:
        """Let the GPU library add each decision's counters in its finishing kernel (rlenv_bind_episode_counters):
        account() then has nothing to do for this env. False (torch reductions per decision) on a library without it."""
        fn = getattr(env.lib, 'rlenv_bind_episode_counters', None)
        if fn is None or self.v.device.type != 'cuda':
            return False
        fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        fn(env.h, ctypes.c_void_p(self.v.data_ptr()))
        env._counters_keep = self.v
        self._attached = env
        return True

    def account(self, env):
        if env is self._attached:
            return
        d = env.done.bool()
        self.v[0] += d.sum()
        self.v[1] += torch.where(d, env.info[:, 3], 0).sum()
        self.v[2] += torch.where(d, env.info[:, 0], 0).sum()
        self.v[3] += (env.events & 2).ne(0).sum()

    def rollout_end(self):
        """All-reduce (sum) this rollout's counters over the default process group (every rank calls it at the same
        point; no-op without one), add them to the totals and start the next rollout."""
        if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
            dist.all_reduce(self.v)
        self.total += self.v
        self.v.zero_()
        return self

    def as_dict(self):
        return {k: float(x) for k, x in zip(FIELDS, self.total.tolist())}
