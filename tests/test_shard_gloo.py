"""The N>1 path on the CPU: two ranks over gloo (one process each, as torchrun runs one per GPU), each stepping its
own shard of envs with its rank seed (rl/train.py:356) through the CPU oracle, with the per-rollout counter all-reduce
of ghostrun-lab_b200/shard.py. The reduced totals equal the sum of the two shards run one after another in one
process, and the shards draw different episodes."""
from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

ROLLOUT, ROLLOUTS, ENVS, SEED = 20, 3, 8, 3


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _shard(rank, oracle):
    from rlenv import RlEnv
    from actions import random_legal
    from shard import EpisodeCounters, rank_seed
    env = RlEnv({'synth00': ENVS}, device='cpu', lib_path=oracle, seed=rank_seed(SEED, rank), sticky=True,
                idle_max=30, dropout=True)
    env.start()
    gen = torch.Generator().manual_seed(SEED + rank)
    ctr = EpisodeCounters('cpu')
    rewards = []
    for r in range(ROLLOUTS):
        for _ in range(ROLLOUT):
            env.actions.copy_(random_legal(env.masks, gen))
            env.step()
            ctr.account(env)
            rewards.append(env.reward.clone())
        yield ctr, torch.stack(rewards)


def _worker(rank, world, port, oracle, out):
    import sys
    sys.path[:0] = out['paths']
    import torch.distributed as dist
    dist.init_process_group('gloo', init_method=f'tcp://127.0.0.1:{port}', rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        totals = []
        for ctr, rewards in _shard(rank, oracle):
            ctr.rollout_end()
            totals.append(ctr.total.clone())
        torch.save(dict(totals=torch.stack(totals), rewards=rewards), out['file'].format(rank=rank))
    finally:
        dist.destroy_process_group()


def test_two_rank_counters_equal_sum_of_shards(oracle_path, tmp_path):
    import sys
    os.environ.setdefault('OMP_NUM_THREADS', '2')
    out = dict(paths=list(sys.path[:3]), file=str(tmp_path / 'rank{rank}.pt'))
    port = _free_port()
    ctx = mp.get_context('spawn')
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(oracle_path), out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0, f'rank process exited with {p.exitcode}'
    res = [torch.load(out['file'].format(rank=r)) for r in range(2)]
    assert torch.equal(res[0]['totals'], res[1]['totals']), 'every rank holds the same reduced totals'
    # the same two shards, one after the other, summed without any collective
    want = []
    shards = [_shard(r, str(oracle_path)) for r in range(2)]
    for _ in range(ROLLOUTS):
        parts = [next(s) for s in shards]
        for ctr, _ in parts:
            ctr.rollout_end()          # no process group here: local totals only
        want.append(parts[0][0].total + parts[1][0].total)
        rewards = [p[1] for p in parts]
    assert torch.equal(res[0]['totals'], torch.stack(want))
    assert torch.equal(res[0]['rewards'], rewards[0]) and torch.equal(res[1]['rewards'], rewards[1])
    assert not torch.equal(rewards[0], rewards[1]), 'rank seeds must give the shards different episodes'
