"""GPU env == CPU oracle, bit for bit: every output of every decision (pictures, emphasis, reward, done, masks,
dropout timeline, pad bytes, events, reward parts, and info where done) and the canonical machine dumps (CPU
registers, RAM, PPU registers, nametables, palette, OAM, board registers, the shown frame log) - the gate of the
reference's rl/tests/gpu_check.py:28-53, with the same action sampler (rl/actions.py random_legal, seeded CPU
generator) and sticky + idle + dropout on."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from rlenv import RlEnv
from actions import random_legal

OUTS = ['obs', 'emph', 'reward', 'done', 'masks', 'timeline', 'pads', 'events', 'parts']


def _pair(counts, oracle_path, gpu_lib_path, seed=11, **kw):
    kw = dict(seed=seed, sticky=True, idle_max=30, dropout=True, **kw)
    g = RlEnv(counts, device='cuda', lib_path=gpu_lib_path, **kw)
    c = RlEnv(counts, device='cpu', lib_path=oracle_path, **kw)
    return g, c


def _compare(g, c, t):
    for k in OUTS:
        a, b = getattr(g, k).cpu(), getattr(c, k)
        if not torch.equal(a, b):
            bad = (a != b).reshape(len(a), -1).any(1).nonzero().flatten().tolist()
            raise AssertionError(f'step {t}: output {k} differs in envs {bad[:8]} ({len(bad)} envs)')
    d = c.done.bool()
    if t and d.any():
        assert torch.equal(g.info.cpu()[d], c.info[d]), f'step {t}: info differs'


def _compare_dumps(g, c, envs, t):
    for e in envs:
        a, b = g.dump(e), c.dump(e)
        if not np.array_equal(a, b):
            where = np.flatnonzero(a != b)
            raise AssertionError(f'step {t} env {e}: machine dump differs at bytes {where[:12].tolist()} '
                                 f'gpu {a[where[:12]].tolist()} cpu {b[where[:12]].tolist()}')
        assert np.array_equal(g.scalars(e), c.scalars(e)), f'step {t} env {e}: scalars differ'


def run_parity(counts, oracle_path, gpu_lib_path, steps, seed=11, dump_every=25):
    g, c = _pair(counts, oracle_path, gpu_lib_path, seed)
    g.start()
    c.start()
    torch.cuda.synchronize()
    gen = torch.Generator().manual_seed(seed)
    envs = sorted({0, g.n - 1, g.n // 2})
    dones = 0
    for t in range(steps + 1):
        torch.cuda.synchronize()
        _compare(g, c, t)
        if t % dump_every == 0:
            _compare_dumps(g, c, envs, t)
        if t == steps:
            break
        dones += int(c.done.sum()) if t else 0
        act = random_legal(c.masks, gen)
        c.actions.copy_(act)
        g.actions.copy_(act.cuda())
        c.step()
        g.step()
    return dones


@pytest.mark.gpu
def test_parity_nrom_short(oracle_path, gpu_lib_path):
    run_parity({'synth00': 8}, oracle_path, gpu_lib_path, steps=40, dump_every=1)


@pytest.mark.gpu
def test_parity_nrom_config1(oracle_path, gpu_lib_path):
    """one synthetic NROM cart, 64 envs, sticky/dropout/idle on; restarts included."""
    dones = run_parity({'synth00': 64}, oracle_path, gpu_lib_path, steps=400, dump_every=50)
    assert dones > 0, 'the run should cover episode restarts'
