"""GPU env == CPU oracle with level starts and places on (BASELINE config 3's reset rule, rl/rlenv.py:172-310,
rl/csrc/rlenv_core.cuh:208-387): slots fill with each decision's best arrival, new episodes start from them (uniform,
then a seeded Dirichlet(1) CDF), places are saved and copied, and the whole state resumes exactly through save/load.
Every output, the start slot of finished episodes, level / progress outputs, slot deaths and machine dumps match."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from rlenv import RlEnv
from actions import random_legal
from test_gpu_parity import _compare, _compare_dumps

COUNTS = {'synth00': 16, 'synth01': 8, 'synth02': 8, 'synth03': 16}


def _same_f32(a, b):
    return torch.equal(a.contiguous().view(torch.int32), b.contiguous().view(torch.int32))


def _compare_levels(g, c, t):
    d = c.done.bool()
    if t and d.any():
        assert torch.equal(g.start_level.cpu()[d], c.start_level[d]), f'step {t}: start_level differs'
    assert torch.equal(g.level_now.cpu(), c.level_now), f'step {t}: level_now differs'
    assert _same_f32(g.progress_now.cpu(), c.progress_now), f'step {t}: progress_now differs'


@pytest.mark.gpu
def test_level_starts_parity(oracle_path, gpu_lib_path):
    kw = dict(seed=5, sticky=True, idle_max=30, dropout=True, level_cap=8, level_slots=6)
    g = RlEnv(COUNTS, device='cuda', lib_path=gpu_lib_path, **kw)
    c = RlEnv(COUNTS, device='cpu', lib_path=oracle_path, **kw)
    g.start()
    c.start()
    gen = torch.Generator().manual_seed(5)
    right = torch.full((c.n,), 3, dtype=torch.int16)
    level_starts = 0
    for t in range(481):
        torch.cuda.synchronize()
        _compare(g, c, t)
        _compare_levels(g, c, t)
        if t and c.done.any():
            level_starts += int((c.start_level[c.done.bool()] > 0).sum())
        if t % 20 == 0:
            for gi in range(len(c.games)):
                assert np.array_equal(g.level_deaths(gi), c.level_deaths(gi)), f'step {t}: slot deaths of game {gi}'
        if t % 80 == 0:
            _compare_dumps(g, c, [0, 17, 30, c.n - 1], t)
        if t == 60:
            for e in (g, c):
                e.set_level_prob(1.0)
        if t == 150:
            ei, si = torch.tensor([1, 2, 5], dtype=torch.int32), torch.tensor([6, 7, 3], dtype=torch.int32)
            g.place_save(0, ei.cuda(), si.cuda())
            c.place_save(0, ei, si)
            torch.cuda.synchronize()
            g.place_copy(2, [1], [6])
            c.place_copy(2, [1], [6])
        if t == 250:
            saved = sorted(c.saved_levels()['synth00'])
            w = np.zeros(8)
            w[saved + [6, 7]] = np.random.default_rng(5).dirichlet(np.ones(len(saved) + 2))
            for e in (g, c):
                e.set_level_plan(0, 1.0, w)
        if t == 480:
            break
        act = random_legal(c.masks, gen)
        act = torch.where(torch.arange(c.n) % 2 == 0, right, act)
        c.actions.copy_(act)
        g.actions.copy_(act.cuda())
        c.step()
        g.step()
    assert level_starts > 0, 'the run should finish episodes that began at a saved level'

    # exact resume: the GPU state (level-start state included) into a fresh env, both continue in lock step with the oracle
    sd = g.state_dict()
    g2 = RlEnv(COUNTS, device='cuda', lib_path=gpu_lib_path, **kw)
    g2.start()
    g2.load_state_dict(sd)
    for e in (g2,):
        e.set_level_plan(0, 1.0, w)
        for gi in range(1, 4):
            e.set_level_plan(gi, 1.0)
    for t in range(40):
        act = random_legal(c.masks, gen)
        c.actions.copy_(act)
        g2.actions.copy_(act.cuda())
        c.step()
        g2.step()
        torch.cuda.synchronize()
        _compare(g2, c, 481 + t)
        _compare_levels(g2, c, 481 + t)


@pytest.mark.gpu
def test_parity_config3(oracle_path, gpu_lib_path):
    """BASELINE config 3 in small: the 12 synthetic game ids (4 boards round-robin: NROM, UxROM, MMC1 with CHR-RAM,
    MMC3 with its line-32 IRQ split), each with its own seeded reward weights, 8 envs each; 16 level-entrance slots
    per game filled by play, every new episode starting from a saved slot (P(level start) = 1), uniform first and
    then with seeded Dirichlet(1) weights over the saved slots (rl/rlenv.py:251-254 CDF)."""
    counts = {f'synth{k:02d}': 8 for k in range(12)}
    kw = dict(seed=31, sticky=True, idle_max=30, dropout=True, level_cap=16)
    g = RlEnv(counts, device='cuda', lib_path=gpu_lib_path, **kw)
    c = RlEnv(counts, device='cpu', lib_path=oracle_path, **kw)
    g.start()
    c.start()
    gen = torch.Generator().manual_seed(31)
    right = torch.full((c.n,), 3, dtype=torch.int16)
    rng = np.random.default_rng(31)
    level_starts = 0
    for t in range(501):
        torch.cuda.synchronize()
        _compare(g, c, t)
        _compare_levels(g, c, t)
        if t and c.done.any():
            level_starts += int((c.start_level[c.done.bool()] > 0).sum())
        if t % 100 == 0:
            _compare_dumps(g, c, [0, 23, 42, 61, 90, c.n - 1], t)
            for gi in range(len(c.games)):
                assert np.array_equal(g.level_deaths(gi), c.level_deaths(gi)), f'step {t}: slot deaths of game {gi}'
        if t == 20:
            for e in (g, c):
                e.set_level_prob(1.0)
        if t == 250:
            for gi, game in enumerate(c.games):
                saved = sorted(c.saved_levels()[game])
                if not saved:
                    continue
                w = np.zeros(16)
                w[saved] = rng.dirichlet(np.ones(len(saved)))
                for e in (g, c):
                    e.set_level_plan(gi, 1.0, w)
        if t == 500:
            break
        act = random_legal(c.masks, gen)
        act = torch.where((torch.arange(c.n) % 2 == 0) | (t < 150), right, act)   # all hold Right at first
        c.actions.copy_(act)
        g.actions.copy_(act.cuda())
        c.step()
        g.step()
    assert level_starts > 0, 'the run should finish episodes that began at a saved level'
