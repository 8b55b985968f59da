"""Level starts and places on the CPU oracle (host logic; rl/rlenv.py:172-310, rl/csrc/rlenv_core.cuh:208-387):
with level-start chance 0 the run is the power-on run (the level coin is drawn only when the chance is set), slots
fill with the best arrival, episodes start from saved slots with the CDF or uniform pick, and the state format keeps
the level-start state last (a state saved without level starts loads into an env with them; a smaller archive
grows)."""
from __future__ import annotations

import numpy as np
import torch

from rlenv import RlEnv
from actions import random_legal

OUTS = ['obs', 'emph', 'reward', 'done', 'masks', 'timeline', 'pads', 'events', 'parts', 'info']


def _drive(env, steps, seed, plan=None):
    gen = torch.Generator().manual_seed(seed)
    right = torch.full((env.n,), 3, dtype=torch.int16)   # dpad Right: the synthetic carts' levels advance
    hist = []
    for t in range(steps):
        if plan is not None:
            plan(env, t)
        a = random_legal(env.masks, gen)
        env.actions.copy_(torch.where(torch.arange(env.n) % 2 == 0, right, a))
        env.step()
        hist.append({k: getattr(env, k).clone() for k in OUTS})
    return hist


def _env(oracle_path, **kw):
    kw = dict(seed=3, sticky=True, idle_max=30, dropout=True, **kw)
    e = RlEnv({'synth00': 8, 'synth03': 8}, device='cpu', lib_path=oracle_path, **kw)
    e.start()
    return e


def test_zero_chance_is_power_on_run(oracle_path):
    a = _drive(_env(oracle_path), 120, 1)
    b = _drive(_env(oracle_path, level_cap=8), 120, 1)
    for t, (x, y) in enumerate(zip(a, b)):
        for k in OUTS:
            assert torch.equal(x[k], y[k]), f'step {t} output {k}'


def test_level_starts_fill_and_are_used(oracle_path):
    env = _env(oracle_path, level_cap=8)
    starts = []

    def plan(e, t):
        if t == 100:
            e.set_level_prob(1.0)
        if t == 300:
            w = np.zeros(8)
            saved = sorted(e.saved_levels()['synth00'])
            w[saved] = np.random.default_rng(0).dirichlet(np.ones(len(saved)))
            e.set_level_plan(0, 1.0, w)
        d = e.done.bool()
        if t and d.any():
            starts.extend(e.start_level[d].tolist())

    _drive(env, 500, 2, plan)
    saved = env.saved_levels()
    assert len(saved['synth00']) >= 3 and len(saved['synth03']) >= 3, saved
    assert 0 not in saved['synth00']           # level 0 is the power-on start: never an arrival
    assert any(s > 0 for s in starts), 'episodes should start from saved levels'
    lv = env.level_deaths(0)
    assert ((lv >= -1)).all() and (lv[1:] >= 0).sum() == len(saved['synth00'])


def test_state_prefix_and_grow(oracle_path):
    plain = _env(oracle_path)
    _drive(plain, 20, 4)
    sd = plain.state_dict()
    lv = _env(oracle_path, level_cap=8)
    lv.load_state_dict(sd)                     # saved without level starts: the tail comes from the fresh env
    assert (lv.level_deaths(0) == -1).all()
    _drive(lv, 200, 5)
    sd8 = lv.state_dict()
    big = _env(oracle_path, level_cap=12)
    big.load_state_dict(sd8)                   # 8 slots -> 12: the new slots are empty
    d8, d12 = lv.level_deaths(0), big.level_deaths(0)
    assert np.array_equal(d12[:8], d8) and (d12[8:] == -1).all()
    a, b = _drive(lv, 30, 6), _drive(big, 30, 6)
    for t, (x, y) in enumerate(zip(a, b)):
        for k in OUTS:
            d = x['done'].bool() if k == 'info' else slice(None)   # info is defined where done
            assert torch.equal(x[k][d], y[k][d]), f'step {t} output {k} after the archive grew'


def test_places(oracle_path):
    env = _env(oracle_path, level_cap=8, level_slots=5)
    _drive(env, 60, 7)
    lvl1, frame1 = int(env.dump(1)[64 + 0x12]), int(env.scalars(1)[1])
    env.place_save(0, torch.tensor([1, 2, 3], dtype=torch.int32), torch.tensor([5, 2, 7], dtype=torch.int32))
    d = env.level_deaths(0)
    assert d[5] == 0 and d[7] == 0 and d[6] == -1      # slot 2 < level_slots: skipped
    env.place_copy(0, [5], [6])
    assert env.level_deaths(0)[6] == 0
    env.set_level_plan(0, 1.0, np.eye(8)[6])           # every new synth00 episode starts from place 6
    env.start()                                        # restart every env now
    for e in range(8):
        assert int(env.dump(e)[64 + 0x12]) == lvl1, f'env {e} did not start from the place'
        assert int(env.scalars(e)[1]) >= frame1 + 4    # ep_frame continues from the saved frame
    starts = []

    def plan(e, t):
        dd = e.done.bool()
        if t and dd[:8].any():
            starts.extend(e.start_level[:8][dd[:8]].tolist())
    _drive(env, 200, 8, plan)
    assert set(starts) <= {6}
