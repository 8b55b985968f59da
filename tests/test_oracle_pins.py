"""The CPU oracle pinned to the reference: its controller against the reference's own compiled host library
(rl/csrc/host_api.cpp: rlc_pad_table, rlc_legal_table, rlc_schedule, rlc_episode_seed) and its reward10 against the
reference's Python RewardTracker (scripts/reward10/reward.py), both through golden vectors committed under
tests/golden/ (made by tests/golden/make_golden.py), and live against oracle/_ref when the reference tree is here.
Rewards are compared as float64 with no tolerance (the reference's rl/tests/test_reward_replay.py:404-426 rule)."""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest

from conftest import oracle_lib, reference_host_lib

GOLD = Path(__file__).resolve().parent / 'golden'
NM = 324
P = ctypes.c_void_p


def ptr(a):
    return a.ctypes.data_as(P)


@pytest.fixture(scope='module')
def orc():
    lib = ctypes.CDLL(str(oracle_lib()))
    lib.oracle_schedule.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_int, P, P]
    lib.oracle_episode_seed.restype = ctypes.c_uint64
    lib.oracle_episode_seed.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64]
    lib.rl10_register_game.argtypes = [ctypes.c_int, P, ctypes.c_int]
    return lib


@pytest.fixture(scope='module')
def cg():
    return np.load(GOLD / 'controller_golden.npz')


def test_pad_table(orc, cg):
    pad = np.zeros(2 * NM, np.uint8)
    orc.oracle_pad_table(ptr(pad))
    assert np.array_equal(pad, cg['pad_table'])


@pytest.mark.parametrize('so,se', [(0, 0), (1, 0), (1, 1)])
def test_legal_and_restrict_tables(orc, cg, so, se):
    legal = np.zeros(9 * NM, np.uint8)
    rest = np.zeros(9 * NM, np.int32)
    orc.oracle_legal_table(so, se, ptr(legal), ptr(rest))
    assert np.array_equal(legal, cg[f'legal_{so}{se}'])
    assert np.array_equal(rest, cg[f'restrict_{so}{se}'])


def test_dropout_schedules_and_timelines(orc, cg):
    n = cg['sched_dropped'].shape[-1]
    nt = cg['sched_timeline'].shape[1]
    for i, s in enumerate(cg['sched_seeds']):
        for en in (0, 1):
            d = np.zeros(n, np.int8)
            t = np.zeros((n, 8 * 45), np.uint8)
            orc.oracle_schedule(int(s), en, n, ptr(d), ptr(t))
            assert np.array_equal(d, cg['sched_dropped'][i, en]), (s, en)
            if en:
                assert np.array_equal(t[:nt], cg['sched_timeline'][i])


def test_episode_seeds(orc, cg):
    got = [orc.oracle_episode_seed(int(a), int(b), int(c)) for a, b, c in cg['episode_triples']]
    assert np.array_equal(np.array(got, np.uint64), cg['episode_seeds'])


def test_dropout_statistics(orc):
    """The reference's spec checks (rl/tests/test_controller.py): runs 8..22, mean gap ~35, ~30% off, ~3.75% per input."""
    n = 200000
    d = np.zeros(n, np.int8)
    orc.oracle_schedule(777, 1, n, ptr(d), None)
    off = d >= 0
    assert 0.26 < off.mean() < 0.34
    for b in range(8):
        assert 0.030 < (d == b).mean() < 0.045
    edges = np.flatnonzero(np.diff(off.astype(np.int8)) != 0) + 1
    runs = np.split(off, edges)
    on_runs = [len(r) for r in runs[1:-1] if r[0]]
    gaps = [len(r) for r in runs[1:-1] if not r[0]]
    assert min(on_runs) >= 8 and max(on_runs) <= 22
    assert 32 < np.mean(gaps) < 38 and min(gaps) >= 1


def test_live_against_reference_host_library(orc):
    ref = reference_host_lib()
    if ref is None:
        pytest.skip('reference tree not present (golden vectors cover this)')
    lib = ctypes.CDLL(str(ref))
    lib.rlc_schedule.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_int, P, P]
    rng = np.random.default_rng(5)
    for s in rng.integers(0, 2**63, 20, dtype=np.uint64):
        a, b = np.zeros(300, np.int8), np.zeros(300, np.int8)
        ta, tb = np.zeros((300, 360), np.uint8), np.zeros((300, 360), np.uint8)
        lib.rlc_schedule(int(s), 1, 300, ptr(a), ptr(ta))
        orc.oracle_schedule(int(s), 1, 300, ptr(b), ptr(tb))
        assert np.array_equal(a, b) and np.array_equal(ta, tb)


def test_reward_replay_matches_python_tracker(orc):
    g = np.load(GOLD / 'reward_golden.npz')
    orc.oracle_reward_replay.argtypes = [ctypes.c_int, P, ctypes.c_int, P, P, P, P, P, P, P, P]
    seen_end, seen_rollback, seen_level, ends = False, False, False, set()
    for k in range(12):
        slug = f'synth{k:02d}'
        spec = np.ascontiguousarray(g[f'{slug}_spec'])
        assert orc.rl10_register_game(12 + k, ptr(spec), len(spec)) == 0
        for ep in range(4):
            key = f'{slug}_e{ep}'
            rows, frames = g[f'{key}_ram'], np.ascontiguousarray(g[f'{key}_frames'])
            n = len(rows)
            ram = np.zeros((n, 2048), np.uint8)
            ram[:, 0x10:0x18] = rows
            rew = np.zeros(n, np.float64); done = np.zeros(n, np.uint8); ev = np.zeros(n, np.uint32)
            lvl = np.zeros(n, np.int32); dea = np.zeros(n, np.int32); end = np.zeros(n, np.uint8)
            parts = np.zeros((n, 7), np.float64)
            assert orc.oracle_reward_replay(12 + k, ptr(ram), n, ptr(frames), ptr(rew), ptr(done), ptr(ev), ptr(lvl),
                                            ptr(dea), ptr(end), ptr(parts)) == 0
            assert np.array_equal(rew, g[f'{key}_reward']), key          # float64, 0 ULP
            assert np.array_equal(done, g[f'{key}_done']), key
            assert np.array_equal(ev, g[f'{key}_events']), key
            assert np.array_equal(dea, g[f'{key}_deaths']), key
            assert np.array_equal(end, g[f'{key}_end']), key
            assert np.allclose(parts.sum(1), rew, atol=1e-12, rtol=0)    # parts sum to the reward
            seen_end |= bool(done.any())
            seen_rollback |= bool((ev & 64).any())
            seen_level |= bool((ev & 2).any())
            ends |= set(end.tolist())
    assert seen_end and seen_rollback and seen_level, 'the traces should cover ends, rollbacks and level events'
    assert {1, 3, 4} <= ends, f'game over, skip and stall ends should all occur ({sorted(ends)})'
