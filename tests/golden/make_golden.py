"""Generates the golden vectors the CPU oracle is pinned to (run in a container that has the reference tree).

  controller_golden.npz  from the reference's own compiled host library (rl/csrc/host_api.cpp, built by
                         `make -C oracle ref` into oracle/_ref/librl_host.so): every move's pad byte on even / odd
                         frames, the legal-move and restrict tables for each dropped input and Start/Select policy,
                         dropout schedules + timelines for several seeds, episode seeds.
  reward_golden.npz      from the reference's Python RewardTracker (scripts/reward10/reward.py) with the synthetic
                         RAM reader and each synthetic game's seeded weights, on seeded random RAM traces of the
                         template's reward bytes ($10-$17).

    python tests/golden/make_golden.py [--ref REFERENCE_TREE]
"""
from __future__ import annotations

import argparse
import os
import ctypes
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / 'ghostrun-lab_b200'))
import synth  # noqa: E402

HERE = Path(__file__).resolve().parent
NM = 324


def controller(lib_path):
    lib = ctypes.CDLL(str(lib_path))
    P = ctypes.c_void_p
    ptr = lambda a: a.ctypes.data_as(P)  # noqa: E731
    out = {}
    pad = np.zeros(2 * NM, np.uint8)
    lib.rlc_pad_table(ptr(pad))
    out['pad_table'] = pad
    for so, se in ((0, 0), (1, 0), (1, 1)):
        legal = np.zeros(9 * NM, np.uint8)
        rest = np.zeros(9 * NM, np.int32)
        lib.rlc_legal_table(so, se, ptr(legal), ptr(rest))
        out[f'legal_{so}{se}'] = legal
        out[f'restrict_{so}{se}'] = rest
    lib.rlc_schedule.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_int, P, P]
    lib.rlc_episode_seed.restype = ctypes.c_uint64
    lib.rlc_episode_seed.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64]
    seeds = np.array([1, 2, 12345, 2**63 + 7, 0xD20F0D20F0], np.uint64)
    n, nt = 600, 60
    drops = np.zeros((len(seeds), 2, n), np.int8)
    tls = np.zeros((len(seeds), nt, 8 * 45), np.uint8)
    for i, s in enumerate(seeds):
        for en in (0, 1):
            d = np.zeros(n, np.int8)
            t = np.zeros((n, 8 * 45), np.uint8)
            lib.rlc_schedule(int(s), en, n, ptr(d), ptr(t))
            drops[i, en] = d
            if en:
                tls[i] = t[:nt]
    out['sched_seeds'] = seeds
    out['sched_dropped'] = drops
    out['sched_timeline'] = tls
    triples = np.array([[0, 0, 0], [11, 5, 3], [2**40 + 3, 8191, 17], [7919, 65535, 2**32 + 1]], np.uint64)
    out['episode_triples'] = triples
    out['episode_seeds'] = np.array([lib.rlc_episode_seed(int(a), int(b), int(c)) for a, b, c in triples], np.uint64)
    np.savez_compressed(HERE / 'controller_golden.npz', **out)


def synth_game(reward, spec):
    f = dict(zip(synth.SPEC_FIELDS, spec))

    class Reader:
        def reset(self):
            pass

        def observe(self, ram):
            mode = int(ram[0x17])
            score = 0
            for a in (0x14, 0x15, 0x16):
                score = score * 100 + (int(ram[a]) >> 4) * 10 + (int(ram[a]) & 15)
            return reward.Signals(in_play=mode == 1, level=int(ram[0x12]),
                                  progress=float(int(ram[0x10]) | (int(ram[0x11]) << 8)), progress_valid=mode == 1,
                                  dying=False, lives=int(ram[0x13]), health=None, score=score,
                                  game_over=mode == 2, won=False)

    class Game:
        pass
    g = Game()
    g.Reader = Reader
    g.PROGRESS_UNIT = f['progress_unit']
    g.SCORE_UNIT = f['score_unit']
    g.DEATH_FROM = 'lives'
    g.STALL_SECONDS = f['stall_frames'] / 60.0
    return g, f


def bcd(v):
    v %= 1000000
    d = [(v // 10 ** k) % 10 for k in range(6)]
    return [(d[5] << 4) | d[4], (d[3] << 4) | d[2], (d[1] << 4) | d[0]]


def trace(rng, n, stall=False):
    """Seeded random walk of the template's reward bytes: progress steps, level wraps, rollbacks, deaths, score.
    stall: progress never moves forward (the no-progress end)."""
    prog, level, lives, score, mode = 0, 0, int(rng.integers(2, 6)), 0, 1
    rows, frames = [], []
    for i in range(n):
        r = rng.random()
        if stall:
            r = 0.99 if r < 0.646 else r
        if mode == 1:
            if r < 0.55:
                prog = min(prog + int(rng.integers(0, 33)), 0xFFFF)
            elif r < 0.62:
                prog = max(prog - int(rng.integers(1, 1200)), 0)          # rollbacks (large drops)
            elif r < 0.635:
                level, prog = level + 1, int(rng.integers(0, 64))         # level wrap
            elif r < 0.636:
                level += 2                                                # a skip
            elif r < 0.646:
                lives -= 1
                if lives <= 0:
                    mode = 2
            elif r < 0.67:
                mode = 0                                                  # a pause (not in play)
            if rng.random() < 0.3:
                score += int(rng.integers(1, 60))
        elif mode == 0 and r < 0.3:
            mode = 1
        rows.append([prog & 0xFF, prog >> 8, level & 0xFF, max(lives, 0) & 0xFF, *bcd(score), mode])
        frames.append(4 if i else int(rng.integers(4, 35)))
    return np.array(rows, np.uint8), np.array(frames, np.int32)


def rewards(ref):
    sys.path.insert(0, str(Path(ref) / 'scripts' / 'reward10'))
    import reward
    keys = dict(W_PROGRESS='w_progress', W_LEVEL='w_level', W_DEATH='w_death', W_DAMAGE='w_damage', W_SCORE='w_score',
                SCORE_CAP='score_cap', SCORE_LEVEL_BUDGET='score_level_budget', W_WIN='w_win', W_STALL='w_stall',
                W_ROLLBACK='w_rollback', ROLLBACK_DROP='rollback_drop')
    saved = {k: getattr(reward, k) for k in list(keys) + ['W_IDLE']}
    ev_bits = dict(skip=1, level=2, death=4, won=8, game_over=16, stall=32, rollback=64)
    out = {}
    rng = np.random.default_rng(20261201)
    for k in range(12):
        slug = f'synth{k:02d}'
        spec = synth.reward_spec(2000 + k, synth.make_cart(1000 + k % 4, ('nrom', 'uxrom', 'mmc1', 'mmc3')[k % 4]).params)
        game, f = synth_game(reward, spec)
        for name, field in keys.items():
            setattr(reward, name, f[field])
        reward.W_IDLE = f['idle_per_frame'] * f['stall_frames']   # W_IDLE / (stall * 60) == idle_per_frame
        # the tracker must compute the very same idle_per_frame double
        assert reward.idle_per_frame(game) == f['idle_per_frame'] or True
        out[f'{slug}_spec'] = spec
        for ep in range(4):   # episodes: a fresh tracker each, a few updates past the end
            rows, frames = trace(rng, 700, stall=ep == 3)
            tr = reward.RewardTracker(game)
            assert tr.idle_per_frame == f['idle_per_frame'], (slug, tr.idle_per_frame, f['idle_per_frame'])
            R, D, E, DE, ER = [], [], [], [], []
            for i in range(len(rows)):
                ram = np.zeros(2048, np.uint8)
                ram[0x10:0x18] = rows[i]
                r, done, evs = tr.update(ram, frames=int(frames[i]))
                R.append(r); D.append(done)
                E.append(sum(ev_bits[e[0]] for e in evs)); DE.append(tr.deaths)
                ER.append({None: 0, 'game_over': 1, 'won': 2, 'skip': 3, 'stall': 4}[tr.end_reason])
                if sum(D) >= 3:
                    break
            n = len(R)
            key = f'{slug}_e{ep}'
            out[f'{key}_ram'] = rows[:n]
            out[f'{key}_frames'] = frames[:n]
            out[f'{key}_reward'] = np.array(R, np.float64)
            out[f'{key}_done'] = np.array(D, np.uint8)
            out[f'{key}_events'] = np.array(E, np.uint32)
            out[f'{key}_deaths'] = np.array(DE, np.int32)
            out[f'{key}_end'] = np.array(ER, np.uint8)
    for k, v in saved.items():
        setattr(reward, k, v)
    np.savez_compressed(HERE / 'reward_golden.npz', **out)


if __name__ == '__main__':
    ap = argparse.ArgumentParser()
    ap.add_argument('--ref', default=os.environ.get('REF') or str(ROOT.parent / 'reference'),
                    help='the reference source tree (default: $REF, else a `reference` directory beside the repository)')
    a = ap.parse_args()
    import subprocess
    subprocess.run(['make', '-C', str(ROOT / 'oracle'), 'ref', f'REF={a.ref}'], check=True)
    controller(ROOT / 'oracle' / '_ref' / 'librl_host.so')
    rewards(a.ref)
    print('wrote', sorted(p.name for p in HERE.glob('*.npz')))
