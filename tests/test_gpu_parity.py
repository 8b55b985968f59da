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
            where = ''
            if k == 'obs':   # the first differing env's frames and picture rows
                d = (a[bad[0]] != b[bad[0]])
                where = '; env %d: ' % bad[0] + ', '.join(
                    f'frame {f} rows {d[f].any(1).nonzero().flatten().tolist()[:8]}' for f in range(d.shape[0]) if d[f].any())
            raise AssertionError(f'step {t}: output {k} differs in envs {bad[:8]} ({len(bad)} envs){where}')
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


def run_parity(counts, oracle_path, gpu_lib_path, steps, seed=11, dump_every=25, roms=None, envs_out=None):
    """Steps a GPU env and an oracle env with the same seeded legal moves and compares them (every output every
    decision, machine dumps every `dump_every`); returns the finished episodes. roms: slug -> iNES image in place of
    the registered cart; envs_out: a list that receives (gpu env, oracle env)."""
    g, c = _pair(counts, oracle_path, gpu_lib_path, seed, roms=roms)
    if envs_out is not None:
        envs_out.extend([g, c])
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
    """one synthetic NROM cart, 64 envs, sticky/dropout/idle on, 2,000 decisions (every output
    every decision, machine dumps every 100); restarts included."""
    dones = run_parity({'synth00': 64}, oracle_path, gpu_lib_path, steps=2000, dump_every=100)
    assert dones > 0, 'the run should cover episode restarts'


@pytest.mark.gpu
def test_parity_config2_subset(oracle_path, gpu_lib_path):
    """BASELINE config 2's check: the 8,192-env GPU run (pictures packed by the renderer) against the CPU oracle on a
    256-env subset. An env's trajectory depends only on its global index, the run seed and its actions, so envs
    0..255 of the big run equal a 256-env run. Packed pictures are compared after rl_unpack6."""
    import ctypes
    N, S = 8192, 256
    kw = dict(seed=5, sticky=True, idle_max=30, dropout=True)
    g = RlEnv({'synth00': N}, device='cuda', lib_path=gpu_lib_path, **kw)
    c = RlEnv({'synth00': S}, device='cpu', lib_path=oracle_path, **kw)
    packed = torch.zeros(N, 4, 224, 180, dtype=torch.uint8, device='cuda')
    g.bind_obs_pack6(packed)
    un = torch.zeros(S, 4, 224, 240, dtype=torch.uint8, device='cuda')
    g.start()
    c.start()
    gen = torch.Generator().manual_seed(5)
    gen_rest = torch.Generator(device='cuda').manual_seed(6)   # the other envs: the bench's device sampler
    stream = lambda: ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)  # noqa: E731
    dones = 0
    for t in range(151):
        assert g.lib.rl_unpack6(ctypes.c_void_p(packed.data_ptr()), ctypes.c_void_p(un.data_ptr()), un.numel(), stream()) == 0
        torch.cuda.synchronize()
        assert torch.equal(un.cpu(), c.obs), f'step {t}: pictures differ'
        for k in ('emph', 'reward', 'done', 'masks', 'timeline', 'pads', 'events', 'parts'):
            assert torch.equal(getattr(g, k)[:S].cpu(), getattr(c, k)), f'step {t}: {k} differs'
        d = c.done.bool()
        if t and d.any():
            dones += int(d.sum())
            assert torch.equal(g.info[:S].cpu()[d], c.info[d]), f'step {t}: info differs'
        if t == 150:
            break
        act = random_legal(c.masks, gen)
        words = torch.randint(-2 ** 31, 2 ** 31, (N,), generator=gen_rest, device='cuda', dtype=torch.int64)
        g.legal_moves(words.to(torch.int32))
        c.actions.copy_(act)
        g.actions[:S].copy_(act.cuda())
        c.step()
        g.step()
    for e in (0, 101, 255):
        assert np.array_equal(g.dump(e), c.dump(e)), f'env {e}: machine dump differs'
    assert dones > 0, 'the run should cover episode restarts'
