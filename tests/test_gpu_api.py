"""The rest of the GPU C-ABI surface against the plain step: per-game and per-range stepping
(rl/csrc/rlenv.cu:247-267), the renderer's fused 6-bit output against rl_pack6 and the reference formula
(rl/tests/test_host_obs_pack6.py:16-30), rl_unpack6, exact resume through save/load (rl/csrc/rlenv.cu:270-298), and
the learner-side gathers rl_gather_rows / rl_gather_envs (rl/csrc/rlenv.cu:400-421)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from rlenv import RlEnv
from actions import random_legal

COUNTS = {'synth00': 24, 'synth03': 16}
OUTS = ['obs', 'emph', 'reward', 'done', 'masks', 'timeline', 'pads', 'events', 'parts']


def _env(gpu_lib_path, seed=9):
    e = RlEnv(COUNTS, device='cuda', lib_path=gpu_lib_path, seed=seed, sticky=True, idle_max=30, dropout=True)
    e.start()
    return e


def _same(a, b, t, what=''):
    for k in OUTS:
        assert torch.equal(getattr(a, k), getattr(b, k)), f'step {t}: {k} differs {what}'


def _pack6_formula(obs: np.ndarray) -> np.ndarray:
    p = obs.reshape(-1, 4).astype(np.uint32) & 63
    v = p[:, 0] | (p[:, 1] << 6) | (p[:, 2] << 12) | (p[:, 3] << 18)
    return np.stack([v & 255, (v >> 8) & 255, (v >> 16) & 255], 1).astype(np.uint8).reshape(-1)


@pytest.mark.gpu
def test_step_game_and_range_match_step(gpu_lib_path):
    a, b, c = _env(gpu_lib_path), _env(gpu_lib_path), _env(gpu_lib_path)
    gen = torch.Generator().manual_seed(1)
    sl = a.game_slices()
    for t in range(30):
        act = random_legal(a.masks.cpu(), gen).cuda()
        for e in (a, b, c):
            e.actions.copy_(act)
        a.step()
        for gi in range(len(b.games)):
            b.step_game(gi, b.obs, b.emph)
        for gi, s in enumerate(sl):
            n = s.stop - s.start
            c.step_range(gi, 0, n // 3, c.obs, c.emph)
            c.step_range(gi, n // 3, n - n // 3, c.obs, c.emph)
        torch.cuda.synchronize()
        _same(a, b, t, 'step_game')
        _same(a, c, t, 'step_range')


@pytest.mark.gpu
def test_step_range_on_concurrent_streams_matches_step(gpu_lib_path):
    """Parts of one game stepped at the same time on different streams (the reference's rollout_split units,
    rl/train.py:569-652) equal the plain step, through episode ends (restarts listed per part)."""
    counts = {'synth00': 256, 'synth03': 128}
    mk = lambda: RlEnv(counts, device='cuda', lib_path=gpu_lib_path, seed=9, sticky=True, idle_max=30, dropout=True)  # noqa: E731
    a, c = mk(), mk()
    a.start(); c.start()
    streams = [torch.cuda.Stream() for _ in range(3)]
    parts = []   # (game, start, count): each game in uneven parts, spread over the streams
    for gi, s in enumerate(c.game_slices()):
        n = s.stop - s.start
        cuts = [0, n // 4, n // 2 + 8, n]
        parts += [(gi, cuts[j], cuts[j + 1] - cuts[j]) for j in range(3)]
    gen = torch.Generator().manual_seed(1)
    ends = 0
    for t in range(150):
        act = random_legal(a.masks.cpu(), gen).cuda()
        a.actions.copy_(act); c.actions.copy_(act)
        a.step()
        main = torch.cuda.current_stream()
        for j, (gi, st, n) in enumerate(parts):
            q = streams[j % len(streams)]
            q.wait_stream(main)
            with torch.cuda.stream(q):
                c.step_range(gi, st, n, c.obs, c.emph)
        for q in streams:
            main.wait_stream(q)
        torch.cuda.synchronize()
        _same(a, c, t, 'step_range on concurrent streams')
        ends += int(a.done.sum())
    assert ends > 0   # restarts were exercised (12 episode ends with these seeds)


@pytest.mark.gpu
def test_fused_pack6_matches_rl_pack6_and_formula(gpu_lib_path):
    a, b = _env(gpu_lib_path), _env(gpu_lib_path)
    packed = torch.zeros(b.n, 4, 224, 180, dtype=torch.uint8, device='cuda')
    b.bind_obs_pack6(packed)
    ref = torch.empty_like(packed)
    back = torch.empty_like(a.obs)
    gen = torch.Generator().manual_seed(2)
    stream = lambda: ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)  # noqa: E731
    for t in range(12):
        act = random_legal(a.masks.cpu(), gen).cuda()
        a.actions.copy_(act)
        b.actions.copy_(act)
        a.step()
        b.step()
        assert a.lib.rl_pack6(ctypes.c_void_p(a.obs.data_ptr()), ctypes.c_void_p(ref.data_ptr()), a.obs.numel(), stream()) == 0
        assert a.lib.rl_unpack6(ctypes.c_void_p(ref.data_ptr()), ctypes.c_void_p(back.data_ptr()), a.obs.numel(), stream()) == 0
        torch.cuda.synchronize()
        assert torch.equal(packed, ref), f'step {t}: fused pack6 != rl_pack6(obs)'
        assert torch.equal(back, a.obs & 63), f'step {t}: unpack6(pack6(obs)) != obs'
        assert torch.equal(a.emph, b.emph)
        if t == 11:
            assert np.array_equal(ref.cpu().numpy().reshape(-1), _pack6_formula(a.obs.cpu().numpy()))
    # ragged sizes (tail groups) through the codec
    x = torch.randint(0, 64, (1_000_003,), dtype=torch.uint8, device='cuda')
    n = x.numel() // 4 * 4
    y = torch.zeros(n // 4 * 3, dtype=torch.uint8, device='cuda')
    z = torch.zeros(n, dtype=torch.uint8, device='cuda')
    assert a.lib.rl_pack6(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()), n, stream()) == 0
    assert a.lib.rl_unpack6(ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(z.data_ptr()), n, stream()) == 0
    torch.cuda.synchronize()
    assert torch.equal(z, x[:n])
    assert np.array_equal(y.cpu().numpy(), _pack6_formula(x[:n].cpu().numpy()))


@pytest.mark.gpu
def test_save_load_exact_resume(gpu_lib_path):
    a = _env(gpu_lib_path)
    gen = torch.Generator().manual_seed(3)
    for _ in range(25):
        a.actions.copy_(random_legal(a.masks.cpu(), gen).cuda())
        a.step()
    sd = a.state_dict()
    acts = [None] * 30
    rec = []
    for t in range(30):
        acts[t] = random_legal(a.masks.cpu(), gen).cuda()
        a.actions.copy_(acts[t])
        a.step()
        rec.append({k: getattr(a, k).clone() for k in OUTS})
    b = _env(gpu_lib_path, seed=77)       # another seed: everything must come from the saved state
    b.load_state_dict(sd)
    for t in range(30):
        b.actions.copy_(acts[t])
        b.step()
        torch.cuda.synchronize()
        for k in OUTS:
            assert torch.equal(getattr(b, k), rec[t][k]), f'resumed step {t}: {k} differs'


@pytest.mark.gpu
def test_gathers(gpu_lib_path):
    a = _env(gpu_lib_path)
    lib = a.lib
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    T, N, row = 5, 40, 161_280
    src = torch.randint(0, 256, (T, N, row), dtype=torch.uint8, device='cuda')
    rows = torch.tensor([0, 7, 199, 3, 3, 120], dtype=torch.int64, device='cuda')
    dst = torch.zeros(len(rows), row, dtype=torch.uint8, device='cuda')
    assert lib.rl_gather_rows(ctypes.c_void_p(dst.data_ptr()), ctypes.c_void_p(src.data_ptr()),
                              ctypes.c_void_p(rows.data_ptr()), len(rows), row, s) == 0
    envs = np.array([39, 0, 17], dtype=np.int64)         # host array (copy-engine gather)
    dst2 = torch.zeros(T, len(envs), row, dtype=torch.uint8, device='cuda')
    assert lib.rl_gather_envs(ctypes.c_void_p(dst2.data_ptr()), ctypes.c_void_p(src.data_ptr()),
                              envs.ctypes.data_as(ctypes.c_void_p), len(envs), T, N, row, s) == 0
    torch.cuda.synchronize()
    assert torch.equal(dst, src.reshape(T * N, row)[rows])
    assert torch.equal(dst2, src[:, torch.from_numpy(envs).cuda()])


@pytest.mark.gpu
def test_episode_counters_in_finishing_kernel(gpu_lib_path):
    """rlenv_bind_episode_counters: the finishing kernel's per-decision sums equal the torch reductions over the
    outputs (counts exactly; returns to float32 rounding of the torch sum)."""
    from shard import EpisodeCounters
    a, b = _env(gpu_lib_path), _env(gpu_lib_path)
    ca, cb = EpisodeCounters(torch.device('cuda')), EpisodeCounters(torch.device('cuda'))
    assert cb.attach(b)
    gen = torch.Generator().manual_seed(3)
    for t in range(400):
        act = random_legal(a.masks.cpu(), gen).cuda()
        a.actions.copy_(act); b.actions.copy_(act)
        a.step(); b.step()
        ca.account(a); cb.account(b)
    torch.cuda.synchronize()
    va, vb = ca.rollout_end().as_dict(), cb.rollout_end().as_dict()
    assert va['finished'] > 0 and va['level_events'] >= 0
    for k in ('finished', 'deaths', 'level_events'):
        assert va[k] == vb[k], (k, va[k], vb[k])
    assert abs(va['return_sum'] - vb['return_sum']) <= 1e-4 * max(1.0, abs(vb['return_sum']))


def _legal_moves_numpy(masks: np.ndarray, words: np.ndarray) -> np.ndarray:
    """The sampler of rl_legal_moves restated: per part, splitmix64 of (word << 32 | part), the high 32 bits scaled
    to the number of allowed choices, the k-th allowed choice."""
    M = (1 << 64) - 1
    lo, cnt, mul = (0, 9, 12, 15, 17), (9, 3, 3, 2, 2), (1, 9, 27, 81, 162)
    out = np.zeros(len(words), np.int16)
    for e, w in enumerate(words.astype(np.uint32).tolist()):
        move = 0
        for p in range(5):
            allowed = [c for c in range(cnt[p]) if masks[e, lo[p] + c]]
            z = (((w << 32) | p) + 0x9E3779B97F4A7C15) & M
            z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
            z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
            z ^= z >> 31
            k = ((z >> 32) * len(allowed)) >> 32
            move += (allowed[k] if allowed else 0) * mul[p]
        out[e] = move
    return out


@pytest.mark.gpu
def test_legal_moves_sampler(gpu_lib_path):
    """rl_legal_moves (the benchmark's device sampler): every move legal under the masks, equal to the restated draw
    bit for bit, and each part uniform over its allowed choices (the distribution of rl/actions.py random_legal)."""
    from actions import unpack, PARTS
    e = _env(gpu_lib_path, seed=4)
    gen = torch.Generator(device='cuda').manual_seed(3)
    for t in range(12):   # masks with dropout in effect somewhere
        e.legal_moves(torch.randint(-2 ** 31, 2 ** 31, (e.n,), generator=gen, device='cuda', dtype=torch.int64).to(torch.int32))
        e.step()
    # legality and the restated draw on the env's masks
    words = torch.randint(-2 ** 31, 2 ** 31, (e.n,), generator=gen, device='cuda', dtype=torch.int64).to(torch.int32)
    e.legal_moves(words)
    torch.cuda.synchronize()
    masks = e.masks.cpu().numpy()
    got = e.actions.cpu().numpy()
    assert np.array_equal(got, _legal_moves_numpy(masks, words.cpu().numpy()))
    parts = unpack(e.actions.cpu())
    for (a, b), pt in zip(PARTS, parts):
        assert bool(torch.from_numpy(masks[:, a:b]).gather(1, pt.view(-1, 1)).all()), 'an illegal part'
    # uniformity: 40 envs x 2,000 draws on fixed masks, every allowed choice of every part near 1 / count
    words = torch.randint(-2 ** 31, 2 ** 31, (2000, e.n), generator=gen, device='cuda', dtype=torch.int64).to(torch.int32)
    draws = []
    for r in range(2000):
        e.legal_moves(words[r])
        draws.append(e.actions.clone())
    d = torch.stack(draws).cpu()
    for p, (a, b) in enumerate(PARTS):
        choice = unpack(d)[p]                      # [2000, n]
        for env in range(e.n):
            allowed = np.flatnonzero(masks[env, a:b])
            counts = np.bincount(choice[:, env].numpy(), minlength=b - a)
            assert counts[allowed].sum() == 2000, (p, env, counts)   # nothing outside the allowed choices
            freq = counts[allowed] / 2000
            assert np.all(np.abs(freq - 1 / len(allowed)) < 0.06), (p, env, freq)


@pytest.mark.gpu
def test_learner_gather_from_pinned_host(gpu_lib_path):
    """The learner half of the 6-bit picture format (rl/train.py:262-295 HostObs, rl/csrc/rlenv.cu:369-421): every
    decision's packed pictures and emphasis go into a pinned host region [T, N, row] (rl_host_alloc,
    rl_memcpy_async); a minibatch of envs is gathered back to the device from that host region, one copy-engine 2-D
    copy per env (rl_gather_envs), and unpacked (rl_unpack6). The result equals the pictures and emphasis an
    identical env (same seed and moves) wrote unpacked, decision by decision."""
    N, T = 48, 16
    row, erow = 4 * 224 * 180, 4 * 224
    kw = dict(lib_path=gpu_lib_path, seed=21, sticky=True, idle_max=30, dropout=True)
    a = RlEnv({'synth00': 24, 'synth02': 24}, device='cuda', **kw)   # NROM and MMC1 (CHR-RAM) rows
    b = RlEnv({'synth00': 24, 'synth02': 24}, device='cuda', **kw)
    packed = torch.zeros(N, 4, 224, 180, dtype=torch.uint8, device='cuda')
    a.bind_obs_pack6(packed)
    lib = a.lib
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    host = lib.rl_host_alloc(T * N * row)
    host_e = lib.rl_host_alloc(T * N * erow)
    assert host and host_e
    try:
        a.start(); b.start()
        gen = torch.Generator().manual_seed(21)
        want_obs, want_emph = [], []
        for t in range(T):
            act = random_legal(b.masks.cpu(), gen).cuda()
            a.actions.copy_(act); b.actions.copy_(act)
            a.step(); b.step()
            assert lib.rl_memcpy_async(ctypes.c_void_p(host + t * N * row), ctypes.c_void_p(packed.data_ptr()), N * row, s) == 0
            assert lib.rl_memcpy_async(ctypes.c_void_p(host_e + t * N * erow), ctypes.c_void_p(a.emph.data_ptr()), N * erow, s) == 0
            want_obs.append(b.obs.clone()); want_emph.append(b.emph.clone())
        torch.cuda.synchronize()
        want_obs, want_emph = torch.stack(want_obs), torch.stack(want_emph)   # [T, N, ...]
        for envs in (np.array([3, 47, 0, 30, 24, 23], np.int64), np.arange(N, dtype=np.int64)[::-1].copy()):
            n = len(envs)
            dst = torch.zeros(T, n, row, dtype=torch.uint8, device='cuda')
            dst_e = torch.zeros(T, n, erow, dtype=torch.uint8, device='cuda')
            assert lib.rl_gather_envs(ctypes.c_void_p(dst.data_ptr()), ctypes.c_void_p(host),
                                      envs.ctypes.data_as(ctypes.c_void_p), n, T, N, row, s) == 0
            assert lib.rl_gather_envs(ctypes.c_void_p(dst_e.data_ptr()), ctypes.c_void_p(host_e),
                                      envs.ctypes.data_as(ctypes.c_void_p), n, T, N, erow, s) == 0
            obs = torch.zeros(T, n, 4, 224, 240, dtype=torch.uint8, device='cuda')
            assert lib.rl_unpack6(ctypes.c_void_p(dst.data_ptr()), ctypes.c_void_p(obs.data_ptr()), obs.numel(), s) == 0
            torch.cuda.synchronize()
            idx = torch.from_numpy(envs).cuda()
            assert torch.equal(obs, want_obs[:, idx]), 'gathered pictures differ from the env\'s own'
            assert torch.equal(dst_e.view(T, n, 4, 224), want_emph[:, idx]), 'gathered emphasis differs'
    finally:
        torch.cuda.synchronize()
        lib.rl_host_free(ctypes.c_void_p(host))
        lib.rl_host_free(ctypes.c_void_p(host_e))
