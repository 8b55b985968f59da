"""Edge cases of the env step on the GPU: ragged game slices (1 env, counts that are no multiple of a warp, six
boards in one env) against the CPU oracle; cartridges the reference's loader refuses (rl/csrc/rlenv_build.hpp:36-84
with describe_mapper, patch:3995-4030) refused the same way by both builds; and BASELINE config 4's per-GPU size
(65,536 envs) through a size-independent property: an env's trajectory depends only on its global index, the run
seed and its actions (rl/csrc/controller.cuh:132-134), so the first envs of the big run equal a small run."""
from __future__ import annotations

import ctypes

import pytest
import torch

from rlenv import RlEnv, synth_cart
from actions import random_legal
from test_gpu_parity import run_parity


@pytest.mark.gpu
def test_parity_ragged_slices(oracle_path, gpu_lib_path):
    counts = {'synth00': 1, 'synth01': 5, 'synth02': 33, 'synth03': 7, 'synth12': 3, 'synth13': 2}
    run_parity(counts, oracle_path, gpu_lib_path, steps=80, dump_every=20)


def bad_roms():
    """(name, iNES bytes, words the refusal names) - each refused by the reference's loader."""
    good = bytearray(synth_cart('synth00').rom)
    truncated = bytes(good[:16 + 20000])
    mapper7 = bytearray(good)
    mapper7[6] = (mapper7[6] & 0x0F) | 0x70          # AxROM: not a supported board
    mmc2_chr_ram = bytearray(synth_cart('synth13').rom)
    mmc2_chr_ram[5] = 0                               # MMC2 without CHR ROM (no CHR-RAM variant)
    mmc2_chr_ram = mmc2_chr_ram[:16 + mmc2_chr_ram[4] * 16384]
    not_ines = b'NES' + bytes(40000)
    return [('truncated', truncated, 'truncated'), ('mapper 7', bytes(mapper7), 'unsupported mapper 7'),
            ('MMC2 with CHR-RAM', bytes(mmc2_chr_ram), 'MMC2'), ('not iNES', not_ines, 'iNES')]


@pytest.mark.parametrize('name,rom,words', bad_roms(), ids=[b[0] for b in bad_roms()])
def test_oracle_refuses_bad_cartridges(name, rom, words, oracle_path):
    game = 'synth13' if 'MMC2' in name else 'synth00'
    with pytest.raises(RuntimeError, match=words):
        RlEnv({game: 2}, device='cpu', lib_path=oracle_path, roms={game: rom})


@pytest.mark.gpu
@pytest.mark.parametrize('name,rom,words', bad_roms(), ids=[b[0] for b in bad_roms()])
def test_gpu_refuses_bad_cartridges(name, rom, words, gpu_lib_path):
    game = 'synth13' if 'MMC2' in name else 'synth00'
    with pytest.raises(RuntimeError, match=words):
        RlEnv({game: 2}, device='cuda', lib_path=gpu_lib_path, roms={game: rom})


@pytest.mark.gpu
def test_parity_cnrom_with_a_larger_prg(oracle_path, gpu_lib_path):
    """CNROM maps PRG pages 0-3, so a 64 KB image runs from its first 32 KB (the loader accepts 16-512 KB,
    patch:4007-4030): the synthetic CNROM cart with 32 KB more PRG behind it."""
    rom = bytearray(synth_cart('synth12').rom)
    prg = rom[4] * 16384
    rom[4] = 4
    big = bytes(rom[:16 + prg]) + bytes((i * 37 + 11) & 0xFF for i in range(prg)) + bytes(rom[16 + prg:])
    g = RlEnv({'synth12': 12}, device='cuda', lib_path=gpu_lib_path, roms={'synth12': big}, seed=4)
    c = RlEnv({'synth12': 12}, device='cpu', lib_path=oracle_path, roms={'synth12': big}, seed=4)
    g.start(); c.start()
    gen = torch.Generator().manual_seed(4)
    for t in range(60):
        torch.cuda.synchronize()
        for k in ('obs', 'emph', 'reward', 'done', 'masks', 'pads', 'events'):
            assert torch.equal(getattr(g, k).cpu(), getattr(c, k)), f'step {t}: {k} differs'
        act = random_legal(c.masks, gen)
        c.actions.copy_(act); g.actions.copy_(act.cuda())
        c.step(); g.step()


@pytest.mark.gpu
def test_config4_size_first_envs_equal_a_small_run(gpu_lib_path):
    N, S = 65536, 64
    kw = dict(seed=21, sticky=True, idle_max=30, dropout=True, lib_path=gpu_lib_path)
    big = RlEnv({'synth00': N}, device='cuda', **kw)
    small = RlEnv({'synth00': S}, device='cuda', **kw)
    packed = torch.zeros(N, 4, 224, 180, dtype=torch.uint8, device='cuda')
    big.bind_obs_pack6(packed)
    un = torch.zeros(S, 4, 224, 240, dtype=torch.uint8, device='cuda')
    big.start()
    small.start()
    gen = torch.Generator().manual_seed(21)
    stream = lambda: ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)  # noqa: E731
    for t in range(13):
        assert big.lib.rl_unpack6(ctypes.c_void_p(packed.data_ptr()), ctypes.c_void_p(un.data_ptr()), un.numel(),
                                  stream()) == 0
        torch.cuda.synchronize()
        assert torch.equal(un, small.obs), f'step {t}: pictures differ'
        for k in ('emph', 'reward', 'done', 'masks', 'timeline', 'pads', 'events', 'parts'):
            assert torch.equal(getattr(big, k)[:S], getattr(small, k)), f'step {t}: {k} differs'
        if t == 12:
            break
        act = random_legal(big.masks.cpu(), gen).cuda()
        big.actions.copy_(act)
        small.actions.copy_(act[:S])
        big.step()
        small.step()
