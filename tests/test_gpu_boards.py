"""GPU env == CPU oracle on the paged boards (BASELINE config 3's mappers): UxROM (synth01), MMC1 with CHR-RAM
(synth02), MMC3 with its scanline IRQ (synth03), CNROM with its CHR bank latch (synth12), MMC2 with its $FD/$FE CHR
latches (synth13: tile and sprite fetches, $2006/$2007 addresses and mid-frame register writes move them), each alone
and all six boards in one env (one game slice per board, each on its own stream pair, as rl/csrc/rlenv.cu:51-182)."""
from __future__ import annotations

import pytest

from test_gpu_parity import run_parity


@pytest.mark.gpu
@pytest.mark.parametrize('game', ['synth01', 'synth02', 'synth03', 'synth12', 'synth13'])
def test_parity_paged_board(game, oracle_path, gpu_lib_path):
    run_parity({game: 16}, oracle_path, gpu_lib_path, steps=120, dump_every=10)


@pytest.mark.gpu
def test_parity_mixed_boards(oracle_path, gpu_lib_path):
    """All six boards in one env; the NROM slice runs the sprite-0 status-bar split variant of its cart (mid-line
    $2006 / $2005 writes after a $2002 poll), so its frames take the sequential renderer beside the other boards'."""
    import synth
    from rlenv import CART_SEED
    counts = {'synth00': 8, 'synth01': 8, 'synth02': 8, 'synth03': 8, 'synth12': 8, 'synth13': 8}
    roms = {'synth00': synth.make_cart(CART_SEED, 'nrom', ppu='split').rom}
    envs = []
    run_parity(counts, oracle_path, gpu_lib_path, steps=200, dump_every=40, roms=roms, envs_out=envs)
    assert envs[0].render_stats()['seq_frames'] > 0


@pytest.mark.gpu
def test_save_load_exact_resume_latched_boards(gpu_lib_path):
    """rlenv_save / rlenv_load (rl/csrc/rlenv.cu:270-298) carry CNROM's bank latch and MMC2's registers and $FD/$FE
    latches: a fresh env (another seed) loaded with the state continues with the same outputs."""
    import torch
    from rlenv import RlEnv
    from actions import random_legal
    counts = {'synth12': 12, 'synth13': 12}
    kw = dict(sticky=True, idle_max=30, dropout=True, lib_path=gpu_lib_path)
    a = RlEnv(counts, device='cuda', seed=8, **kw)
    a.start()
    gen = torch.Generator().manual_seed(8)
    for _ in range(70):   # past the MMC2 cart's first mid-frame register write (frame 64)
        a.actions.copy_(random_legal(a.masks.cpu(), gen).cuda())
        a.step()
    sd = a.state_dict()
    acts, rec = [], []
    for t in range(40):
        acts.append(random_legal(a.masks.cpu(), gen).cuda())
        a.actions.copy_(acts[t])
        a.step()
        rec.append({k: getattr(a, k).clone() for k in ('obs', 'emph', 'reward', 'done', 'masks', 'pads', 'events')})
    b = RlEnv(counts, device='cuda', seed=99, **kw)
    b.start()
    b.load_state_dict(sd)
    for t in range(40):
        b.actions.copy_(acts[t])
        b.step()
        torch.cuda.synchronize()
        for k, v in rec[t].items():
            assert torch.equal(getattr(b, k), v), f'resumed step {t}: {k} differs'


@pytest.mark.gpu
def test_parity_dmc_sample_channel(oracle_path, gpu_lib_path):
    """The DMC sample channel on the GPU against the oracle (patch:405-567; the oracle's DMC is pinned by the
    reference's own known-answer tests): the NROM cart's DMC variant starts a sample every frame (looped on odd frames)
    and keeps $4015 in RAM; every output each decision, and the machine dumps (CPU cycle counter, the DMC's state,
    RAM) every 10 decisions, match."""
    import torch
    import synth
    from rlenv import RlEnv
    from actions import random_legal
    from test_gpu_parity import _compare, _compare_dumps
    rom = synth.make_cart(1000, 'nrom', dmc=True).rom
    kw = dict(seed=6, sticky=True, idle_max=30, dropout=True, roms={'synth00': rom})
    g = RlEnv({'synth00': 24}, device='cuda', lib_path=gpu_lib_path, **kw)
    c = RlEnv({'synth00': 24}, device='cpu', lib_path=oracle_path, **kw)
    g.start(); c.start()
    gen = torch.Generator().manual_seed(6)
    for t in range(61):
        torch.cuda.synchronize()
        _compare(g, c, t)
        if t % 10 == 0:
            _compare_dumps(g, c, [0, 11, 23], t)
            assert c.dump(0)[64 + synth.ZP_DMC] & 0x10, 'the sample should be playing when $4015 is read'
        if t == 60:
            break
        act = random_legal(c.masks, gen)
        c.actions.copy_(act); g.actions.copy_(act.cuda())
        c.step(); g.step()
