"""The mid-frame PPU variants of the synthetic carts (synth.make_cart(..., ppu=...)) produce the PPU traffic they are
named for, read back from the CPU oracle's frame logs (both banks: the shown frame and the one before it), so the GPU
tests that run them (tests/test_gpu_raster.py) exercise the paths they claim to:
  split   $2006 and $2005 writes during the picture, after a $2002 sprite-0 poll;
  raster  more than 4 palette writes per frame, rendering switched off and on (mask writes) during the picture;
  vread   $2007 reads during the picture."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import synth
from rlenv import RlEnv, CART_SEED
from actions import random_legal

EV_MASK, EV_SCROLL, EV_ADDR, EV_DREAD, EV_PAL = 2, 3, 4, 6, 7
LOG_WORDS = 16 + 2 * 256


def _frame_events(c, env):
    """(kind, fceumm line) of every event in both frame-log banks of oracle env `env`."""
    buf = np.zeros(2 * LOG_WORDS, np.uint32)
    assert c.lib.oracle_log_banks(ctypes.c_void_p(c.h), env, buf.ctypes.data_as(ctypes.c_void_p)) == 0
    out = []
    for w in (buf[:LOG_WORDS], buf[LOG_WORDS:]):
        n = int(w[0] & 0x7FFFFFFF)
        ev = [(int(w[16 + 2 * k]) >> 24, ((int(w[16 + 2 * k]) & 0x1FFFF) + 11 + 16) // 341) for k in range(min(n, 256))]
        out.append(ev)
    return out


@pytest.mark.parametrize('variant', synth.PPU_VARIANTS)
def test_ppu_variant_events(variant, oracle_path):
    rom = synth.make_cart(CART_SEED, 'nrom', ppu=variant).rom
    c = RlEnv({'synth00': 8}, device='cpu', lib_path=oracle_path, seed=3, sticky=True, idle_max=30, dropout=True,
              roms={'synth00': rom})
    c.start()
    gen = torch.Generator().manual_seed(3)
    for _ in range(4):
        c.actions.copy_(random_legal(c.masks, gen))
        c.step()
    for env in range(8):
        for frame in _frame_events(c, env):
            visible = [k for k, line in frame if line < 240]
            if variant == 'split':
                assert visible.count(EV_ADDR) == 2 and visible.count(EV_SCROLL) == 2, frame
            elif variant == 'raster':
                assert visible.count(EV_PAL) == 6 and visible.count(EV_MASK) == 12, frame
            else:
                assert visible.count(EV_DREAD) == 3, frame
