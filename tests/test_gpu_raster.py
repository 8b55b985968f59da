"""GPU env == CPU oracle on the mid-frame PPU programs real games run while the picture is drawn, which the
registered synthetic carts never do (synth.make_cart(..., ppu=...), on NROM, on MMC1 with CHR-RAM, and on MMC3,
whose two-phase renderer draws lines with mid-line writes itself and whose scanline IRQ fires inside the programs):

  split   polls $2002 bit 6 until sprite 0 hits, then writes $2006 / $2005 inside that line (a status-bar split):
          the CPU-visible sprite-0 flag and a write inside a line's drawn part;
  raster  6 times a frame: rendering off, a palette entry rewritten, the VRAM address restored, rendering on: more
          palette versions than the two-phase renderer keeps, lines drawn with rendering off, rendering switched on
          inside lines and hblanks;
  vread   $2007 reads with rendering on (the read moves the VRAM address as the PPU's own increments do).

These frames go to the sequential renderer (k_render_seq, the reference's frame-log replay, patch:1408 and
patch:1600-1631), to the walk's own handling of hblank writes, or on MMC3 to the walk's exact split lines; the
emulator's sprite-0 flag follows patch:1740-1789. Each run: 300 decisions of 64 envs with sticky moves, idle starts
and dropout, every output every decision, machine dumps every 25; the run must have drawn frames through the
sequential renderer or (MMC3) lines through the walk's exact path."""
from __future__ import annotations

import pytest

import synth
from rlenv import CART_SEED
from test_gpu_parity import run_parity

BOARD_GAME = {'nrom': ('synth00', 0), 'mmc1': ('synth02', 2), 'mmc3': ('synth03', 3)}   # slug, cart seed offset


@pytest.mark.gpu
@pytest.mark.parametrize('board', ['nrom', 'mmc1', 'mmc3'])
@pytest.mark.parametrize('variant', synth.PPU_VARIANTS)
def test_parity_mid_frame_ppu(board, variant, oracle_path, gpu_lib_path):
    game, k = BOARD_GAME[board]
    rom = synth.make_cart(CART_SEED + k, board, ppu=variant).rom
    envs = []
    run_parity({game: 64}, oracle_path, gpu_lib_path, steps=300, dump_every=25, roms={game: rom}, envs_out=envs)
    stats = envs[0].render_stats()
    assert stats['seq_frames'] + (stats['split_lines'] if board == 'mmc3' else 0) > 0, \
        f'no frame or line took the sequential path: {stats}'
