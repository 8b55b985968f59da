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
    counts = {'synth00': 8, 'synth01': 8, 'synth02': 8, 'synth03': 8, 'synth12': 8, 'synth13': 8}
    run_parity(counts, oracle_path, gpu_lib_path, steps=200, dump_every=40)
