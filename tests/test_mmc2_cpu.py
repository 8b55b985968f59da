"""The MMC2 cart (synth13) on the CPU oracle exercises every latch path the board has (patch:615-665, 1385-1402,
1791-1815): latch changes the CPU puts on the PPU bus mid-frame are logged as register-6/7 events, CHR register
writes mid-frame as register-0..3 events, and the vblank resolve leaves latches the frame's own fetches picked."""
from __future__ import annotations

import numpy as np
import torch

from rlenv import RlEnv
from actions import random_legal

EV_MMC2 = 10


def _events(d: np.ndarray):
    h = d[4544:4544 + 64].view(np.uint32)
    n = int(h[0] & 0x7FFFFFFF)
    return h, d[4544 + 64:4544 + 64 + 8 * n].view(np.uint32).reshape(-1, 2)


def test_mmc2_cart_moves_latches_on_the_oracle(oracle_path):
    e = RlEnv({'synth13': 4}, device='cpu', lib_path=oracle_path, seed=3, sticky=True, idle_max=8, dropout=True)
    e.start()
    g = torch.Generator().manual_seed(1)
    seen = set()
    latches = set()
    for _ in range(160):
        e.actions.copy_(random_legal(e.masks, g))
        e.step()
        for k in range(4):
            d = e.dump(k)
            _, ev = _events(d)
            for w0, w1 in ev:
                if (w0 >> 24) == EV_MMC2:
                    aux, value = int((w1 >> 8) & 0xFF), int(w1 & 0xFF)
                    seen.add(aux)
                    if aux >= 6:
                        assert value in (0, 1)
            regs = d[4448:4464]
            latches.add((int(regs[6]), int(regs[7])))
            # the CHR pages of each half follow the register its latch picks
            pages = d[4480:4512].view(np.uint32) >> 10
            for half in range(2):
                bank = int(regs[2 * half + regs[6 + half]])
                assert [int(p) for p in pages[4 * half:4 * half + 4]] == [(4 * bank + i) & 127 for i in range(4)]
    assert 7 in seen      # the mid-frame $1FD8 address moved latch 1
    assert all(v <= 1 for pair in latches for v in pair)
