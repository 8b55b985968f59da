"""The policy network used by the end-to-end rollout measurement (ghostrun-lab_b200/policy.py, the reference's
rl/model.py:96-217 architecture): its size, and that the ordered heads only choose legal move parts."""
from __future__ import annotations

import pytest
import torch

from actions import PARTS, unpack
from policy import Policy


def _masks(n, gen):
    m = (torch.rand(n, 19, generator=gen) < 0.6).to(torch.uint8)
    for a, b in PARTS:   # at least one legal choice per part
        m[torch.arange(n), a + torch.randint(0, b - a, (n,), generator=gen)] = 1
    return m


def test_parameter_count_matches_reference():
    # rl/model.py with its defaults (core 512, CNN 32/64/64, stem 16, 101 value bins, no moods): 6.33M parameters
    assert sum(p.numel() for p in Policy(torch.rand(512, 3)).parameters()) == 6_332_263


def test_act_chooses_legal_parts():
    gen = torch.Generator().manual_seed(3)
    torch.manual_seed(3)
    pol = Policy(torch.rand(512, 3))
    masks = _masks(256, gen)
    parts, logp = pol.act(torch.randn(256, 512, generator=gen), masks, gen)
    for (a, b), c in zip(PARTS, parts):
        assert bool((masks[torch.arange(256), a + c] == 1).all())
    assert bool((logp <= 0).all())


@pytest.mark.gpu
def test_decide_on_packed_pictures(gpu_lib_path):
    import stem
    stem._lib(gpu_lib_path)
    dev = torch.device('cuda')
    gen = torch.Generator(device=dev).manual_seed(5)
    torch.manual_seed(5)
    pol = Policy(torch.rand(512, 3)).to(dev).to(memory_format=torch.channels_last)
    B = 96
    packed = torch.randint(0, 256, (B, 4, 224, 180), generator=gen, device=dev, dtype=torch.int32).to(torch.uint8)
    emph = torch.randint(0, 8, (B, 4, 224), generator=gen, device=dev, dtype=torch.int32).to(torch.uint8)
    tl = torch.randint(0, 2, (B, 8, 45), generator=gen, device=dev, dtype=torch.int32).to(torch.uint8)
    prev = [torch.zeros(B, dtype=torch.long, device=dev) for _ in range(5)]
    masks = _masks(B, torch.Generator().manual_seed(5)).to(dev)
    h = torch.zeros(B, 512, device=dev)
    mv, parts, logp, val, h2 = pol.decide(packed, emph, tl, prev, masks, h, torch.ones(B, dtype=torch.bool, device=dev),
                                          gen, chunk=40)
    assert mv.dtype == torch.int16 and mv.shape == (B,) and val.shape == (B, 101) and h2.shape == (B, 512)
    for (a, b), c in zip(PARTS, unpack(mv)):
        assert bool((masks[torch.arange(B, device=dev), a + c] == 1).all())
    assert bool(torch.isfinite(h2).all()) and bool(torch.isfinite(logp).all())
