"""The fused colour lookup + stem convolution (rl_stem_fwd, tcgen05) against an fp64 torch reference of the same
op (rl/model.py:141-149 stem_conv on the bf16 picture, rl/fused.py:163-169): palette values and weights rounded to
bf16 as the reference does, products exact, sums in fp32 on the tensor cores, so the bf16 outputs agree to bf16
rounding (tolerance below). The 6-bit packed input gives the same outputs bit for bit. The palette is a seeded
stand-in (any [512, 3] table is a valid input)."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from stem import fused_stem

torch.backends.cudnn.allow_tf32 = False
torch.backends.cuda.matmul.allow_tf32 = False


def _inputs(B, seed):
    g = torch.Generator().manual_seed(seed)
    obs = torch.randint(0, 64, (B, 4, 224, 240), generator=g, dtype=torch.uint8)
    emph = torch.randint(0, 8, (B, 4, 224), generator=g, dtype=torch.uint8)
    pal = torch.randint(0, 256, (512, 3), generator=g).float() / 255.0
    w = torch.randn(16, 12, 2, 2, generator=g) * 0.2
    b = torch.randn(16, generator=g) * 0.1
    return obs, emph, pal, w, b


def _reference(obs, emph, pal, w, b):
    """fp64: x = bf16(palette)[colour | emph << 6] -> conv2d(bf16(w), stride 2) + bf16(bias)."""
    palb = pal.to(torch.bfloat16).double()
    idx = obs.long() | (emph.long() << 6).unsqueeze(-1)                    # B,4,H,W
    x = palb[idx]                                                        # B,4,H,W,3
    x = x.permute(0, 1, 4, 2, 3).reshape(obs.shape[0], 12, 224, 240)     # frame-major RGB channels
    return F.conv2d(x, w.to(torch.bfloat16).double(), b.to(torch.bfloat16).double(), stride=2)


def _pack6(obs):
    v = obs.reshape(-1, 4).int() & 63
    g = v[:, 0] | (v[:, 1] << 6) | (v[:, 2] << 12) | (v[:, 3] << 18)
    out = torch.stack([g & 255, (g >> 8) & 255, (g >> 16) & 255], 1).to(torch.uint8)
    return out.reshape(obs.shape[0], 4, 224, 180)


@pytest.mark.gpu
@pytest.mark.parametrize('B', [1, 3, 16])
def test_stem_matches_reference(B):
    obs, emph, pal, w, b = _inputs(B, 7 + B)
    out = fused_stem(obs.cuda(), emph.cuda(), pal, w, b)
    assert out.shape == (B, 16, 112, 120) and out.dtype == torch.bfloat16
    ref = _reference(obs, emph, pal, w, b)
    got = out.float().cpu().double()
    err = (got - ref).abs()
    tol = 2.0 ** -7 * ref.abs() + 1e-3
    bad = err > tol
    assert not bad.any(), f'{int(bad.sum())} outputs off, worst {float(err.max()):.4g}'
    packed = fused_stem(_pack6(obs).cuda(), emph.cuda(), pal, w, b, packed=True)
    assert torch.equal(packed, out), 'packed input must give the same outputs'


@pytest.mark.gpu
def test_stem_rejects_cpu():
    obs, emph, pal, w, b = _inputs(1, 1)
    with pytest.raises(RuntimeError):
        fused_stem(obs, emph, pal, w, b)
