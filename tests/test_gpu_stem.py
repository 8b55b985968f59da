"""The fused colour lookup + stem convolution (rl_stem_fwd, tcgen05) against an fp64 torch reference of the same
op (rl/model.py:141-149 stem_conv on the bf16 picture, rl/fused.py:163-169): palette values and weights rounded to
bf16 as the reference does, products exact, sums in fp32 on the tensor cores, so the bf16 outputs agree to bf16
rounding (tolerance below). The 6-bit packed input gives the same outputs bit for bit. The backward (rl_stem_bwd,
rl/fused.py:89-160: dW = sum_p g[p] x[p]^T, dbias = sum_p g[p]) against fp64 autograd of the same convolution. The
palette is a seeded stand-in (any [512, 3] table is a valid input)."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from stem import fused_stem, palette4, stem_backward

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


def _x(obs, emph, pal):
    palb = pal.to(torch.bfloat16).double()
    idx = obs.long() | (emph.long() << 6).unsqueeze(-1)
    return palb[idx].permute(0, 1, 4, 2, 3).reshape(obs.shape[0], 12, 224, 240)


def _reference_grads(obs, emph, pal, g):
    """fp64 gradients of conv2d(x, w, b, stride 2) for the output gradient g [B, 112, 120, 16], and the sums of
    |terms| (the scale of the fp32 rounding)."""
    x = _x(obs, emph, pal)
    w = torch.zeros(16, 12, 2, 2, dtype=torch.float64, requires_grad=True)
    b = torch.zeros(16, dtype=torch.float64, requires_grad=True)
    F.conv2d(x, w, b, stride=2).backward(g.double().permute(0, 3, 1, 2))
    wa = torch.zeros(16, 12, 2, 2, dtype=torch.float64, requires_grad=True)
    ba = torch.zeros(16, dtype=torch.float64, requires_grad=True)
    F.conv2d(x.abs(), wa, ba, stride=2).backward(g.double().abs().permute(0, 3, 1, 2))
    return w.grad, b.grad, wa.grad, ba.grad


@pytest.mark.gpu
@pytest.mark.parametrize('B', [1, 5])
def test_stem_backward_matches_reference(B):
    obs, emph, pal, w, b = _inputs(B, 31 + B)
    gen = torch.Generator().manual_seed(B)
    g = torch.randn(B, 112, 120, 16, generator=gen).to(torch.bfloat16)
    dw, db = stem_backward(g.cuda(), obs.cuda(), emph.cuda(), palette4(pal).cuda())
    rw, rb, sw, sb = _reference_grads(obs, emph, pal, g.float())
    ew = (dw.cpu().double().reshape(16, 12, 2, 2) - rw).abs()
    eb = (db.cpu().double() - rb).abs()
    assert bool((ew <= 1e-5 * sw + 1e-6).all()), f'dW worst {float(ew.max()):.4g}'
    assert bool((eb <= 1e-5 * sb + 1e-6).all()), f'dbias worst {float(eb.max()):.4g}'
    dw6, db6 = stem_backward(g.cuda(), _pack6(obs).cuda(), emph.cuda(), palette4(pal).cuda(), packed=True)
    assert torch.equal(dw6, dw) and torch.equal(db6, db), 'packed input must give the same gradients'


@pytest.mark.gpu
def test_stem_autograd():
    """fused_stem trains its weight and bias: their gradients are the backward's, cast to the parameters' dtype."""
    obs, emph, pal, w, b = _inputs(2, 5)
    w = w.cuda().requires_grad_(True)
    b = b.cuda().requires_grad_(True)
    gen = torch.Generator().manual_seed(9)
    g = torch.randn(2, 16, 112, 120, generator=gen)
    out = fused_stem(obs.cuda(), emph.cuda(), pal, w, b)
    (out.float() * g.cuda()).sum().backward()
    rw, rb, sw, sb = _reference_grads(obs, emph, pal, g.to(torch.bfloat16).float().permute(0, 2, 3, 1))
    tol = 2.0 ** -7 * rw.abs() + 1e-5 * sw + 1e-6
    assert bool(((w.grad.cpu().double() - rw).abs() <= tol).all())
    assert bool(((b.grad.cpu().double() - rb).abs() <= 2.0 ** -7 * rb.abs() + 1e-5 * sb + 1e-6).all())
