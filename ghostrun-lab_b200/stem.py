"""The policy's input stem on the B200 library: colour lookup + 2x2 stride-2 convolution fused in one tcgen05 kernel
(rl_stem_fwd), with the reference's fused_stem interface (rl/fused.py:163-169):

    out = fused_stem(obs, emph, palette_rgb, weight, bias)      # [B, 16, 112, 120] bf16, channels-last strides

obs: [B, 4, 224, 240] uint8 colour numbers, or the 6-bit packed rollout pictures [B, 4, 224, 180] (packed=True);
emph: [B, 4, 224] uint8; palette_rgb: [512, 3] float (index colour | emphasis << 6); weight: [16, 12, 2, 2];
bias: [16]. Computed in bf16 (inputs, weights and output; fp32 sums). Differentiable in weight and bias, as the
reference's custom op (rl/fused.py:148-160): the backward (rl_stem_bwd, tcgen05) recomputes the inputs from the colour
numbers and returns dW = sum_p g[p] x[p]^T and dbias = sum_p g[p] in fp32, cast to the parameters' dtypes."""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

from rlenv import default_lib

_LIB = None


def _lib(path=None):
    global _LIB
    if _LIB is None or path is not None:
        lib = ctypes.CDLL(str(path or default_lib()))
        P = ctypes.c_void_p
        lib.rl_stem_fwd.argtypes = [P, P, P, P, P, P, ctypes.c_longlong, ctypes.c_int, P, P]
        lib.rl_stem_error.restype = ctypes.c_char_p
        lib.rl_stem_bwd.argtypes = [P, P, P, P, P, P, ctypes.c_longlong, ctypes.c_int, P, ctypes.c_size_t, P, P]
        lib.rl_stem_bwd_work_bytes.restype = ctypes.c_size_t
        _LIB = lib
    return _LIB


def palette4(palette_rgb: torch.Tensor) -> torch.Tensor:
    """[512, 3] float -> [512, 4] bf16 (R, G, B, 0): the bf16-rounded picture values the stem multiplies."""
    return torch.nn.functional.pad(palette_rgb.to(torch.bfloat16), (0, 1)).contiguous()


def _check_inputs(obs, emph, packed):
    if obs.device.type != 'cuda':
        raise RuntimeError('the fused stem runs on the GPU only')
    B = obs.shape[0]
    assert obs.dtype == torch.uint8 and obs.is_contiguous() and emph.is_contiguous()
    assert obs.shape == ((B, 4, 224, 180) if packed else (B, 4, 224, 240)) and emph.shape == (B, 4, 224)
    return B


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def stem_forward(obs, emph, pal4, w48, b16, packed=False, lib_path=None, check=True):
    """[B, 112, 120, 16] bf16 (channels-last storage) from bf16 pal4 [512, 4], w48 [16, 48] and b16 [16]."""
    B = _check_inputs(obs, emph, packed)
    out = torch.empty(B, 112, 120, 16, dtype=torch.bfloat16, device=obs.device)
    err = torch.zeros(1, dtype=torch.int32, device=obs.device)
    lib = _lib(lib_path)
    rc = lib.rl_stem_fwd(_p(obs), _p(emph), _p(pal4), _p(w48), _p(b16), _p(out), B, int(bool(packed)), _p(err),
                         _stream(obs.device))
    if rc != 0:
        raise RuntimeError(f'rl_stem_fwd: {lib.rl_stem_error().decode()}')
    if check and int(err.item()) != 0:
        raise RuntimeError('rl_stem_fwd: a tensor-core tile did not complete')
    return out


def stem_backward(grad, obs, emph, pal4, packed=False, lib_path=None, check=True):
    """grad [B, 112, 120, 16] (the output's gradient, channels-last) -> (dW [16, 48], dbias [16]) fp32."""
    B = _check_inputs(obs, emph, packed)
    dev = obs.device
    g = grad.to(torch.bfloat16).contiguous()
    assert g.shape == (B, 112, 120, 16)
    lib = _lib(lib_path)
    nbytes = int(lib.rl_stem_bwd_work_bytes())
    work = torch.empty(nbytes // 4, dtype=torch.float32, device=dev)
    dw = torch.empty(16, 48, dtype=torch.float32, device=dev)
    db = torch.empty(16, dtype=torch.float32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    rc = lib.rl_stem_bwd(_p(g), _p(obs), _p(emph), _p(pal4), _p(dw), _p(db), B, int(bool(packed)), _p(work), nbytes,
                         _p(err), _stream(dev))
    if rc != 0:
        raise RuntimeError(f'rl_stem_bwd: {lib.rl_stem_error().decode()}')
    if check and int(err.item()) != 0:
        raise RuntimeError('rl_stem_bwd: a tensor-core tile did not complete')
    return dw, db


class _FusedStem(torch.autograd.Function):
    @staticmethod
    def forward(ctx, obs, emph, pal4, w48, b16, packed, lib_path, check):
        ctx.save_for_backward(obs, emph, pal4)
        ctx.opts = (packed, lib_path, check)
        return stem_forward(obs, emph, pal4, w48, b16, packed, lib_path, check)

    @staticmethod
    def backward(ctx, grad):
        obs, emph, pal4 = ctx.saved_tensors
        packed, lib_path, check = ctx.opts
        dw, db = stem_backward(grad, obs, emph, pal4, packed, lib_path, check)
        # autograd casts each gradient to its input's dtype (bf16 here), as the reference's .to(ctx.wdtype)
        return None, None, None, dw, db, None, None, None


def fused_stem(obs, emph, palette_rgb, weight, bias, packed=False, lib_path=None, check=True):
    _check_inputs(obs, emph, packed)
    dev = obs.device
    pal = palette4(palette_rgb.to(dev))
    w = weight.reshape(weight.shape[0], 48).to(device=dev, dtype=torch.bfloat16)
    b = bias.to(device=dev, dtype=torch.bfloat16)
    assert w.shape == (16, 48) and b.shape == (16,)
    out = _FusedStem.apply(obs, emph, pal, w.contiguous(), b.contiguous(), packed, lib_path, check)
    return out.permute(0, 3, 1, 2)
