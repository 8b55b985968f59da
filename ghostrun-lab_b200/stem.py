"""The policy's input stem on the B200 library: colour lookup + 2x2 stride-2 convolution fused in one tcgen05 kernel
(rl_stem_fwd), with the reference's fused_stem interface (rl/fused.py:163-169):

    out = fused_stem(obs, emph, palette_rgb, weight, bias)      # [B, 16, 112, 120] bf16, channels-last strides

obs: [B, 4, 224, 240] uint8 colour numbers, or the 6-bit packed rollout pictures [B, 4, 224, 180] (packed=True);
emph: [B, 4, 224] uint8; palette_rgb: [512, 3] float (index colour | emphasis << 6); weight: [16, 12, 2, 2];
bias: [16]. Computed in bf16 (inputs, weights and output; fp32 sums). Forward only."""
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
        _LIB = lib
    return _LIB


def palette4(palette_rgb: torch.Tensor) -> torch.Tensor:
    """[512, 3] float -> [512, 4] bf16 (R, G, B, 0): the bf16-rounded picture values the stem multiplies."""
    return torch.nn.functional.pad(palette_rgb.to(torch.bfloat16), (0, 1)).contiguous()


def fused_stem(obs, emph, palette_rgb, weight, bias, packed=False, lib_path=None, check=True):
    if obs.device.type != 'cuda':
        raise RuntimeError('the fused stem runs on the GPU only')
    B = obs.shape[0]
    assert obs.dtype == torch.uint8 and obs.is_contiguous() and emph.is_contiguous()
    assert obs.shape == ((B, 4, 224, 180) if packed else (B, 4, 224, 240)) and emph.shape == (B, 4, 224)
    dev = obs.device
    pal = palette4(palette_rgb.to(dev))
    w = weight.reshape(weight.shape[0], 48).to(device=dev, dtype=torch.bfloat16).contiguous()
    b = bias.to(device=dev, dtype=torch.bfloat16).contiguous()
    assert w.shape == (16, 48) and b.shape == (16,)
    out = torch.empty(B, 112, 120, 16, dtype=torch.bfloat16, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    lib = _lib(lib_path)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    rc = lib.rl_stem_fwd(p(obs), p(emph), p(pal), p(w), p(b), p(out), B, int(bool(packed)), p(err),
                         ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    if rc != 0:
        raise RuntimeError(f'rl_stem_fwd: {lib.rl_stem_error().decode()}')
    if check and int(err.item()) != 0:
        raise RuntimeError('rl_stem_fwd: a tensor-core tile did not complete')
    return out.permute(0, 3, 1, 2)
