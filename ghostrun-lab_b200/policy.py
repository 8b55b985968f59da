"""The reference's 12-game policy network (rl/model.py:96-217, ~6.33M parameters) as the consumer of the env's outputs
for the end-to-end rollout measurement (bench.py --workload config5): random initialisation, bf16 autocast.

Only the input stem is this library's own kernel (stem.fused_stem: palette lookup + 2x2 stride-2 convolution on the
renderer's 6-bit packed pictures, tcgen05); the rest is torch (cuDNN convolutions, cuBLAS linears) and stands in for
the caller's network. Architecture (rl/model.py:1-16 docstring): stem 12 -> 16 channels; three conv sequences
32 / 64 / 64 (conv 3x3, max-pool 3/2, two residual blocks, rl/model.py:32-61); ReLU + global mean -> 64; dropout
timeline 8x45 -> 64; previous move (5 one-hot parts, 19); Linear -> 512; two SimBa blocks (LayerNorm, 512-2048-512,
rl/model.py:64-72); LayerNorm; GRU cell 512 (fp32); ordered action heads d-pad 9 -> A 3 -> B 3 -> Start 2 ->
Select 2, each conditioned on the earlier parts' choices and masked by the legal parts (rl/model.py:176-194); value
head of 101 bins.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from actions import PARTS, pack
from stem import fused_stem

SIZES = [b - a for a, b in PARTS]   # 9, 3, 3, 2, 2
NEG = -1e9


class Residual(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.a = nn.Conv2d(c, c, 3, padding=1)
        self.b = nn.Conv2d(c, c, 3, padding=1)

    def forward(self, x):
        return x + self.b(F.relu(self.a(F.relu(x))))


class ConvStage(nn.Module):
    def __init__(self, cin, cout):
        super().__init__()
        self.conv = nn.Conv2d(cin, cout, 3, padding=1)
        self.res = nn.Sequential(Residual(cout), Residual(cout))

    def forward(self, x):
        return self.res(F.max_pool2d(self.conv(x), 3, 2, 1))


class Simba(nn.Module):
    def __init__(self, d, mult=4):
        super().__init__()
        self.ln = nn.LayerNorm(d)
        self.up = nn.Linear(d, d * mult)
        self.down = nn.Linear(d * mult, d)

    def forward(self, x):
        return x + self.down(F.relu(self.up(self.ln(x))))


class Policy(nn.Module):
    def __init__(self, palette_rgb: torch.Tensor, core=512, cnn=(32, 64, 64), stem=16, bins=101):
        super().__init__()
        self.register_buffer('palette', palette_rgb.float().clone(), persistent=False)   # [512, 3] in [0, 1]
        self.stem = nn.Conv2d(12, stem, 2, stride=2)
        stages, c = [], stem
        for o in cnn:
            stages.append(ConvStage(c, o))
            c = o
        self.cnn = nn.Sequential(*stages)
        self.timeline = nn.Linear(8 * 45, 64)
        self.inp = nn.Linear(c + 64 + sum(SIZES), core)
        self.blocks = nn.Sequential(Simba(core), Simba(core))
        self.ln = nn.LayerNorm(core)
        self.gru = nn.GRUCell(core, core)
        self.heads = nn.ModuleList(nn.Linear(core, n) for n in SIZES)
        self.cond = nn.ModuleList(nn.ModuleList(nn.Embedding(SIZES[j], SIZES[k]) for j in range(k)) for k in range(5))
        self.value = nn.Linear(core, bins)

    def encode(self, packed, emph, timeline, prev_parts):
        """packed [B,4,224,180] 6-bit pictures, emph [B,4,224], timeline [B,8,45] u8, prev_parts [5][B] long -> [B, core].
        Call under bf16 autocast."""
        x = fused_stem(packed, emph, self.palette, self.stem.weight, self.stem.bias, packed=True, check=False)
        x = F.relu(self.cnn(x)).mean((2, 3))
        t = F.relu(self.timeline(timeline.flatten(1).to(x.dtype)))
        p = torch.cat([F.one_hot(prev_parts[k], n) for k, n in enumerate(SIZES)], 1).to(x.dtype)
        return self.ln(self.blocks(self.inp(torch.cat([x, t.to(x.dtype), p], 1))))

    def act(self, h, masks, generator=None):
        """One move per row, part by part (each part sees the earlier choices), sampled among the legal choices.
        Returns (parts: 5 long tensors, summed log-probability [B])."""
        chosen, logp = [], torch.zeros(h.shape[0], device=h.device)
        for k, (a, b) in enumerate(PARTS):
            lg = self.heads[k](h)
            for j in range(k):
                lg = lg + self.cond[k][j](chosen[j])
            lg = lg.float().masked_fill(masks[:, a:b] == 0, NEG)
            lp = lg.log_softmax(-1)
            c = torch.multinomial(lp.exp(), 1, generator=generator).squeeze(1)
            logp = logp + lp.gather(1, c[:, None]).squeeze(1)
            chosen.append(c)
        return chosen, logp

    @torch.no_grad()
    def decide(self, packed, emph, timeline, prev_parts, masks, h, starts, generator=None, chunk=2048):
        """One rollout decision for a batch of envs: encode (in batches of `chunk`, as the reference's rollout
        encoder, rl/train.py:460-464), GRU (memory cleared at episode starts), move, value.
        Returns (move ids int16 [B], parts, logp [B], value logits [B, bins], new h [B, core] fp32)."""
        with torch.autocast('cuda', dtype=torch.bfloat16):
            z = torch.cat([self.encode(packed[a:a + chunk], emph[a:a + chunk], timeline[a:a + chunk],
                                       [p[a:a + chunk] for p in prev_parts])
                           for a in range(0, packed.shape[0], chunk)])
        h = self.gru(z.float(), h * (~starts).unsqueeze(1).float())
        parts, logp = self.act(h, masks, generator)
        return pack(parts), parts, logp, self.value(h), h
