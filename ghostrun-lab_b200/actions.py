"""The 324-move encoding of the environment's actions and a seeded random legal-move sampler.

A move id packs five independent choices, least significant first: the d-pad (9 choices: neutral and the 8
directions), A (3: off, held, turbo), B (3), Start (2) and Select (2), so id = d + 9 a + 27 b + 81 start + 162 select.
The environment's 19 mask bytes list which choice of each part is allowed at the next decision, in the same part
order. This is the encoding and sampler API of the reference's rl/actions.py (pack, unpack, random_legal), which a
drop-in must share: seeded action streams only match the reference's if the same torch.multinomial calls are made
in the same order.
"""
import torch

# (first mask byte, one past the last) of each part, and the weight of the part's choice in a move id
PARTS = [(0, 9), (9, 12), (12, 15), (15, 17), (17, 19)]
MULT = [1, 9, 27, 81, 162]
_RADIX = [9, 3, 3, 2, 2]


def pack(parts):
    """Five per-part choice tensors (long, d-pad first) -> int16 move ids."""
    ids = parts[0] * MULT[0]
    for choice, weight in zip(parts[1:], MULT[1:]):
        ids = ids + choice * weight
    return ids.to(torch.int16)


def unpack(ids):
    """int16 / long move ids -> the five per-part choice tensors (long), d-pad first."""
    ids = ids.long()
    return [(ids // weight) % radix for weight, radix in zip(MULT, _RADIX)]


def random_legal(masks, gen=None):
    """One move per row of `masks` ([N, 19] mask bytes): each part drawn uniformly among the choices its mask allows,
    part by part in d-pad, A, B, Start, Select order, from `gen`."""
    parts = []
    for lo, hi in PARTS:
        parts.append(torch.multinomial(masks[:, lo:hi].float(), 1, generator=gen).squeeze(1))
    return pack(parts)
