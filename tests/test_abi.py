"""The drop-in boundary: the GPU library loads, exports every entry point include/rlenv_api.h declares, and fails
loudly (NULL + message) instead of falling back to a CPU path when there is no CUDA device."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / 'include' / 'rlenv_api.h'


def declared():
    text = re.sub(r'//[^\n]*', '', HEADER.read_text())
    return sorted(set(re.findall(r'\b((?:rlenv|rl10|rl)_[a-z0-9_]+)\s*\(', text)))


@pytest.fixture(scope='module')
def lib():
    import sys
    sys.path.insert(0, str(ROOT / 'ghostrun-lab_b200'))
    import build
    return ctypes.CDLL(str(build.build()))


def test_header_lists_the_reference_surface():
    names = set(declared())
    ref = {'rlenv_create', 'rlenv_num_envs', 'rlenv_set_episode_level_end', 'rlenv_bind', 'rlenv_bind_parts',
           'rlenv_bind_obs', 'rlenv_start', 'rlenv_step', 'rlenv_state_bytes', 'rlenv_save', 'rlenv_load',
           'rlenv_error', 'rlenv_destroy', 'rlenv_num_games', 'rlenv_step_game', 'rlenv_step_range',
           'rlenv_set_no_render', 'rl_host_alloc', 'rl_host_free', 'rl_pack6', 'rl_unpack6', 'rl_memcpy_async',
           'rl_gather_rows', 'rl_gather_envs'}
    assert ref <= names, sorted(ref - names)


# The reference loader's ctypes declarations (rl/rlenv.py:78-120; P pointer, I int, U64 uint64, SZ size_t, D double),
# plus the two extras it calls without declaring (rl/csrc/rlenv.cu:247, 364-366). A library bound through that loader
# must take exactly these arguments: ctypes converts by these kinds and passes nothing else.
REFERENCE_ARGTYPES = {
    'rlenv_create': ['I', 'P', 'P', 'P', 'P', 'P', 'P', 'U64', 'I', 'I', 'I', 'I'],
    'rlenv_num_envs': ['P'], 'rlenv_bind': ['P'] * 11, 'rlenv_bind_parts': ['P', 'P'],
    'rlenv_bind_obs': ['P', 'P', 'P'], 'rlenv_start': ['P', 'P'], 'rlenv_step': ['P', 'P'],
    'rlenv_state_bytes': ['P'], 'rlenv_save': ['P', 'P', 'P'], 'rlenv_load': ['P', 'P', 'P'], 'rlenv_error': [],
    'rlenv_destroy': ['P'], 'rlenv_set_episode_level_end': ['P', 'I'], 'rlenv_enable_level_starts': ['P', 'I'],
    'rlenv_set_level_plan': ['P', 'I', 'D', 'P'], 'rlenv_bind_start': ['P', 'P'], 'rlenv_bind_level': ['P', 'P'],
    'rlenv_bind_progress': ['P', 'P'], 'rlenv_level_deaths': ['P', 'I', 'P', 'P'],
    'rlenv_enable_places': ['P', 'I', 'I'], 'rlenv_place_save': ['P', 'I', 'P', 'P', 'I', 'P'],
    'rlenv_place_copy': ['P', 'I', 'P', 'P', 'I', 'P'], 'rlenv_level_layout': ['P', 'I', 'P'],
    'rl_host_alloc': ['SZ'], 'rl_host_free': ['P'], 'rl_memcpy_async': ['P', 'P', 'SZ', 'P'],
    'rl_gather_rows': ['P', 'P', 'P', 'I', 'SZ', 'P'], 'rl_gather_envs': ['P', 'P', 'P', 'I', 'I', 'I', 'SZ', 'P'],
    'rl_pack6': ['P', 'P', 'SZ', 'P'], 'rl_unpack6': ['P', 'P', 'SZ', 'P'],
    'rlenv_step_game': ['P', 'I', 'P', 'P', 'P'], 'rlenv_step_range': ['P', 'I', 'I', 'I', 'P', 'P', 'P'],
    'rlenv_num_games': ['P'], 'rlenv_set_no_render': ['P', 'I'],
}


def header_signatures():
    """name -> parameter kinds, from the declarations in include/rlenv_api.h."""
    text = re.sub(r'//[^\n]*', '', HEADER.read_text())
    out = {}
    for name, params in re.findall(r'\b((?:rlenv|rl10|rl)_[a-z0-9_]+)\s*\(([^()]*)\)\s*;', text):
        kinds = []
        for p in (x.strip() for x in params.split(',')):
            if p in ('', 'void'):
                continue
            kinds.append('P' if '*' in p else 'SZ' if 'size_t' in p else 'U64' if 'uint64_t' in p
                         else 'D' if 'double' in p else 'I' if re.search(r'\b(int|unsigned)\b', p) else '?' + p)
        out[name] = kinds
    return out


def test_header_signatures_match_the_reference_loader():
    sigs = header_signatures()
    assert set(sigs) == set(declared())
    wrong = {n: (sigs.get(n), want) for n, want in REFERENCE_ARGTYPES.items() if sigs.get(n) != want}
    assert not wrong, wrong


def test_every_declared_symbol_is_exported(lib):
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_create_without_gpu_fails_loudly(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip('a GPU is present')
    import numpy as np
    sys_path = str(ROOT / 'ghostrun-lab_b200')
    import sys
    sys.path.insert(0, sys_path)
    import synth
    cart = synth.make_cart(1000, 'nrom')
    lib.rlenv_create.restype = ctypes.c_void_p
    lib.rlenv_error.restype = ctypes.c_char_p
    roms = (ctypes.c_char_p * 1)(cart.rom)
    boots = (ctypes.c_char_p * 1)(cart.boot_pads)
    h = lib.rlenv_create(1, (ctypes.c_int * 1)(12), roms, (ctypes.c_size_t * 1)(len(cart.rom)), boots,
                         (ctypes.c_size_t * 1)(len(cart.boot_pads)), (ctypes.c_int * 1)(4), ctypes.c_uint64(1), 1, 0,
                         1, 0)
    assert not h
    assert b'GPU' in lib.rlenv_error()


def test_rlenv_refuses_cpu_without_a_library():
    import sys
    sys.path.insert(0, str(ROOT / 'ghostrun-lab_b200'))
    from rlenv import RlEnv
    with pytest.raises(RuntimeError, match='GPU only'):
        RlEnv({'synth00': 2}, device='cpu')
