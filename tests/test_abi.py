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
