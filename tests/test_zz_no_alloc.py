"""rlenv_dump_envs_noalloc (the dump that allocates no device memory) == rlenv_dump_env, through the C-ABI.

Two calls in a row on the same file-scope scratch: the first fills all 8 records, the second dumps fewer, different
envs, so a record left over from the first call, or one not cleared, would show. Sizes beyond the fixed maximum
are rejected with a message. Collected last so that it also runs after every other test in one process."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from rlenv import RlEnv
from actions import random_legal

MAX_ENVS = 8          # RLENV_DUMP_NOALLOC_MAX_ENVS
DUMP = 23040          # RLENV_DUMP_BYTES


class _DefaultPool:
    """The device's default memory pool through the driver API (libcuda): its used-memory high-water mark, reset
    before a call and read after it, shows whether the call allocated from it (rlenv_dump_env's staging does)."""
    USED_MEM_HIGH = 8   # CU_MEMPOOL_ATTR_USED_MEM_HIGH

    def __init__(self, device):
        self.cu = ctypes.CDLL('libcuda.so.1')
        dev = ctypes.c_int()
        assert self.cu.cuDeviceGet(ctypes.byref(dev), device) == 0
        self.pool = ctypes.c_void_p()
        assert self.cu.cuDeviceGetDefaultMemPool(ctypes.byref(self.pool), dev) == 0

    def reset_high(self):
        zero = ctypes.c_uint64(0)
        assert self.cu.cuMemPoolSetAttribute(self.pool, self.USED_MEM_HIGH, ctypes.byref(zero)) == 0

    def high(self):
        v = ctypes.c_uint64()
        assert self.cu.cuMemPoolGetAttribute(self.pool, self.USED_MEM_HIGH, ctypes.byref(v)) == 0
        return v.value


def _noalloc(env, envs):
    fn = env.lib.rlenv_dump_envs_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    idx = (ctypes.c_int * max(len(envs), 1))(*envs)
    out = np.full(max(len(envs), 1) * DUMP, 0xA5, dtype=np.uint8)
    rc = fn(env.h, ctypes.cast(idx, ctypes.c_void_p), len(envs), out.ctypes.data_as(ctypes.c_void_p), env._stream())
    return rc, out.reshape(-1, DUMP)


@pytest.mark.gpu
def test_dump_noalloc_matches_dump_env(gpu_lib_path):
    env = RlEnv({'synth00': 40}, device='cuda', lib_path=gpu_lib_path, seed=5, sticky=True, idle_max=30, dropout=True)
    env.start()
    gen = torch.Generator().manual_seed(5)
    for _ in range(6):
        env.actions.copy_(random_legal(env.masks.cpu(), gen).cuda())
        env.step()
    torch.cuda.synchronize()

    for envs in ([0, 1, 2, 3, 4, 5, 6, 39], [37, 5, 20]):
        rc, got = _noalloc(env, envs)
        assert rc == 0, env.lib.rlenv_error().decode()
        for i, e in enumerate(envs):
            want = env.dump(e)
            assert np.array_equal(got[i], want), f'env {e}: bytes {np.flatnonzero(got[i] != want)[:12].tolist()}'

    # allocates nothing: the default pool's high-water mark moves for the allocating dump and stays 0 for this one
    torch.cuda.synchronize()
    pool = _DefaultPool(torch.cuda.current_device())
    pool.reset_high()
    env.dump(3)
    assert pool.high() > 0, 'the check should see rlenv_dump_env\'s staging allocation'
    pool.reset_high()
    rc, _ = _noalloc(env, [3, 4])
    assert rc == 0 and pool.high() == 0, 'rlenv_dump_envs_noalloc allocated from the device pool'

    rc, _ = _noalloc(env, list(range(MAX_ENVS + 1)))
    assert rc != 0 and b'1..8 envs' in env.lib.rlenv_error()
    rc, _ = _noalloc(env, [])
    assert rc != 0
    rc, _ = _noalloc(env, [40])
    assert rc != 0 and b'bad env index' in env.lib.rlenv_error()
