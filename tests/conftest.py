"""Test set-up: the `gpu` marker (tests that need a B200), library paths, and the oracle / reference loaders."""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / 'ghostrun-lab_b200'
ORACLE = ROOT / 'oracle'
sys.path.insert(0, str(PKG))
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA device (B200)')


def oracle_lib() -> Path:
    """The CPU oracle (test infrastructure), built from oracle/ on first use."""
    lib = ORACLE / 'liboracle_rlenv.so'
    srcs = [ORACLE / n for n in ('oracle_api.cpp', 'env.hpp', 'nes.hpp')]
    if not lib.exists() or any(s.stat().st_mtime > lib.stat().st_mtime for s in srcs):
        subprocess.run(['make', '-C', str(ORACLE), 'all'], check=True, capture_output=True)
    return lib


def reference_tree():
    """The reference source tree (read only, test infrastructure): the environment variable REF, else a `reference`
    directory beside the repository; None when neither holds the reference's rl/csrc/host_api.cpp."""
    import os
    ref = Path(os.environ.get('REF') or ROOT.parent / 'reference')
    return ref if (ref / 'rl' / 'csrc' / 'host_api.cpp').exists() else None


def reference_host_lib():
    """The reference's own controller / reward10 host library (oracle/_ref, compiled from the reference tree when it is
    present), or None."""
    lib = ORACLE / '_ref' / 'librl_host.so'
    ref = reference_tree()
    if not lib.exists() and ref is not None:
        subprocess.run(['make', '-C', str(ORACLE), 'ref', f'REF={ref}'], check=True, capture_output=True)
    return lib if lib.exists() else None


@pytest.fixture(scope='session')
def oracle_path():
    return oracle_lib()


@pytest.fixture(scope='session')
def gpu_lib_path():
    """The in-tree GPU library (built on first use), or the build named by RL_CUDA_LIB (rl/rlenv.py:58-60)."""
    import os
    import torch
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    if os.environ.get('RL_CUDA_LIB'):
        return Path(os.environ['RL_CUDA_LIB'])
    sys.path.insert(0, str(PKG))
    import build
    return build.build()
