"""Build librlenv_b200.so in-tree for sm_100a (nvcc, one object per board compiled in parallel).

    python ghostrun-lab_b200/build.py [--force]

The library lands next to this file (ghostrun-lab_b200/librlenv_b200.so) so it travels with the repository
snapshot; it is rebuilt when a source under csrc/ or a header under include/ is newer than it.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
from pathlib import Path
import subprocess
import sys

HERE = Path(__file__).resolve().parent
CSRC = HERE / 'csrc'
INCLUDE = HERE.parent / 'include'   # the C-ABI header the definitions are compiled against
OUT = HERE / 'librlenv_b200.so'
BUILD = HERE / '_build'
UNITS = ['rlenv_b200.cu', 'board_nrom.cu', 'board_uxrom.cu', 'board_mmc1.cu', 'board_mmc3.cu', 'board_cnrom.cu', 'board_mmc2.cu', 'stem.cu']
NVCC = os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc' if Path('/usr/local/cuda/bin/nvcc').exists() else 'nvcc')
FLAGS = ['-gencode', 'arch=compute_100a,code=sm_100a', '-O3', '-std=c++17', '-lineinfo', '-fmad=false',
         '--expt-relaxed-constexpr', '-Xcompiler', '-fPIC', '-Xcompiler', '-ffp-contract=off']


def stale() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [*CSRC.iterdir(), *INCLUDE.glob('*.h')])


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return OUT
    BUILD.mkdir(exist_ok=True)
    extra = ['-Xptxas', '-v'] if verbose else []

    def compile_unit(u):
        obj = BUILD / (Path(u).stem + '.o')
        cmd = [NVCC, *FLAGS, *extra, '-c', str(CSRC / u), '-o', str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f'nvcc failed on {u}:\n{r.stderr[-4000:]}')
        return obj, r.stderr

    with cf.ThreadPoolExecutor(len(UNITS)) as ex:
        results = list(ex.map(compile_unit, UNITS))
    if verbose:
        for _, err in results:
            sys.stderr.write(err)
    objs = [str(o) for o, _ in results]
    tmp = OUT.with_suffix('.so.tmp')
    subprocess.run([NVCC, '-gencode', 'arch=compute_100a,code=sm_100a', '-shared', '-cudart', 'static', *objs,
                    '-o', str(tmp)], check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == '__main__':
    print(build(force='--force' in sys.argv, verbose='-v' in sys.argv))
