"""bench.py's output contract, checked on the CPU: the reference arm (the oracle port on the host cores) prints one
JSON line with the keys, units and values the benchmark driver reads, and the workload names follow the env count.
The GPU arm's line (roofline, clocks, gpu_launches, e2e with copies) is produced only on a GPU box."""
from __future__ import annotations

import importlib.util
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _bench_module():
    spec = importlib.util.spec_from_file_location('bench_under_test', ROOT / 'bench.py')
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, str(ROOT / 'bench.py'), '--impl', 'reference', '--steps', '1', '--warmup', '1'],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith('{')]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    for k in ('impl', 'metric', 'value', 'unit', 'n_gpus', 'steps', 'warmup', 'ms_per_step', 'higher_is_better',
              'scaling', 'vs_baseline', 'dtype', 'data', 'config', 'cpu_baseline', 'e2e'):
        assert k in d, k
    assert d['impl'] == 'reference' and d['n_gpus'] == 1 and d['steps'] == 1 and d['warmup'] == 1
    assert d['metric'] == 'decisions/s (4 NES frames each)' and d['unit'] == 'decisions/s'
    assert d['higher_is_better'] is True and d['scaling'] == 'weak' and d['value'] > 0
    cb = d['cpu_baseline']
    assert cb['kind'] == 'port' and cb['cores'] >= 1 and cb['value'] == d['value'] and cb['sample']
    assert d['e2e'] == {'value': d['value'], 'unit': 'decisions/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}
    assert d['config']['workload'].startswith('config 2')
    # the GPU arm reports the same config (bench.workload_config), so the driver sees one workload in both arms
    import types
    assert d['config'] == json.loads(json.dumps(_bench_module().workload_config(types.SimpleNamespace(envs=8192), 1)))


def test_workload_names_follow_the_env_count():
    b = _bench_module()
    assert b.nrom_workload(None).startswith('config 2: synthetic NROM, 8192 envs/GPU')
    assert b.nrom_workload(65536).startswith('config 4 (per GPU)')
    assert '2048 envs/GPU' in b.nrom_workload(2048)


def test_reference_arm_under_torchrun_prints_once():
    """Under torchrun only rank 0 runs the reference arm and prints; the other ranks exit 0 without work."""
    r = subprocess.run([sys.executable, '-m', 'torch.distributed.run', '--nnodes=1', '--nproc-per-node', '2',
                        '--master-addr', '127.0.0.1', '--master-port', '29533', str(ROOT / 'bench.py'),
                        '--impl', 'reference', '--gpus', '2', '--steps', '1', '--warmup', '1'],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith('{')]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    assert d['impl'] == 'reference' and d['n_gpus'] == 2 and d['value'] > 0
