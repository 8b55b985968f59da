"""Benchmark of the batched NES environment step on B200 (the BASELINE metric: decisions/s and NES frames/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--envs E]
    torchrun --nproc-per-node N bench.py --gpus N ...        (one process per GPU, NCCL)

Workload (per GPU): E = 8192 envs of the seeded synthetic NROM cart 'synth00', 4 frames per
decision, sticky moves, dropout and 0..30 idle frames at episode starts on, pictures packed to 6 bits by the
renderer. Weak scaling: every GPU steps its own 8192 envs (seed * 7919 + rank); the per-rollout episode counters
are all-reduced with NCCL every 128 decisions. Every env starts its first episode at the same decision, so --age
(1024) untimed decisions run before the W warm-up decisions: the timed steps see the steady-state restart rate.
  value   decisions/s with everything resident in HBM (env step only, CUDA events on the env's stream).
  e2e     the same through the public API with host buffers: each decision copies its actions host->device from
          pinned memory, steps, and copies the packed pictures (+ emphasis, reward, done, masks) device->host into a
          pinned rollout ring; copies overlap the next decision's step on a copy stream.
  roofline  the render kernel (the dominant one): algorithmic bytes per launch / its CUDA-event time vs the
          measured HBM copy bandwidth (MEASURED_PEAKS.json).
  cpu_baseline  the CPU oracle (restated reference CPU build, OpenMP over envs) on this host's cores, rank 0, N=1.
Prints ONE JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
from pathlib import Path
import re
import statistics
import subprocess
import sys
import threading
import time

# More hardware work queues than CUDA's default 8: a multi-game env runs a main and a side stream per game
# (set before the CUDA context exists; a user of the library sets it the same way).
os.environ.setdefault('CUDA_DEVICE_MAX_CONNECTIONS', '32')

ROOT = Path(__file__).resolve().parent
PKG = ROOT / 'ghostrun-lab_b200'
sys.path.insert(0, str(PKG))

METRIC = 'decisions/s (4 NES frames each)'
UNIT = 'decisions/s'
GAME = 'synth00'


def nrom_workload(envs) -> str:
    """The workload name of the synthetic-NROM line at `envs` envs per GPU: BASELINE config 2 at 8,192, config 4's
    per-GPU size at 65,536, else config 2's workload at that size."""
    envs = int(envs or 8192)
    if envs == 8192:
        return 'config 2: synthetic NROM, 8192 envs/GPU, 4 frames/decision, pack6 on'
    if envs == 65536:
        return 'config 4 (per GPU): synthetic NROM, 65536 envs/GPU, 4 frames/decision, pack6 on'
    return f'config 2 workload at {envs} envs/GPU: synthetic NROM, 4 frames/decision, pack6 on'
PACKED_ROW = 4 * 224 * 240 // 4 * 3   # 161,280 bytes of packed pictures per decision
EMPH_ROW = 4 * 224


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=300)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    ap.add_argument('--envs', type=int, default=None, help='envs per GPU (default 8192; 32768 for --workload config3)')
    ap.add_argument('--workload', default='config2', choices=['config2', 'config3', 'config5', 'stem', 'learner'],
                    help='config2: synthetic NROM (the headline); config3: 12 synthetic games on 4 boards with level '
                         'starts; config5: config 2 with the reference policy network choosing the moves; stem: the '
                         'policy input stem (colour lookup + 2x2 conv, tcgen05) on packed pictures; learner: '
                         'minibatches of rollout rows gathered from a pinned host region and unpacked')
    ap.add_argument('--units', type=int, default=4, help='config5: parts of the envs, each on its own stream')
    ap.add_argument('--seed', type=int, default=1)
    ap.add_argument('--age', type=int, default=1024,
                    help='untimed decisions before the warm-up, so that episode restarts run at their steady-state rate')
    ap.add_argument('--ring', type=int, default=4, help='pinned host rollout slots (decisions) for e2e')
    ap.add_argument('--cpu-leg', action='store_true', help=argparse.SUPPRESS)
    ap.add_argument('--cpu-seconds', type=float, default=15.0)
    ap.add_argument('--cpu-steps', type=int, default=0, help=argparse.SUPPRESS)
    ap.add_argument('--no-cpu', action='store_true')
    return ap.parse_args()


# ------------------------------------------------------------------------------------------------ CPU leg

def cpu_leg(args):
    """Runs in its own process (OMP_NUM_THREADS fixed before the oracle's OpenMP starts). Prints a JSON dict.
    --cpu-steps K: exactly W warm-up + K timed decisions (the reference arm); the env count is cut to a sample of the
    workload when K + W full-size decisions would not fit in --cpu-seconds. Otherwise: as many decisions of the full
    workload as fit in --cpu-seconds (the cpu_baseline leg)."""
    import torch
    from rlenv import RlEnv
    from actions import random_legal
    oracle = ROOT / 'oracle' / 'liboracle_rlenv.so'
    if not oracle.exists():
        subprocess.run(['make', '-C', str(ROOT / 'oracle'), 'all'], check=True, capture_output=True)

    def make(n):
        e = RlEnv({GAME: n}, device='cpu', seed=args.seed * 7919, sticky=True, idle_max=30, dropout=True, lib_path=oracle)
        e.start()
        return e

    E = args.envs
    env = make(E)
    gen = torch.Generator().manual_seed(args.seed)
    env.actions.copy_(random_legal(env.masks, gen)); env.step()
    t0 = time.perf_counter()
    env.actions.copy_(random_legal(env.masks, gen)); env.step()
    one = time.perf_counter() - t0
    if args.cpu_steps > 0:
        K, W = args.cpu_steps, max(args.warmup, 0)
        if (K + W) * one > args.cpu_seconds:
            E = max(256, int(E * args.cpu_seconds / ((K + W) * one)) // 64 * 64)
            env = make(E)
        for _ in range(W):
            env.actions.copy_(random_legal(env.masks, gen)); env.step()
        steps = K
    else:
        steps = int(max(2, min(200, args.cpu_seconds / max(one, 1e-6))))
    t0 = time.perf_counter()
    for t in range(steps):   # every decision's moves drawn from its masks (the sampler's time is part of the step)
        env.actions.copy_(random_legal(env.masks, gen)); env.step()
    dt = time.perf_counter() - t0
    cores = int(os.environ.get('OMP_NUM_THREADS', os.cpu_count()))
    print(json.dumps(dict(value=steps * E / dt, steps=steps, seconds=dt, cores=cores, envs=E, split=cpu_split())))


def cpu_split(frames=600):
    """One thread, one console of the workload's cart: microseconds per frame spent emulating and drawing (the
    reference's rl/bench/split_cpu.cpp method, through the oracle's oracle_split_frames)."""
    import ctypes
    import numpy as np
    from rlenv import synth_cart
    lib = ctypes.CDLL(str(ROOT / 'oracle' / 'liboracle_rlenv.so'))
    cart = synth_cart(GAME)
    rom, boot = np.frombuffer(cart.rom, np.uint8), np.frombuffer(cart.boot_pads, np.uint8)
    out = np.zeros(2)
    rc = lib.oracle_split_frames(rom.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(len(rom)),
                                 boot.ctypes.data_as(ctypes.c_void_p), len(boot), frames, out.ctypes.data_as(ctypes.c_void_p))
    if rc != 0:
        return None
    return dict(emulate_us_per_frame=round(float(out[0]), 2), draw_us_per_frame=round(float(out[1]), 2),
                frames=frames, threads=1, method='rl/bench/split_cpu.cpp (emulate = step_until, draw = render_obs)')


def run_cpu_leg(args, seconds, steps=0):
    cmd = [sys.executable, __file__, '--cpu-leg', '--envs', str(args.envs), '--seed', str(args.seed),
           '--warmup', str(args.warmup), '--cpu-seconds', str(seconds), '--cpu-steps', str(steps)]
    envv = dict(os.environ, OMP_NUM_THREADS=str(os.cpu_count()), CUDA_VISIBLE_DEVICES='')
    out = subprocess.run(cmd, capture_output=True, text=True, env=envv, timeout=900)
    if out.returncode != 0:
        raise RuntimeError(out.stderr[-2000:])
    return json.loads(out.stdout.strip().splitlines()[-1])


def cpu_model():
    try:
        for line in Path('/proc/cpuinfo').read_text().splitlines():
            if line.startswith('model name'):
                return line.split(':', 1)[1].strip()
    except OSError:
        pass
    return 'unknown'


# ------------------------------------------------------------------------------------------------ clocks

class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled while the timed region runs: NVML read-only queries every
    10 ms from a thread (a timed region of a few tens of milliseconds still gets samples), else nvidia-smi every
    200 ms. `index` is the CUDA device; NVML finds the same GPU by its PCI bus id."""
    Q = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,'
         'clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,'
         'clocks_event_reasons.sw_power_cap')
    # NVML clock-event reason bits
    BITS = {'sw_power_cap': 0x4, 'hw_slowdown': 0x8, 'sw_thermal_slowdown': 0x20, 'hw_thermal_slowdown': 0x40,
            'hw_power_brake_slowdown': 0x80}

    def __init__(self, index):
        self.index, self.proc, self.lines = index, None, []
        self.samples, self.stop, self.nvml = [], threading.Event(), None

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        pr = torch.cuda.get_device_properties(self.index)
        bus = f'{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0'
        return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)

    def _poll(self):
        nv, h = self.nvml
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        while not self.stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                self.samples.append((sm, mx, rs))
            except Exception:
                pass
            self.stop.wait(0.01)

    def __enter__(self):
        try:
            self.nvml = self._nvml_handle()
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            return self
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--query-gpu={self.Q}', '--format=csv,noheader,nounits',
                                          '-i', str(self.index), '-lms', '200'], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.nvml is not None:
            self.stop.set()
            self.t.join(timeout=2)
            return
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], [], set()
        if self.nvml is not None:
            for a, b, rs in self.samples:
                sm.append(float(a)); mx.append(float(b))
                reasons.update(n for n, bit in self.BITS.items() if rs & bit)
            src = 'nvml 10 ms'
        else:
            names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
            for line in self.lines:
                f = [x.strip() for x in line.split(',')]
                if len(f) < 9:
                    continue
                try:
                    sm.append(float(f[1])); mx.append(float(f[2]))
                except ValueError:
                    continue
                for n, v in zip(names, f[5:9]):
                    if v.lower().startswith('active'):
                        reasons.add(n)
            src = 'nvidia-smi 200 ms'
        if not sm:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=[], samples=0, source=src)
        return dict(sm_mhz=statistics.median(sm), sm_max_mhz=max(mx), reasons=sorted(reasons), samples=len(sm),
                    source=src)


# ------------------------------------------------------------------------------------------------ GPU arm

def measured_peaks():
    p = ROOT / 'MEASURED_PEAKS.json'
    if p.exists():
        d = json.loads(p.read_text())
        return float(d['hbm_gbs']), 'measured'
    return 6650.0, 'fallback'


def profile_instructions(kernel):
    """(warp instructions of one main-pass launch, envs of that capture) from the committed ncu summary of `kernel`
    on the synthetic NROM workload, or None."""
    p = ROOT / 'profiles' / f'{kernel}_synth00.md'
    if p.exists():
        t = p.read_text()
        m, e = re.search(r'warp_instructions_per_launch:\s*([0-9]+)', t), re.search(r'profile_envs:\s*([0-9]+)', t)
        if m and e:
            return int(m.group(1)), int(e.group(1))
    return None


# Output bytes of one env and decision with packed pictures: packed rows + emphasis + masks + timeline + pads + reward +
# done + events + info + parts (rl/csrc/rlenv_api.h:15-19 shapes)
OUTPUT_BYTES_PACK6 = PACKED_ROW + EMPH_ROW + 19 + 360 + 4 + 4 + 1 + 4 + 32 + 28


def render_traffic_per_env_frame():
    """DRAM bytes per rendered (env, frame) from the committed ncu summary of the render kernel, if any."""
    p = ROOT / 'profiles' / 'k_render_synth00.md'
    if p.exists():
        m = re.search(r'traffic_bytes_per_env_frame:\s*([0-9.]+)', p.read_text())
        if m:
            return float(m.group(1))
    return None


def random_words(shape, gen, dev):
    """int32 random bits for RlEnv.legal_moves (one word per env and decision), drawn on `dev`."""
    import torch
    return torch.randint(-2 ** 31, 2 ** 31, shape, generator=gen, device=dev, dtype=torch.int64).to(torch.int32)


def workload_config(args, world):
    """The `config` both arms report for the NROM workloads (the driver compares the two arms' configs)."""
    return dict(workload=nrom_workload(args.envs), envs_per_gpu=args.envs, frames_per_decision=4,
                moves='each decision: every move part uniform among the choices the last masks allow '
                      '(rl/actions.py random_legal)',
                sticky=True, dropout=True, idle_max=30, pack6=True, parallelism=f'dp{world}',
                inputs_exceed_l2=True, l2_note='per-step state + outputs > 1.5 GB (L2 is 126 MB)')


def rank_seed_for_stem(seed):
    from shard import rank_seed
    return rank_seed(seed, 0)


def stem_arm(args):
    """The policy's input stem (rl_stem_fwd, tcgen05) on B = --envs samples of 6-bit packed pictures: samples/s.
    Roofline: HBM bytes (packed pictures + emphasis in, bf16 features out) per call / its CUDA-event time."""
    import torch
    from stem import fused_stem
    B, K, W = args.envs, args.steps, args.warmup
    dev = torch.device('cuda', 0)
    g = torch.Generator(device=dev).manual_seed(args.seed)
    obs6 = torch.randint(0, 256, (B, 4, 224, 180), generator=g, device=dev, dtype=torch.int32).to(torch.uint8)
    emph = torch.randint(0, 8, (B, 4, 224), generator=g, device=dev, dtype=torch.int32).to(torch.uint8)
    pal = torch.rand(512, 3, generator=g, device=dev)
    w = torch.randn(16, 12, 2, 2, generator=g, device=dev) * 0.2
    b = torch.randn(16, generator=g, device=dev) * 0.1
    for _ in range(W):
        fused_stem(obs6, emph, pal, w, b, packed=True, check=False)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(0)
    with clk:
        e0.record()
        for _ in range(K):
            out = fused_stem(obs6, emph, pal, w, b, packed=True, check=False)
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / K
    in_bytes = obs6.numel() + emph.numel()
    out_bytes = out.numel() * 2
    peak, kind = measured_peaks()
    achieved = (in_bytes + out_bytes) / (ms / 1e3) / 1e9
    # backward (rl_stem_bwd): reads the output gradient and the packed pictures again, writes dW / dbias
    from stem import palette4, stem_backward
    gout = (torch.randn(B, 112, 120, 16, generator=g, device=dev) * 0.1).to(torch.bfloat16)
    pal4 = palette4(pal)
    for _ in range(W):
        stem_backward(gout, obs6, emph, pal4, packed=True, check=False)
    torch.cuda.synchronize()
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    b0.record()
    for _ in range(K):
        stem_backward(gout, obs6, emph, pal4, packed=True, check=False)
    b1.record()
    torch.cuda.synchronize()
    bwd_ms = b0.elapsed_time(b1) / K
    bwd_bytes = in_bytes + gout.numel() * 2
    # the same on pictures the env drew (synth00, aged 64 decisions): runs of equal colours make the palette gathers
    # broadcasts instead of bank conflicts
    from rlenv import RlEnv
    env = RlEnv({GAME: B}, device=dev, seed=rank_seed_for_stem(args.seed), sticky=True, idle_max=30, dropout=True)
    env_px = torch.empty(B, 4, 224, 180, dtype=torch.uint8, device=dev)
    env.bind_obs_pack6(env_px)
    env.start()
    for _ in range(64):
        env.legal_moves(random_words((B,), g, dev))
        env.step()
    env_emph = env.emph.clone()
    del env
    for _ in range(W):
        fused_stem(env_px, env_emph, pal, w, b, packed=True, check=False)
        stem_backward(gout, env_px, env_emph, pal4, packed=True, check=False)
    torch.cuda.synchronize()
    r0, r1, r2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    r0.record()
    for _ in range(K):
        fused_stem(env_px, env_emph, pal, w, b, packed=True, check=False)
    r1.record()
    for _ in range(K):
        stem_backward(gout, env_px, env_emph, pal4, packed=True, check=False)
    r2.record()
    torch.cuda.synchronize()
    env_fwd_ms, env_bwd_ms = r0.elapsed_time(r1) / K, r1.elapsed_time(r2) / K
    # e2e: the learner's view - the packed rollout slice from pinned host memory, the stem, a per-channel mean back
    host6 = obs6.cpu().pin_memory()
    hoste = emph.cpu().pin_memory()
    d6, de = torch.empty_like(obs6), torch.empty_like(emph)
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(K):
        d6.copy_(host6, non_blocking=True)
        de.copy_(hoste, non_blocking=True)
        o = fused_stem(d6, de, pal, w, b, packed=True, check=False)
        m = o.float().mean(dim=(0, 2, 3)).cpu()
    f1.record()
    torch.cuda.synchronize()
    ems = f0.elapsed_time(f1) / K
    return dict(metric='stem samples/s (4-frame pictures -> 16x112x120 bf16 features)', value=round(B / (ms / 1e3), 1),
                unit='samples/s', n_gpus=1, steps=K, warmup=W, ms_per_step=round(ms, 4), higher_is_better=True,
                scaling='weak', vs_baseline=None, dtype='bf16', data='synthetic (random packed pictures, palette, weights)',
                config=dict(workload=f'policy input stem, {B} samples of 6-bit packed pictures', batch=B,
                            inputs_exceed_l2=True),
                e2e=dict(value=round(B / (ems / 1e3), 1), unit='samples/s', h2d_bytes_per_step=in_bytes,
                         d2h_bytes_per_step=16 * 4),
                roofline=dict(bound='hbm', achieved=round(achieved, 1), peak=peak, unit='GB/s', frac=round(achieved / peak, 4),
                              traffic=None, kernel='k_stem_fwd<packed>', bytes_per_call=in_bytes + out_bytes,
                              peak_source=f'{kind} (MEASURED_PEAKS.json hbm_gbs)' if kind == 'measured' else 'fallback'),
                env_pictures=dict(note='the same calls on pictures the env drew (synth00, 64 decisions in)',
                                  fwd_ms=round(env_fwd_ms, 4), bwd_ms=round(env_bwd_ms, 4),
                                  fwd_frac=round((in_bytes + out_bytes) / (env_fwd_ms / 1e3) / 1e9 / peak, 4)),
                backward=dict(ms=round(bwd_ms, 4), samples_per_s=round(B / (bwd_ms / 1e3), 1),
                              achieved_gbs=round(bwd_bytes / (bwd_ms / 1e3) / 1e9, 1),
                              frac=round(bwd_bytes / (bwd_ms / 1e3) / 1e9 / peak, 4), bytes_per_call=bwd_bytes,
                              kernel='k_stem_bwd<packed> + k_stem_bwd_reduce'),
                gpu_launches=K, clocks=clk.summary(), cpu_baseline=None,
                checksum=[round(float(x), 5) for x in m[:4]])


def learner_arm(args):
    """The learner half of the packed picture format (rl/train.py:262-295 HostObs._fetch): T decisions of packed rows
    and emphasis of --envs envs (at most 2,048: the pinned region is T x envs x 162,176 bytes) written by the env into
    a pinned host region, then K minibatches of 256 random envs gathered back to the device, one copy-engine 2-D copy
    per env (rl_gather_envs), and unpacked to colour numbers (rl_unpack6). value: env-decisions of rollout rows
    gathered per second; GB/s against a plain pinned host->device copy of the same bytes."""
    import ctypes
    import numpy as np
    import torch
    from rlenv import RlEnv
    dev = torch.device('cuda', 0)
    E, T, B, K, W = min(args.envs, 2048), 16, 256, args.steps, args.warmup
    row, erow = PACKED_ROW, EMPH_ROW
    env = RlEnv({GAME: E}, device=dev, seed=args.seed * 7919, sticky=True, idle_max=30, dropout=True)
    packed = torch.empty(E, 4, 224, 180, dtype=torch.uint8, device=dev)
    env.bind_obs_pack6(packed)
    env.start()
    lib = env.lib
    s = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    host, host_e = lib.rl_host_alloc(T * E * row), lib.rl_host_alloc(T * E * erow)
    if not host or not host_e:
        raise RuntimeError('rl_host_alloc failed')
    g = torch.Generator(device=dev).manual_seed(args.seed)
    try:
        for t in range(T):   # the rollout: every decision's rows into slot t of the host region
            env.legal_moves(random_words((E,), g, dev))
            env.step()
            lib.rl_memcpy_async(ctypes.c_void_p(host + t * E * row), ctypes.c_void_p(packed.data_ptr()), E * row, s)
            lib.rl_memcpy_async(ctypes.c_void_p(host_e + t * E * erow), ctypes.c_void_p(env.emph.data_ptr()), E * erow, s)
        torch.cuda.synchronize(dev)
        rng = np.random.default_rng(args.seed)
        picks = [np.ascontiguousarray(rng.permutation(E)[:B].astype(np.int64)) for _ in range(K + W)]
        dst = torch.empty(T, B, row, dtype=torch.uint8, device=dev)
        dst_e = torch.empty(T, B, erow, dtype=torch.uint8, device=dev)
        obs = torch.empty(T, B, 4, 224, 240, dtype=torch.uint8, device=dev)

        def batch(k):
            envs = picks[k]
            lib.rl_gather_envs(ctypes.c_void_p(dst.data_ptr()), ctypes.c_void_p(host), envs.ctypes.data_as(ctypes.c_void_p),
                               B, T, E, row, s)
            lib.rl_gather_envs(ctypes.c_void_p(dst_e.data_ptr()), ctypes.c_void_p(host_e),
                               envs.ctypes.data_as(ctypes.c_void_p), B, T, E, erow, s)
            lib.rl_unpack6(ctypes.c_void_p(dst.data_ptr()), ctypes.c_void_p(obs.data_ptr()), obs.numel(), s)

        for k in range(W):
            batch(k)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clk = ClockSampler(0)
        with clk:
            e0.record()
            for k in range(K):
                batch(W + k)
            e1.record()
            torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / K
        moved = T * B * (row + erow)
        # the link: one plain pinned host->device copy of the same bytes
        flat = torch.empty(moved, dtype=torch.uint8, device=dev)
        l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        lib.rl_memcpy_async(ctypes.c_void_p(flat.data_ptr()), ctypes.c_void_p(host), moved, s)
        l0.record()
        for _ in range(3):
            lib.rl_memcpy_async(ctypes.c_void_p(flat.data_ptr()), ctypes.c_void_p(host), moved, s)
        l1.record()
        torch.cuda.synchronize(dev)
        link = 3 * moved / (l0.elapsed_time(l1) / 1e3) / 1e9
        # the unpack alone (device side of the minibatch)
        u0, u1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        u0.record()
        for _ in range(K):
            lib.rl_unpack6(ctypes.c_void_p(dst.data_ptr()), ctypes.c_void_p(obs.data_ptr()), obs.numel(), s)
        u1.record()
        torch.cuda.synchronize(dev)
        ums = u0.elapsed_time(u1) / K
        peak, kind = measured_peaks()
        unpack_gbs = (dst.numel() + obs.numel()) / (ums / 1e3) / 1e9
    finally:
        torch.cuda.synchronize(dev)
        lib.rl_host_free(ctypes.c_void_p(host))
        lib.rl_host_free(ctypes.c_void_p(host_e))
    gbs = moved / (ms / 1e3) / 1e9
    return dict(metric='rollout rows gathered (env-decisions/s: pinned host -> device + unpack)',
                value=round(T * B / (ms / 1e3), 1), unit='env-decisions/s', n_gpus=1, steps=K, warmup=W,
                ms_per_step=round(ms, 4), higher_is_better=True, scaling='weak', vs_baseline=None, dtype='u8',
                data='synthetic (seeded NROM cart synth00, random legal moves)',
                config=dict(workload=f'learner minibatch: {B} of {E} envs x {T} decisions of packed rows from pinned '
                                     'host memory, gathered and unpacked', envs=E, decisions=T, minibatch=B,
                            inputs_exceed_l2=True),
                e2e=dict(value=round(T * B / (ms / 1e3), 1), unit='env-decisions/s', h2d_bytes_per_step=moved,
                         d2h_bytes_per_step=0, note='the whole step is the host -> device gather'),
                link=dict(achieved_gbs=round(gbs, 1), plain_copy_gbs=round(link, 1), frac=round(gbs / link, 3)),
                roofline=dict(bound='host link', achieved=round(gbs, 1), peak=round(link, 1), unit='GB/s',
                              frac=round(gbs / link, 3), traffic=None, kernel='rl_gather_envs (copy engine)',
                              peak_source='measured here: one pinned host->device copy of the same bytes'),
                unpack=dict(ms=round(ums, 4), achieved_gbs=round(unpack_gbs, 1), frac=round(unpack_gbs / peak, 4),
                            peak=peak, kernel='k_unpack6'),
                gpu_launches=K, clocks=clk.summary(), cpu_baseline=None)


def config5_arm(args):
    """E envs per GPU of config 2's cart with the reference's policy network (random init, bf16)
    choosing every move, as the reference's per-unit rollout (rl/train.py:569-652): the envs are split into --units
    parts, each running its own chain (stem + CNN + MLP + GRU + ordered heads -> moves -> its env step_range) on its
    own CUDA stream, so one part's inference overlaps another's emulation. decisions/s.
      value  the rollout with everything on the device (moves sampled on the device: no host inputs).
      e2e    the same, plus each decision's rollout storage read back to pinned host memory on the part's stream:
             packed pictures, emphasis, reward, done, log-probability.
    Also measured alone in the same process: the env (plain step, random moves) and the policy (one unit)."""
    import torch
    import torch.distributed as dist
    from rlenv import RlEnv, default_lib
    from shard import rank_seed
    from policy import Policy
    import build as gbuild

    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        import datetime
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120), device_id=dev)
    if not default_lib().exists():
        gbuild.build()
    E, K, W, U = args.envs, args.steps, args.warmup, max(1, args.units)
    # the reference rollout's settings (rl/train.py:342-345): cuDNN picks its fastest algorithms, TF32 allowed
    torch.backends.cudnn.benchmark = True
    torch.backends.cuda.matmul.allow_tf32 = True
    torch.backends.cudnn.allow_tf32 = True
    env = RlEnv({GAME: E}, device=dev, seed=rank_seed(args.seed, rank), sticky=True, idle_max=30, dropout=True)
    packed = torch.empty(E, 4, 224, 180, dtype=torch.uint8, device=dev)
    env.bind_obs_pack6(packed)
    env.start()
    g = torch.Generator(device=dev).manual_seed(args.seed + rank)
    for _ in range(args.age):   # spread the first episodes' ends to the steady-state restart rate
        env.legal_moves(random_words((E,), g, dev))
        env.step()
    torch.manual_seed(args.seed)
    palette = torch.rand(512, 3, generator=torch.Generator().manual_seed(args.seed))   # a seeded stand-in colour table
    pol = Policy(palette).to(dev).to(memory_format=torch.channels_last).eval()
    n_params = sum(p.numel() for p in pol.parameters())
    cuts = [E * j // U for j in range(U + 1)]
    units = [slice(cuts[j], cuts[j + 1]) for j in range(U)]
    streams = [torch.cuda.Stream(dev) for _ in range(U)]
    gens = [torch.Generator(device=dev).manual_seed(args.seed * 1000 + rank * 16 + j) for j in range(U)]
    h = torch.zeros(E, 512, device=dev)
    prev = [torch.zeros(E, dtype=torch.long, device=dev) for _ in range(5)]
    starts = torch.ones(E, dtype=torch.bool, device=dev)
    ends = torch.zeros(U, dtype=torch.float64, device=dev)
    R = max(2, args.ring)
    row = PACKED_ROW + EMPH_ROW + 4 + 1 + 4
    ring = torch.empty((R, E * row), dtype=torch.uint8).pin_memory()

    def unit_step(j, t, store):
        sl, n = units[j], units[j].stop - units[j].start
        mv, parts, logp, _, hj = pol.decide(packed[sl], env.emph[sl], env.timeline[sl], [p[sl] for p in prev],
                                            env.masks[sl], h[sl], starts[sl], gens[j])
        h[sl] = hj
        env.actions[sl] = mv
        env.step_range(0, sl.start, n, env.obs, env.emph)
        done = env.done[sl].bool()
        starts[sl] = done
        for k in range(5):
            prev[k][sl] = parts[k] * (~done).long()
        ends[j] += done.sum()
        if store:   # this part's rollout rows into the pinned ring slot of step t
            slot = ring[t % R]
            a = sl.start
            slot[a * PACKED_ROW:sl.stop * PACKED_ROW].copy_(packed[sl].view(-1), non_blocking=True)
            b0 = E * PACKED_ROW
            slot[b0 + a * EMPH_ROW:b0 + sl.stop * EMPH_ROW].copy_(env.emph[sl].view(-1), non_blocking=True)
            b1 = b0 + E * EMPH_ROW
            slot[b1 + a * 4:b1 + sl.stop * 4].copy_(env.reward[sl].view(torch.uint8), non_blocking=True)
            b2 = b1 + E * 4
            slot[b2 + a:b2 + sl.stop].copy_(env.done[sl], non_blocking=True)
            b3 = b2 + E
            slot[b3 + a * 4:b3 + sl.stop * 4].copy_(logp.view(torch.uint8), non_blocking=True)

    def rollout(steps, t0, store):
        main = torch.cuda.current_stream(dev)
        for q in streams:
            q.wait_stream(main)
        for t in range(steps):
            for j in range(U):
                with torch.cuda.stream(streams[j]):
                    unit_step(j, t0 + t, store)
        for q in streams:
            main.wait_stream(q)

    def timed(fn):
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize(dev)
        ms = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return float(ms.item())

    rollout(W, 0, False)
    env.set_timing(True)
    env.timing(reset=True)
    clk = ClockSampler(local)
    with clk:
        ms = timed(lambda: rollout(K, 0, False))
    tm = env.timing(reset=True)
    env.set_timing(False)
    rollout(1, 0, True)   # warm the copy path
    ms_e2e = timed(lambda: rollout(K, 0, True))

    # the two halves alone, same process: the env with random legal moves, the policy on all envs as one unit
    words = random_words((K, E), g, dev)

    def env_only():
        for t in range(K):
            env.legal_moves(words[t])
            env.step()

    def policy_only():
        hh = h.clone()
        for _ in range(K):
            pol.decide(packed, env.emph, env.timeline, prev, env.masks, hh, starts, gens[0])

    ms_env = timed(env_only)
    ms_pol = timed(policy_only)
    tot = ends.sum()
    if world > 1:
        dist.all_reduce(tot)
    res = None
    if rank == 0:
        value = K * E * world / (ms / 1e3)
        peak, peak_kind = measured_peaks()
        render_ms = tm['ms']['render'] / K
        alg_bytes = E * 4 * (PACKED_ROW // 4 + 224 + 2048 + 256 + 64)
        achieved = alg_bytes / (render_ms / 1e3) / 1e9
        res = dict(
            metric=METRIC, value=round(value, 1), unit=UNIT, n_gpus=world, steps=K, warmup=W,
            ms_per_step=round(ms / K, 4), higher_is_better=True, scaling='weak', vs_baseline=None, dtype='u8+bf16',
            data='synthetic (seeded NROM cart synth00; random-init policy, seeded stand-in palette)',
            config=dict(workload=f'config 5: config 2 cart, {E} envs/GPU + the reference policy network '
                                 f'({n_params} parameters, bf16) choosing every move, {U} parts on their own streams',
                        envs_per_gpu=E, units=U, policy_parameters=n_params, frames_per_decision=4,
                        parallelism=f'dp{world} (env + policy shards)', aged_decisions=args.age,
                        inputs_exceed_l2=True),
            frames_per_s=round(4 * value, 1),
            e2e=dict(value=round(K * E * world / (ms_e2e / 1e3), 1), unit=UNIT, h2d_bytes_per_step=0,
                     d2h_bytes_per_step=E * row,
                     note='moves come from the policy on the device; each decision\'s packed pictures, emphasis, '
                          'reward, done and log-probability go to a pinned host ring on the part\'s stream'),
            alone=dict(env_ms_per_step=round(ms_env / K, 4), policy_ms_per_step=round(ms_pol / K, 4),
                       env_decisions_per_s=round(K * E / (ms_env / 1e3), 1),
                       policy_decisions_per_s=round(K * E / (ms_pol / 1e3), 1)),
            roofline=dict(bound='hbm', achieved=round(achieved, 1), peak=peak, unit='GB/s', frac=round(achieved / peak, 4),
                          traffic=None, kernel='k_render',
                          peak_source=f'{peak_kind} (MEASURED_PEAKS.json hbm_gbs)' if peak_kind == 'measured' else 'fallback',
                          render_ms_per_decision=round(render_ms, 4)),
            kernel_ms_per_step={k: round(v / K, 4) for k, v in tm['ms'].items()},
            gpu_launches=tm['total_launches'] + K * U,   # env kernels + one stem launch per part and decision
            clocks=clk.summary(), episodes_ended=int(tot.item()), cpu_baseline=None)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return res


def gpu_arm(args):
    import numpy as np
    import torch
    import torch.distributed as dist
    from rlenv import RlEnv, default_lib
    from shard import EpisodeCounters, rank_seed
    import build as gbuild

    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        import datetime
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120), device_id=dev)
    if not default_lib().exists():
        gbuild.build()
    E = args.envs
    c3 = args.workload == 'config3'
    if c3:   # 12 game ids round-robin over the 4 boards, 16 level-start slots per game
        games = [f'synth{k:02d}' for k in range(12)]
        counts = {gname: E // 12 + (1 if k < E % 12 else 0) for k, gname in enumerate(games)}
        env = RlEnv(counts, device=dev, seed=rank_seed(args.seed, rank), sticky=True, idle_max=30, dropout=True,
                    level_cap=16)
    else:
        env = RlEnv({GAME: E}, device=dev, seed=rank_seed(args.seed, rank), sticky=True, idle_max=30, dropout=True)
    packed = [torch.empty(E * PACKED_ROW, dtype=torch.uint8, device=dev) for _ in range(2)]
    env.bind_obs_pack6(packed[0])
    env.start()
    # moves: each decision, every move part uniform among the choices the last masks allow (the reference sampler's
    # distribution), drawn on the device by the library's sampler kernel from random words made up front
    g = torch.Generator(device=dev).manual_seed(args.seed + rank)
    K, W = args.steps, args.warmup
    words_dev = random_words((K + W, E), g, dev)
    counters = EpisodeCounters(dev)

    def account():
        counters.account(env)

    stream = torch.cuda.current_stream(dev)
    # every env starts its first episode at once; aging spreads the episode ends to the steady-state restart rate
    right = torch.full((E,), 3, dtype=torch.int16, device=dev)   # d-pad choice 3 (Right), nothing else pressed
    for t in range(args.age):
        env.legal_moves(random_words((E,), g, dev))
        if c3:   # level-entrance slots fill by play: every env holds Right first (where its mask allows), half of
            # them throughout
            if t == 20:
                env.set_level_prob(1.0)
            hold = ((torch.arange(E, device=dev) % 2 == 0) | (t < args.age // 2)) & (env.masks[:, 3] != 0)
            env.actions.copy_(torch.where(hold, right, env.actions))
        env.step()
    lv_info = None
    if c3:   # every new episode starts from a saved slot, Dirichlet(1) weights over each game's saved slots
        import numpy as np
        rng = np.random.default_rng(args.seed + rank)
        saved = env.saved_levels()
        for gi, gname in enumerate(env.games):
            lv = sorted(saved[gname])
            if lv:
                w = np.zeros(16)
                w[lv] = rng.dirichlet(np.ones(len(lv)))
                env.set_level_plan(gi, 1.0, w)
        lv_info = {gname: len(v) for gname, v in saved.items()}
    counters.attach(env)   # the finishing kernel adds the counters from here on (account() is then a no-op)
    for t in range(W):
        env.legal_moves(words_dev[t]); env.step(); account()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()

    # ---- value: device-resident; CUDA events around the render launches only (the roofline kernel; events around
    # every launch cost ~5% of the step)
    env.set_timing(True, kinds=('render',))
    env.timing(reset=True)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(local)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    with clk:
        ev0.record(stream)
        for t in range(K):
            env.legal_moves(words_dev[W + t])
            env.step()
            account()
            if (t + 1) % 128 == 0:
                counters.rollout_end()
        counters.rollout_end()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    tm = env.timing(reset=True)
    env.set_timing(False)
    ms_t = torch.tensor([ms], device=dev, dtype=torch.float64)
    per_rank = [ms]
    if world > 1:   # every rank's device time (the same collective on every rank), then the max
        gathered = [torch.zeros_like(ms_t) for _ in range(world)]
        dist.all_gather(gathered, ms_t)
        per_rank = [float(x.item()) for x in gathered]
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    value = K * E * world / (ms_max / 1e3)
    # per-kernel breakdown: the same K decisions again with every launch timed (not part of value)
    env.set_timing(True)
    env.timing(reset=True)
    for t in range(K):
        env.legal_moves(words_dev[W + t])
        env.step()
        account()
        if (t + 1) % 128 == 0:
            counters.rollout_end()
    counters.rollout_end()
    torch.cuda.synchronize(dev)
    tm_all = env.timing(reset=True)
    env.set_timing(False)

    # ---- e2e: public API with host buffers (pinned), copies overlapped on a copy stream
    R = max(2, args.ring)
    host_words = random_words((K, E), torch.Generator().manual_seed(args.seed + 7919 * rank), 'cpu').pin_memory()
    words_buf = torch.empty(E, dtype=torch.int32, device=dev)
    ring = torch.empty((R, E * (PACKED_ROW + EMPH_ROW)), dtype=torch.uint8).pin_memory()
    small = torch.empty((R, E * (4 + 1 + 19)), dtype=torch.uint8).pin_memory()
    copy = torch.cuda.Stream(dev)
    done_ev = [torch.cuda.Event() for _ in range(2)]
    emph_buf = [torch.empty(E * EMPH_ROW, dtype=torch.uint8, device=dev) for _ in range(2)]
    env_obs_emph_keep = env.emph
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h2d = d2h = 0
    e0.record(stream)
    for t in range(K):
        b = t & 1
        stream.wait_event(done_ev[b]) if t >= 2 else None   # the copy of this buffer two steps ago finished
        env.bind_obs_pack6(packed[b])
        env.bind_obs(env.obs, emph_buf[b].view(E, 4, 224))
        words_buf.copy_(host_words[t], non_blocking=True)   # the decision's random bits, host -> device
        h2d += E * 4
        env.legal_moves(words_buf)
        env.step()
        account()
        if (t + 1) % 128 == 0:
            counters.rollout_end()
        # small per-env results on the env's stream (the next step overwrites them), pictures on the copy stream
        sm = small[t % R]
        sm[:E * 4].copy_(env.reward.view(torch.uint8), non_blocking=True)
        sm[E * 4:E * 5].copy_(env.done, non_blocking=True)
        sm[E * 5:].copy_(env.masks.view(-1), non_blocking=True)
        ready = torch.cuda.Event()
        ready.record(stream)
        copy.wait_event(ready)
        with torch.cuda.stream(copy):
            slot = ring[t % R]
            slot[:E * PACKED_ROW].copy_(packed[b], non_blocking=True)
            slot[E * PACKED_ROW:].copy_(emph_buf[b], non_blocking=True)
        d2h += E * (PACKED_ROW + EMPH_ROW + 4 + 1 + 19)
        done_ev[b].record(copy)
    counters.rollout_end()
    stream.wait_stream(copy)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    env.bind_obs(env.obs, env_obs_emph_keep)
    e2e_ms = e0.elapsed_time(e1)
    ems = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ems, op=dist.ReduceOp.MAX)
    e2e_value = K * E * world / (float(ems.item()) / 1e3)

    # host link reference: one pinned D2H copy of a step's bytes
    link = None
    if rank == 0:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ring[0][:packed[0].numel()].copy_(packed[0], non_blocking=True)
        t0.record(stream)
        for _ in range(3):
            ring[0][:packed[0].numel()].copy_(packed[0], non_blocking=True)
        t1.record(stream)
        torch.cuda.synchronize(dev)
        link = 3 * packed[0].numel() / (t0.elapsed_time(t1) / 1e3) / 1e9

    result = None
    if rank == 0:
        peak, peak_kind = measured_peaks()
        # the decision's main render launches (one per game) draw the E envs' 4 frames between them
        render_ms = tm['ms']['render'] / K
        env_frames = E * 4
        alg_bytes = env_frames * (PACKED_ROW // 4 + 224 + 2048 + 256 + 64)   # per decision: packed out, emph, NT, OAM, log header
        achieved = alg_bytes / (render_ms / 1e3) / 1e9
        tr = render_traffic_per_env_frame()
        # the whole step against HBM: outputs + the env state read and written once (S_env = the saved state per env,
        # rlenv_state_bytes / envs)
        s_env = env.lib.rlenv_state_bytes(env.h) / E
        step_bytes = OUTPUT_BYTES_PACK6 + 2 * s_env
        step_gbs = value / world * step_bytes / 1e9
        # issue-slot use of the two hot kernels: warp instructions of a main-pass launch (committed ncu capture,
        # scaled to these envs) / (device time per decision x 148 SMs x 4 schedulers x median SM clock)
        sm_mhz = clk.summary().get('sm_mhz') or 1965.0
        issue = {}
        for kern, kind in (('k_frames', 'frames'), ('k_render', 'render')):
            pi = profile_instructions(kern)
            kms = tm_all['ms'][kind] / K
            if pi and kms > 0:
                inst = pi[0] * E / pi[1]
                issue[kern] = dict(warp_instructions_per_decision=round(inst), ms_per_decision=round(kms, 4),
                                   issue_frac=round(inst / (kms * 1e-3 * 148 * 4 * sm_mhz * 1e6), 4))
        result = dict(
            metric=METRIC, value=round(value, 1), unit=UNIT, n_gpus=world, steps=K, warmup=W,
            ms_per_step=round(ms_max / K, 4), higher_is_better=True, scaling='weak', vs_baseline=None, dtype='u8',
            data='synthetic (seeded NROM cart synth00, random legal moves)' if not c3 else
                 'synthetic (12 seeded games synth00-11 on NROM/UxROM/MMC1/MMC3, random legal moves, half holding '
                 'Right while aging)',
            config=workload_config(args, world) if not c3 else
                   dict(workload=f'config 3: 12 synthetic games on 4 boards, {E} envs/GPU, 16 level-start slots per '
                                 'game, P(level start)=1 with Dirichlet(1) weights, pack6 on',
                        level_slots_saved=lv_info, envs_per_gpu=E, frames_per_decision=4, parallelism=f'dp{world}',
                        inputs_exceed_l2=True, l2_note='per-step state + outputs > 1.5 GB (L2 is 126 MB)'),
            aged_decisions=args.age, collective='NCCL all-reduce of the episode counters every 128 decisions',
            per_rank_ms_per_step=[round(x / K, 4) for x in per_rank],
            frames_per_s=round(4 * value, 1),
            e2e=dict(value=round(e2e_value, 1), unit=UNIT, h2d_bytes_per_step=h2d // K, d2h_bytes_per_step=d2h // K,
                     pinned_ring_slots=R, host_link_gbs=round(link, 1) if link else None,
                     link_achieved_gbs=round(d2h / K * e2e_value / E / world / 1e9, 1),
                     link_frac=round(d2h / K * e2e_value / E / world / 1e9 / link, 3) if link else None,
                     note='packed 6-bit pictures + emphasis + reward/done/masks to a pinned host ring every decision'),
            roofline=dict(bound='hbm', achieved=round(achieved, 1), peak=peak, unit='GB/s', frac=round(achieved / peak, 4),
                          traffic=round(tr * env_frames) if tr else None, kernel='k_render',
                          peak_source=f'{peak_kind} (MEASURED_PEAKS.json hbm_gbs)' if peak_kind == 'measured' else 'fallback',
                          algorithmic_bytes_per_decision=alg_bytes, render_ms_per_decision=round(render_ms, 4),
                          render_launches_per_decision=round(tm['launches']['render'] / K, 2),
                          traffic_note='ncu DRAM bytes of a main render launch per env-frame drawn, x env-frames',
                          issue=issue,
                          step=dict(state_bytes_per_env=round(s_env, 1), output_bytes_per_decision=OUTPUT_BYTES_PACK6,
                                    bytes_per_decision=round(step_bytes), achieved_gbs_per_gpu=round(step_gbs, 1),
                                    frac=round(step_gbs / peak, 4),
                                    note='outputs + 2 x S_env per decision (the whole step as one HBM pass)')),
            kernel_ms_per_step={k: round(v / K, 4) for k, v in tm_all['ms'].items()},
            kernel_ms_note='every launch timed in a second pass of the same K decisions (events around every launch '
                           'slow the step ~5%; the timed pass times the render launches only)',
            gpu_launches=tm['total_launches'],
            clocks=clk.summary(),
            episodes=counters.as_dict(),
        )
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


def main():
    args = parse()
    if args.envs is None:
        args.envs = 32768 if args.workload == 'config3' else 8192
    if args.cpu_leg:
        cpu_leg(args)
        return
    rank = int(os.environ.get('RANK', '0'))
    world = int(os.environ.get('WORLD_SIZE', '1'))
    if args.impl == 'reference':
        # the reference's CPU implementation of the path: the oracle port (the real CPU build needs NeSLE, which
        # is not vendored), all host threads, a bounded sample of config 2
        if rank != 0:
            return
        r = run_cpu_leg(args, seconds=150.0, steps=args.steps)
        sample = f"{r['steps']} timed decisions x {r['envs']} envs" + (
            f" (a sample of the {args.envs}-env workload, sized to end within minutes)" if r['envs'] < args.envs else '')
        line = dict(impl='reference', metric=METRIC, value=round(r['value'], 1), unit=UNIT, n_gpus=world,
                    steps=r['steps'], warmup=args.warmup, ms_per_step=round(1e3 * r['seconds'] / r['steps'], 3),
                    higher_is_better=True, scaling='weak', vs_baseline=None, dtype='u8',
                    data='synthetic (seeded NROM cart synth00, random legal moves)',
                    config=workload_config(args, world), envs_timed=r['envs'],
                    cpu_baseline=dict(value=round(r['value'], 1), unit=UNIT, cores=r['cores'], kind='port',
                                      sample=sample, cpu=cpu_model(),
                                      core_us_per_env_frame=round(r['cores'] * 1e6 / (4 * r['value']), 1),
                                      split_one_thread=r['split']),
                    e2e=dict(value=round(r['value'], 1), unit=UNIT, h2d_bytes_per_step=0, d2h_bytes_per_step=0))
        print(json.dumps(line), flush=True)
        return
    if args.workload == 'stem':
        print(json.dumps(stem_arm(args)), flush=True)
        return
    if args.workload == 'learner':
        print(json.dumps(learner_arm(args)), flush=True)
        return
    if args.workload == 'config5':
        res = config5_arm(args)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            r = run_cpu_leg(args, seconds=args.cpu_seconds)
            cpu = dict(value=round(r['value'], 1), unit=UNIT, cores=r['cores'], kind='port',
                       sample=f"{r['steps']} decisions x {args.envs} envs (config 2 workload)", cpu=cpu_model(),
                       core_us_per_env_frame=round(r['cores'] * 1e6 / (4 * r['value']), 1), split_one_thread=r['split'])
        except Exception as ex:   # reported, never silent
            cpu = dict(value=None, unit=UNIT, cores=os.cpu_count(), kind='port', sample=f'failed: {ex}'[:200])
    res = gpu_arm(args)
    if res is not None:
        res['cpu_baseline'] = cpu
        print(json.dumps(res), flush=True)


if __name__ == '__main__':
    main()
