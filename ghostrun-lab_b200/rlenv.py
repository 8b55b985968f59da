"""Python side of the B200 batched NES environment: a drop-in for the reference's rl/rlenv.py (RlEnv, GAMES, the
same constructor, tensors, methods and error behaviour), over the C-ABI library librlenv_b200.so.

    env = RlEnv({'synth00': 8192}, device='cuda', seed=1)
    env.start()                       # first observation in env.obs / env.emph, legal parts in env.masks
    env.actions.copy_(moves)          # int16 packed move ids, legal under env.masks
    env.step()                        # env.obs, reward, done, masks, timeline, pads, events, info updated in place

Everything stays on the device; nothing is copied to the host per step. The library runs on the GPU only: there is no
CPU fallback. `lib_path` selects another library with the same C-ABI (the tests point it at the CPU oracle).

Games: the reference's 12 commercial slugs keep their rl10 ids 0..11 (their ROMs and RAM readers are not part of this
build), and 14 seeded synthetic games 'synth00'..'synth13' (ids 12..25) run on the synthetic cartridges of synth.py:
game k < 12 uses board ('nrom', 'uxrom', 'mmc1', 'mmc3')[k % 4], synth12 the CNROM board, synth13 the MMC2 board, each
with its own seeded reward weights.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np
import torch

import synth

PKG = Path(__file__).resolve().parent
REF_GAMES = ['smb', 'pacman', 'excitebike', 'contra', 'castlevania', 'gradius', 'zelda', 'tetris', 'tecmobowl', 'kage',
             'finalmission', 'punchout']   # rl/games_manifest.json order = rl10 game ids 0..11
SYNTH_GAMES = [f'synth{k:02d}' for k in range(14)]   # synth12: the CNROM cart, synth13: the MMC2 cart
GAMES = REF_GAMES + SYNTH_GAMES
BOARDS = ('nrom', 'uxrom', 'mmc1', 'mmc3')
CART_SEED, REWARD_SEED = 1000, 2000
OBS_H, OBS_W, FRAMES = 224, 240, 4
MASK_BYTES, TIMELINE, INFO = 19, 8 * 45, 8
PART_NAMES = ('progress', 'level', 'death', 'damage', 'score', 'win', 'stall')
NUM_PARTS = len(PART_NAMES)
END_NAMES = {0: 'none', 1: 'game_over', 2: 'won', 3: 'skip', 4: 'stall', 5: 'fault', 6: 'level_clear', 7: 'frame_limit'}
DUMP_BYTES = 23040


def default_lib() -> Path:
    """The in-tree GPU library (built by ghostrun-lab_b200/build.py, or __graft_entry__.build())."""
    return Path(os.environ.get('RL_CUDA_LIB', PKG / 'librlenv_b200.so'))


def synth_cart(slug: str) -> synth.Cart:
    k = SYNTH_GAMES.index(slug)
    if k == 12:
        return synth.make_cart(CART_SEED + 4, 'cnrom')
    if k == 13:
        return synth.make_cart(CART_SEED + 5, 'mmc2')
    return synth.make_cart(CART_SEED + k % 4, BOARDS[k % 4])


def synth_spec(slug: str) -> np.ndarray:
    k = SYNTH_GAMES.index(slug)
    return synth.reward_spec(REWARD_SEED + k, synth_cart(slug).params)


def _load(path: Path):
    lib = ctypes.CDLL(str(path))
    P, I, U64, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64, ctypes.c_size_t
    lib.rlenv_create.restype = P
    lib.rlenv_create.argtypes = [I, P, P, P, P, P, P, U64, I, I, I, I]
    lib.rlenv_num_envs.argtypes = [P]
    lib.rlenv_bind.argtypes = [P] * 11
    lib.rlenv_bind_parts.argtypes = [P, P]
    lib.rlenv_bind_obs.argtypes = [P, P, P]
    lib.rlenv_start.argtypes = [P, P]
    lib.rlenv_step.argtypes = [P, P]
    lib.rlenv_state_bytes.restype = SZ
    lib.rlenv_state_bytes.argtypes = [P]
    lib.rlenv_save.argtypes = [P, P, P]
    lib.rlenv_load.argtypes = [P, P, P]
    lib.rlenv_error.restype = ctypes.c_char_p
    lib.rlenv_destroy.argtypes = [P]
    lib.rl10_register_game.argtypes = [I, P, I]
    if hasattr(lib, 'rlenv_set_episode_level_end'):
        lib.rlenv_set_episode_level_end.argtypes = [P, I]
    if hasattr(lib, 'rlenv_set_no_render'):
        lib.rlenv_set_no_render.argtypes = [P, I]
    if hasattr(lib, 'rlenv_bind_obs_pack6'):
        lib.rlenv_bind_obs_pack6.argtypes = [P, P]
        lib.rlenv_set_timing.argtypes = [P, I]
        lib.rlenv_timing.argtypes = [P, P, I]
    if hasattr(lib, 'rlenv_set_timing_kinds'):
        lib.rlenv_set_timing_kinds.argtypes = [P, ctypes.c_uint]
    if hasattr(lib, 'rlenv_dump_env'):
        lib.rlenv_dump_env.argtypes = [P, I, P, P]
        lib.rlenv_env_scalars.argtypes = [P, I, P, P]
    if hasattr(lib, 'rlenv_render_stats'):
        lib.rlenv_render_stats.argtypes = [P, P, I, P]
    if hasattr(lib, 'rlenv_enable_places'):
        lib.rlenv_enable_level_starts.argtypes = [P, I]
        lib.rlenv_enable_places.argtypes = [P, I, I]
        lib.rlenv_set_level_plan.argtypes = [P, I, ctypes.c_double, P]
        lib.rlenv_bind_start.argtypes = [P, P]
        lib.rlenv_bind_level.argtypes = [P, P]
        lib.rlenv_bind_progress.argtypes = [P, P]
        lib.rlenv_level_deaths.argtypes = [P, I, P, P]
        lib.rlenv_place_save.argtypes = [P, I, P, P, I, P]
        lib.rlenv_place_copy.argtypes = [P, I, P, P, I, P]
        lib.rlenv_level_layout.argtypes = [P, I, P]
    for name, args in (('rl_pack6', [P, P, SZ, P]), ('rl_unpack6', [P, P, SZ, P]), ('rl_memcpy_async', [P, P, SZ, P]),
                       ('rl_gather_rows', [P, P, P, I, SZ, P]), ('rl_gather_envs', [P, P, P, I, I, I, SZ, P]),
                       ('rlenv_step_game', [P, I, P, P, P]), ('rlenv_step_range', [P, I, I, I, P, P, P]),
                       ('rl_legal_moves', [P, P, P, I, P])):
        if hasattr(lib, name):
            getattr(lib, name).argtypes = args
    if hasattr(lib, 'rl_host_alloc'):
        lib.rl_host_alloc.restype = P
        lib.rl_host_alloc.argtypes = [SZ]
        lib.rl_host_free.argtypes = [P]
    return lib


class RlEnv:
    def __init__(self, counts: dict, device='cuda', seed=0, sticky=True, idle_max=30, dropout=True, roms=None,
                 lib_path=None, level_cap=0, level_slots=None, boot=None):
        """counts: game slug -> number of envs (envs are laid out in GAMES order). roms: optional slug -> iNES bytes
        or path (synthetic slugs default to their generated cartridge); boot: optional slug -> boot pad bytes.
        level_cap > 0: save level starts (levels 0..level_cap-1 of each game, the best arrival of each decision), used
        by new episodes with the chance set by set_level_prob / set_level_plan (default 0). self.start_level: slot a
        finished episode started from, -1 = power-on (valid where done).
        level_slots < level_cap: only slots 0..level_slots-1 are level starts; the rest are places, saved by
        place_save. (rl/rlenv.py:172-243.)"""
        self.device = torch.device(device)
        self.games = [g for g in GAMES if counts.get(g, 0) > 0]
        unknown = set(counts) - set(GAMES)
        if unknown:
            raise ValueError(f'unknown games {sorted(unknown)}')
        self.counts = [int(counts[g]) for g in self.games]
        self.n = sum(self.counts)
        self.game_of_env = torch.tensor(sum(([GAMES.index(g)] * c for g, c in zip(self.games, self.counts)), []),
                                        dtype=torch.long, device=self.device)
        cuda = self.device.type == 'cuda'
        if lib_path is None:
            if not cuda:
                raise RuntimeError('librlenv_b200 runs on the GPU only; pass lib_path= for another build of the C-ABI')
            lib_path = default_lib()
            if not Path(lib_path).exists():
                raise RuntimeError(f'{lib_path} is missing: build it with ghostrun-lab_b200/build.py')
        self.lib = _load(Path(lib_path))
        roms, boot = roms or {}, boot or {}
        rom_bytes, boots = [], []
        for g in self.games:
            if g in SYNTH_GAMES:
                cart = synth_cart(g)
                spec = synth_spec(g)
                if self.lib.rl10_register_game(GAMES.index(g), spec.ctypes.data_as(ctypes.c_void_p), len(spec)) != 0:
                    raise RuntimeError(self.lib.rlenv_error().decode())
                rom_bytes.append(_bytes(roms.get(g, cart.rom)))
                boots.append(bytes(boot.get(g, cart.boot_pads)))
            else:
                if g not in roms or g not in boot:
                    raise RuntimeError(f'{g}: a commercial game needs roms= and boot= (no ROMs ship with this build)')
                rom_bytes.append(_bytes(roms[g]))
                boots.append(bytes(boot[g]))
        self._keep = [rom_bytes, boots]
        arr = lambda T, xs: (T * len(xs))(*xs)  # noqa: E731
        rom_p = arr(ctypes.c_char_p, rom_bytes)
        boot_p = arr(ctypes.c_char_p, boots)
        self._keep += [rom_p, boot_p]
        dev_index = self.device.index if self.device.index is not None else (torch.cuda.current_device() if cuda else 0)
        if cuda:
            torch.cuda.set_device(dev_index)
            torch.zeros(1, device=self.device)   # torch's CUDA context exists first
        self.h = self.lib.rlenv_create(
            len(self.games), arr(ctypes.c_int, [GAMES.index(g) for g in self.games]), rom_p,
            arr(ctypes.c_size_t, [len(r) for r in rom_bytes]), boot_p, arr(ctypes.c_size_t, [len(b) for b in boots]),
            arr(ctypes.c_int, self.counts), seed, int(sticky), int(idle_max), int(dropout), dev_index)
        if not self.h:
            raise RuntimeError(f'rlenv_create: {self.lib.rlenv_error().decode()}')
        N, d = self.n, self.device
        self.actions = torch.zeros(N, dtype=torch.int16, device=d)
        self.obs = torch.zeros(N, FRAMES, OBS_H, OBS_W, dtype=torch.uint8, device=d)
        self.emph = torch.zeros(N, FRAMES, OBS_H, dtype=torch.uint8, device=d)
        self.reward = torch.zeros(N, dtype=torch.float32, device=d)
        self.done = torch.zeros(N, dtype=torch.uint8, device=d)
        self.masks = torch.zeros(N, MASK_BYTES, dtype=torch.uint8, device=d)
        self.timeline = torch.zeros(N, 8, 45, dtype=torch.uint8, device=d)
        self.pads = torch.zeros(N, FRAMES, dtype=torch.uint8, device=d)
        self.events = torch.zeros(N, dtype=torch.int32, device=d)
        self.info = torch.zeros(N, INFO, dtype=torch.float32, device=d)
        p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        self.lib.rlenv_bind(self.h, p(self.actions), p(self.obs), p(self.emph), p(self.reward), p(self.done),
                            p(self.masks), p(self.timeline), p(self.pads), p(self.events), p(self.info))
        self.parts = torch.zeros(N, NUM_PARTS, dtype=torch.float32, device=d)
        self.lib.rlenv_bind_parts(self.h, p(self.parts))
        self.level_cap = int(level_cap)
        self.level_slots = int(level_slots if level_slots is not None else level_cap)
        self.start_level = torch.full((N,), -1, dtype=torch.int32, device=d)
        if self.level_cap > 0:
            rc = (self.lib.rlenv_enable_places(self.h, self.level_cap, self.level_slots) if self.level_slots < self.level_cap
                  else self.lib.rlenv_enable_level_starts(self.h, self.level_cap))
            self._check(rc, 'level starts')
            self.lib.rlenv_bind_start(self.h, p(self.start_level))
            self.level_now = torch.full((N,), -1, dtype=torch.int32, device=d)    # level after the last decision
            self.lib.rlenv_bind_level(self.h, p(self.level_now))
            # within-level progress / one level's progress unit, NaN = not valid now; never an actor input
            self.progress_now = torch.full((N,), float('nan'), dtype=torch.float32, device=d)
            self.lib.rlenv_bind_progress(self.h, p(self.progress_now))

    # ---- level starts and places (rl/rlenv.py:245-310)
    def set_level_prob(self, prob: float):
        """Chance that a new episode starts from a saved level start (uniform over the game's saved levels)."""
        assert self.level_cap > 0 or prob == 0
        for gi in range(len(self.games)):
            self.set_level_plan(gi, prob)

    def set_level_plan(self, gi, prob, weights=None):
        """Game gi's chance of a level start and its slot weights ([level_cap], only saved slots > 0, sum 1; None =
        uniform over the saved slots). Call between decisions."""
        if self.level_cap == 0:
            return
        cdf = None
        if weights is not None:
            w = np.asarray(weights, np.float64)
            cdf = np.minimum(np.cumsum(w) * 2.0 ** 32, 2.0 ** 32 - 1).astype(np.uint32)
            cdf[np.flatnonzero(w)[-1]:] = 2 ** 32 - 1
        if self.device.type == 'cuda':
            torch.cuda.synchronize(self.device)
        self.lib.rlenv_set_level_plan(self.h, gi, float(prob), None if cdf is None else cdf.ctypes.data_as(ctypes.c_void_p))

    def saved_levels(self):
        """game slug -> {level: deaths of the saved arrival} (synchronous)."""
        out = {}
        for gi, g in enumerate(self.games):
            buf = self.level_deaths(gi)
            out[g] = {int(l): int(dd) for l, dd in enumerate(buf[:self.level_slots]) if dd >= 0}
        return out

    def level_deaths(self, gi) -> np.ndarray:
        """Deaths of every saved slot of game gi, -1 = nothing saved (synchronous)."""
        buf = np.full(max(self.level_cap, 1), -1, np.int32)
        if self.level_cap > 0:
            if self.device.type == 'cuda':
                torch.cuda.synchronize(self.device)
            self._check(self.lib.rlenv_level_deaths(self.h, gi, buf.ctypes.data_as(ctypes.c_void_p), self._stream()),
                        'level_deaths')
        return buf[:self.level_cap]

    def place_save(self, gi, env_idx, slot_idx):
        """After a step, on the current stream: env env_idx[j] (index within game gi) -> place slot slot_idx[j]
        (skipped where < level_slots). int32 tensors on the env's device."""
        assert env_idx.dtype == torch.int32 and slot_idx.dtype == torch.int32 and env_idx.is_contiguous()
        self._check(self.lib.rlenv_place_save(self.h, gi, ctypes.c_void_p(env_idx.data_ptr()),
                                              ctypes.c_void_p(slot_idx.data_ptr()), int(env_idx.numel()), self._stream()),
                    'place_save')

    def place_copy(self, gi, src, dst):
        """Slot src[j] -> slot dst[j] of game gi (whole saved state), synchronous."""
        a, b = np.ascontiguousarray(src, np.int32), np.ascontiguousarray(dst, np.int32)
        if len(a):
            self._check(self.lib.rlenv_place_copy(self.h, gi, a.ctypes.data_as(ctypes.c_void_p),
                                                  b.ctypes.data_as(ctypes.c_void_p), len(a), self._stream()), 'place_copy')

    def level_layout(self, gi):
        out = np.zeros(5, np.uint32)
        self.lib.rlenv_level_layout(self.h, gi, out.ctypes.data_as(ctypes.c_void_p))
        return dict(stride=int(out[0]), key_cap=int(out[1]), st=int(out[2]), cap=int(out[3]), levels=int(out[4]))

    def _grow_archive(self, buf, old_cap, need):
        """A state saved with old_cap slots per game -> this env's level_cap (new slots empty); None if buf is not
        such a state. The level-start state is last: per game records, trackers, keys, targets, frames, deaths."""
        lay = [self.level_layout(gi) for gi in range(len(self.games))]
        sizes = lambda cap, l: [cap * l['stride'], cap * l['st'], cap * l['key_cap'] * 4, cap * 8, cap * 4, cap * 4]  # noqa: E731
        old_tail = sum(sum(sizes(old_cap, l)) for l in lay)
        if len(buf) - old_tail + sum(sum(sizes(self.level_cap, l)) for l in lay) != need:
            return None
        out, o = [buf[:len(buf) - old_tail]], len(buf) - old_tail
        for l in lay:
            for k, (a, b) in enumerate(zip(sizes(old_cap, l), sizes(self.level_cap, l))):
                out.append(buf[o:o + a])
                o += a
                out.append(np.full(b - a, 0xFF, np.uint8) if k == 5 else np.zeros(b - a, np.uint8))   # deaths -1 = empty
        return np.concatenate(out)

    # ---- the reference API
    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream if self.device.type == 'cuda' else 0)

    def _check(self, rc, what):
        if rc != 0:
            raise RuntimeError(f'{what}: {self.lib.rlenv_error().decode()}')

    def start(self):
        self._check(self.lib.rlenv_start(self.h, self._stream()), 'rlenv_start')

    def step(self):
        self._check(self.lib.rlenv_step(self.h, self._stream()), 'rlenv_step')

    def step_game(self, gi, obs, emph):
        """Step only the gi-th game (of self.games) on the current stream, its pictures into obs/emph ([N,...] whole
        batch tensors; only that game's rows are written). GPU library only."""
        self._check(self.lib.rlenv_step_game(self.h, gi, ctypes.c_void_p(obs.data_ptr()), ctypes.c_void_p(emph.data_ptr()),
                                             self._stream()), 'rlenv_step_game')

    def step_range(self, gi, start, count, obs, emph):
        """Like step_game, for envs [start, start+count) of the gi-th game only. GPU library only."""
        self._check(self.lib.rlenv_step_range(self.h, gi, start, count, ctypes.c_void_p(obs.data_ptr()),
                                              ctypes.c_void_p(emph.data_ptr()), self._stream()), 'rlenv_step_range')

    def set_episode_level_end(self, level):
        self.lib.rlenv_set_episode_level_end(self.h, int(level))

    def set_no_render(self, value: bool):
        self.lib.rlenv_set_no_render(self.h, int(bool(value)))

    def drop_obs_buffers(self):
        self.obs = self.emph = None

    def bind_obs(self, obs, emph):
        """Write the next pictures into these tensors ([N,4,224,240] / [N,4,224] uint8, contiguous, same device)."""
        assert obs.is_contiguous() and emph.is_contiguous() and obs.shape == (self.n, FRAMES, OBS_H, OBS_W)
        self._obs_keep = (obs, emph)
        self.lib.rlenv_bind_obs(self.h, ctypes.c_void_p(obs.data_ptr()), ctypes.c_void_p(emph.data_ptr()))

    def bind_obs_pack6(self, packed):
        """Let the renderer write the pictures as packed 6-bit colour numbers ([N,4,224,180] uint8, the rl_pack6
        layout of obs) into `packed` instead of filling env.obs; None restores the byte output."""
        if packed is None:
            self.lib.rlenv_bind_obs_pack6(self.h, None)
            self._packed_keep = None
            return
        assert packed.is_contiguous() and packed.dtype == torch.uint8 and packed.numel() == self.n * FRAMES * OBS_H * OBS_W // 4 * 3
        self._packed_keep = packed
        self.lib.rlenv_bind_obs_pack6(self.h, ctypes.c_void_p(packed.data_ptr()))

    def set_timing(self, on: bool, kinds=None):
        """Record CUDA events around kernel launches (per-kernel device time, see timing()); kinds: names of the
        kinds to time (timing() order), None = all."""
        names = ('frames', 'render', 'finish', 'restart_frames', 'restart_render', 'pack6')
        mask = 0xFFFFFFFF if kinds is None else sum(1 << names.index(k) for k in kinds)
        self.lib.rlenv_set_timing_kinds(self.h, mask)
        self.lib.rlenv_set_timing(self.h, int(bool(on)))

    def timing(self, reset=False) -> dict:
        """Per-kernel device milliseconds and launch counts since the last reset."""
        out = np.zeros(13, np.float64)
        self._check(self.lib.rlenv_timing(self.h, out.ctypes.data_as(ctypes.c_void_p), int(bool(reset))), 'timing')
        names = ('frames', 'render', 'finish', 'restart_frames', 'restart_render', 'pack6')
        return dict(ms={k: float(out[i]) for i, k in enumerate(names)},
                    launches={k: int(out[6 + i]) for i, k in enumerate(names)}, total_launches=int(out[12]))

    def legal_moves(self, words):
        """env.actions <- one legal move per env under env.masks, each move part uniform among its allowed choices
        (the distribution of actions.random_legal), drawn from `words` (int32 / uint32 random bits [N] on the env's
        device) by the library's own kernel on the current stream. GPU library only."""
        assert words.numel() == self.n and words.element_size() == 4 and words.is_contiguous()
        self._check(self.lib.rl_legal_moves(ctypes.c_void_p(self.masks.data_ptr()), ctypes.c_void_p(words.data_ptr()),
                                            ctypes.c_void_p(self.actions.data_ptr()), self.n, self._stream()),
                    'rl_legal_moves')

    def render_stats(self, reset=False) -> dict:
        """How the pictures since the last reset were drawn: frames the sequential renderer drew (`seq_frames`) and
        lines with a write inside their drawn part the two-phase renderer drew exactly (`split_lines`). GPU library
        only (synchronous)."""
        out = np.zeros(2, np.uint64)
        self._check(self.lib.rlenv_render_stats(self.h, out.ctypes.data_as(ctypes.c_void_p), int(bool(reset)),
                                                self._stream()), 'render_stats')
        return dict(seq_frames=int(out[0]), split_lines=int(out[1]))

    def game_slices(self):
        out, a = [], 0
        for c in self.counts:
            out.append(slice(a, a + c))
            a += c
        return out

    def state_dict(self) -> dict:
        """Exact resume state of every env plus the observation outputs."""
        buf = np.empty(self.lib.rlenv_state_bytes(self.h), np.uint8)
        if self.device.type == 'cuda':
            torch.cuda.synchronize(self.device)
        self._check(self.lib.rlenv_save(self.h, buf.ctypes.data_as(ctypes.c_void_p), self._stream()), 'rlenv_save')
        outs = {k: getattr(self, k).cpu() for k in ('obs', 'emph', 'masks', 'timeline', 'done', 'reward')
                if getattr(self, k) is not None}
        return dict(env=buf, outputs=outs, games=self.games, counts=self.counts, level_cap=self.level_cap)

    def load_state_dict(self, sd):
        assert sd['games'] == self.games and sd['counts'] == self.counts, 'env layout changed'
        buf = np.ascontiguousarray(sd['env'])
        need = self.lib.rlenv_state_bytes(self.h)
        old_cap = sd.get('level_cap', 64)
        if len(buf) < need and self.level_cap > old_cap > 0:
            grown = self._grow_archive(buf, old_cap, need)
            buf = buf if grown is None else grown
        if len(buf) < need and self.level_cap > 0:
            # saved before level starts were on: the level-start state comes last; take it from this fresh env
            buf = np.concatenate([buf, self.state_dict()['env'][len(buf):]])
        assert len(buf) == need, 'env state size changed'
        if self.device.type == 'cuda':
            torch.cuda.synchronize(self.device)
        self._check(self.lib.rlenv_load(self.h, buf.ctypes.data_as(ctypes.c_void_p), self._stream()), 'rlenv_load')
        for k, v in sd['outputs'].items():
            if getattr(self, k) is not None:
                getattr(self, k).copy_(v)

    # ---- parity / debugging (both the GPU library and the CPU oracle export these)
    def dump(self, env_index: int) -> np.ndarray:
        """Canonical machine state of one env (CPU registers, RAM, PPU, board, shown frame log)."""
        out = np.zeros(DUMP_BYTES, np.uint8)
        if self.device.type == 'cuda':
            torch.cuda.synchronize(self.device)
            rc = self.lib.rlenv_dump_env(self.h, int(env_index), out.ctypes.data_as(ctypes.c_void_p), self._stream())
        else:
            rc = self.lib.oracle_dump_env(ctypes.c_void_p(self.h), int(env_index), out.ctypes.data_as(ctypes.c_void_p))
        self._check(rc, 'dump')
        return out

    def scalars(self, env_index: int) -> np.ndarray:
        """target, ep_frame, episode, fault, sticky counter of one env."""
        out = np.zeros(5, np.uint64)
        if self.device.type == 'cuda':
            torch.cuda.synchronize(self.device)
            rc = self.lib.rlenv_env_scalars(self.h, int(env_index), out.ctypes.data_as(ctypes.c_void_p), self._stream())
        else:
            rc = self.lib.oracle_env_scalars(ctypes.c_void_p(self.h), int(env_index), out.ctypes.data_as(ctypes.c_void_p))
        self._check(rc, 'scalars')
        return out

    def __del__(self):
        if getattr(self, 'h', None):
            self.lib.rlenv_destroy(self.h)
            self.h = None


def _bytes(x) -> bytes:
    if isinstance(x, (bytes, bytearray)):
        return bytes(x)
    return Path(x).read_bytes()
