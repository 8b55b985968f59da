"""The Python drop-in: ghostrun-lab_b200/rlenv.py's RlEnv has the reference class's methods, parameter names and
defaults (rl/rlenv.py:173-386) and sets every public attribute the reference's callers read (rl/train.py,
rl/evaluate.py). The reference's surface is restated here so the check needs nothing outside this repository."""
from __future__ import annotations

import ast
import inspect
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / 'ghostrun-lab_b200'

# rl/rlenv.py: method -> parameter names after self (line of the def)
REFERENCE_METHODS = {
    '__init__': ['counts', 'device', 'seed', 'sticky', 'idle_max', 'dropout', 'roms', 'lib_path', 'level_cap',
                 'level_slots'],                                       # 173
    'set_level_prob': ['prob'],                                        # 240
    'set_level_plan': ['gi', 'prob', 'weights'],                       # 246
    'saved_levels': [],                                                # 260
    'place_save': ['gi', 'env_idx', 'slot_idx'],                       # 273
    'place_copy': ['gi', 'src', 'dst'],                                # 281
    'level_layout': ['gi'],                                            # 288
    'drop_obs_buffers': [],                                            # 311
    'bind_obs': ['obs', 'emph'],                                       # 315
    'set_episode_level_end': ['level'],                                # 324
    'start': [],                                                       # 327
    'step': [],                                                        # 331
    'step_game': ['gi', 'obs', 'emph'],                                # 335
    'step_range': ['gi', 'start', 'count', 'obs', 'emph'],             # 342
    'game_slices': [],                                                 # 348
    'state_dict': [],                                                  # 356
    'load_state_dict': ['sd'],                                         # 367
}
# rl/rlenv.py:173-174: the constructor's defaults
REFERENCE_INIT_DEFAULTS = {'device': 'cuda', 'seed': 0, 'sticky': True, 'idle_max': 30, 'dropout': True,
                           'roms': None, 'lib_path': None, 'level_cap': 0, 'level_slots': None}
# rl/rlenv.py:176-239: public attributes set on the instance
REFERENCE_ATTRIBUTES = ['device', 'games', 'counts', 'n', 'game_of_env', 'lib', 'h', 'actions', 'obs', 'emph', 'reward',
                        'done', 'masks', 'timeline', 'pads', 'events', 'info', 'parts', 'level_cap', 'level_slots',
                        'start_level', 'level_now', 'progress_now']


def _rlenv_class():
    sys.path.insert(0, str(PKG))
    from rlenv import RlEnv
    return RlEnv


def test_methods_and_parameters_match_the_reference():
    cls = _rlenv_class()
    wrong = {}
    for name, want in REFERENCE_METHODS.items():
        fn = getattr(cls, name, None)
        if fn is None:
            wrong[name] = 'missing'
            continue
        params = [p for p in inspect.signature(fn).parameters.values() if p.name != 'self']
        got = [p.name for p in params][:len(want)]
        extra = [p for p in params[len(want):] if p.default is inspect.Parameter.empty]
        if got != want or extra:
            wrong[name] = (got, want, [p.name for p in extra])
    assert not wrong, wrong


def test_constructor_defaults_match_the_reference():
    sig = inspect.signature(_rlenv_class().__init__)
    got = {k: sig.parameters[k].default for k in REFERENCE_INIT_DEFAULTS}
    assert got == REFERENCE_INIT_DEFAULTS


def test_public_attributes_are_set():
    tree = ast.parse((PKG / 'rlenv.py').read_text())
    cls = next(n for n in ast.walk(tree) if isinstance(n, ast.ClassDef) and n.name == 'RlEnv')
    stored = {a.attr for a in ast.walk(cls) if isinstance(a, ast.Attribute) and isinstance(a.value, ast.Name)
              and a.value.id == 'self' and isinstance(a.ctx, ast.Store)}
    missing = [a for a in REFERENCE_ATTRIBUTES if a not in stored]
    assert not missing, missing
