"""Pins the oracle: the reference library built here (oracle/_ref) reproduces the golden
fixtures that tests/golden/make_golden.py generated from the reference."""
import sys

import numpy as np

from conftest import GOLDEN

sys.path.insert(0, str(GOLDEN))
import make_golden  # noqa: E402


def test_engine_trace_matches_golden(ref_roster):
    g = np.load(GOLDEN / "engine_trace.npz")
    hashes, _, _ = ref_roster.random_play(g["p1"], g["p2"], g["x1"], g["x2"], int(g["frames"]), int(g["seed"]))
    assert np.array_equal(hashes, g["hashes"])


def test_env_trace_matches_golden(roster_raw):
    from t8b._lib import EnvConfig
    g = np.load(GOLDEN / "env_trace.npz")
    config = EnvConfig.from_buffer_copy(g["config"].tobytes())
    digests, actions = make_golden.env_run(roster_raw, int(g["n"]), int(g["steps"]), config, int(g["seed"]),
                                           g["opponents"], g["aggression"], g["scenarios"], g["learner_is_p1"],
                                           g["p1"], g["p2"], 7)
    assert np.array_equal(actions, g["actions"])
    assert np.array_equal(digests, g["digests"])


def test_oracle_state_hash_is_fnv1a_over_words(ref_roster):
    state = ref_roster.reset_state(0, 1, -0.8, 0.8)
    words = state.view(np.uint32)
    h = np.uint64(0xCBF29CE484222325)
    with np.errstate(over="ignore"):
        for w in words:
            h = (h ^ np.uint64(w)) * np.uint64(0x100000001B3)
    from oracle import ref
    import ctypes as C
    assert int(h) == ref.lib().t8ref_state_hash(state.ctypes.data_as(C.c_void_p))
