import lzma
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tekken8-agent_b200"))
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built sm_100a library")


@pytest.fixture(scope="session")
def roster_raw() -> bytes:
    return lzma.decompress((GOLDEN / "roster41.bin.xz").read_bytes())


@pytest.fixture(scope="session")
def roster(roster_raw):
    from t8b import roster as roster_module
    return roster_module.parse(roster_raw)


@pytest.fixture(scope="session")
def ref_roster(roster_raw):
    from oracle import ref
    return ref.RefRoster(roster_raw)


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
