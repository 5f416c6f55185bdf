"""The counter RNG's shortcuts are exact (CPU, no GPU needed): draw(prefix_of(seed, stream), c)
equals hash3(seed, stream, c), and below_with (a reciprocal quotient estimate plus one
correction) equals the 64-bit remainder of below for the bounds the scripted opponent uses and
for every bound up to 2^20 on random draws. The check compiles a host program from the
library's own contract header with nvcc and runs it on the CPU."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "tekken8-agent_b200" / "csrc"

PROGRAM = r"""
#include "contract.cuh"
#include <cstdio>
using namespace t8b;
int main() {
    uint64_t state = 0x12345678abcdefull, bad = 0, checked = 0;
    const int fixed[] = {1, 2, 3, 7, 22, 100, 187, 346, 65535, 65536, 1048575};
    for (int i = 0; i < 400000; ++i) {
        state = mix64(state);
        const uint64_t bits = state;
        for (int bound : fixed) {
            bad += below_with(bits, bound, 1.0 / bound) != below(bits, bound);
            ++checked;
        }
        const int any = 1 + static_cast<int>(mix64(bits) % 1048575u);
        bad += below_with(bits, any, 1.0 / any) != below(bits, any);
        const uint64_t seed = mix64(bits ^ 1u), stream = bits % 40000u, counter = mix64(bits ^ 2u);
        bad += draw(prefix_of(seed, stream), counter) != hash3(seed, stream, counter);
        checked += 2;
    }
    // extremes of the 64-bit range
    const uint64_t edges[] = {0ull, 1ull, 0xffffffffull, 0x100000000ull, 0xffffffffffffffffull, 0xfffffffffffffffeull,
                              0x8000000000000000ull, 0x7fffffffffffffffull};
    for (uint64_t e : edges) {
        for (int bound = 1; bound < 4096; ++bound) {
            bad += below_with(e, bound, 1.0 / bound) != below(e, bound);
            ++checked;
        }
    }
    std::printf("%llu %llu\n", static_cast<unsigned long long>(checked), static_cast<unsigned long long>(bad));
    return bad == 0 ? 0 : 1;
}
"""


def test_rng_shortcuts_are_exact(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).exists():
        pytest.skip("nvcc is not available")
    src = tmp_path / "rng_check.cu"
    src.write_text(PROGRAM)
    exe = tmp_path / "rng_check"
    subprocess.run([nvcc, "-O2", "-std=c++17", f"-I{CSRC}", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)],
                   check=True, capture_output=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    checked, bad = (int(v) for v in out.stdout.split())
    assert checked > 5_000_000 and bad == 0 and out.returncode == 0
