"""The legality shortcuts are exact (CPU, no GPU needed): universal_mask, which decides the 22
universal candidates of a fighter once per fight for the warp-parallel mask kernels (k_masks and
the engine-parity random play), and Legality, which the scripted opponents use to check many
candidates of one state (can_act and that word taken once, and no move probed where none can
pass), both equal candidate_ok
(candidate_legal, full_move_contract.hpp:42-49) candidate by candidate, on random fights that
reach every branch: postures, stun, throw-break windows, heat and Heat Dash contacts, knock-down
timers, moves and universals in progress, finished rounds, and move gates with every requirement
flag. The library's scripted random opponent (checking its probes through Legality and skipping
the move probes that cannot pass) also picks the same candidate as probing them one by one
with candidate_ok. The check compiles a host program from the library's own headers with
nvcc."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "tekken8-agent_b200" / "csrc"

PROGRAM = r"""
#include "contract.cuh"
#include <cstdio>
#include <cstring>
#include <vector>
using namespace t8b;
// scripted_candidate (full_move_contract.hpp:90-119) probing one candidate at a time with
// candidate_ok: the form the library's random_opponent must agree with
int random_opponent_one_by_one(const Match& m, const Fight& s, int p, double aggression, uint64_t prefix,
                               uint64_t counter) {
    const DCharacter& ch = *m.side[p];
    const bool close = mag(s.f[p].x - s.f[1 - p].x) < 1.6;
    uint64_t draw_index = 0;
    const int roll = below(draw(prefix, counter * 64u + draw_index++), 100);
    if (!close && roll < 55) {
        const int approach = roll < 30 ? 3 : 1;
        if (candidate_ok(m, s, p, approach)) return approach;
    }
    if (close && roll < 15) {
        const int guard = roll < 8 ? 0 : 5;
        if (candidate_ok(m, s, p, guard)) return guard;
    }
    const int share = static_cast<int>((close ? 55.0 : 15.0) + 30.0 * aggression);
    if (ch.candidate_count > kUniversalCount && below(draw(prefix, counter * 64u + draw_index++), 100) < share) {
        for (int k = 0; k < 24; ++k) {
            const int c = kUniversalCount + below(draw(prefix, counter * 64u + draw_index++), ch.candidate_count - kUniversalCount);
            if (candidate_ok(m, s, p, c)) return c;
        }
    }
    for (int k = 0; k < 24; ++k) {
        const int c = below(draw(prefix, counter * 64u + draw_index++), kUniversalCount);
        if (candidate_ok(m, s, p, c)) return c;
    }
    return 0;
}
int main() {
    uint64_t state = 0x9a3c5e7f11ull;
    const auto next = [&](uint64_t bound) { state = mix64(state); return state % bound; };
    Cfg cfg;
    std::memset(&cfg, 0, sizeof cfg);
    cfg.dash_frames = 12; cfg.backdash_frames = 15; cfg.sidestep_frames = 10; cfg.heat_dash_frames = 9;
    cfg.knockdown_frames = 20; cfg.tech_window_frames = 8;
    std::vector<DMove> moves(16);
    for (size_t i = 0; i < moves.size(); ++i) {
        std::memset(&moves[i], 0, sizeof(DMove));
        moves[i].total_frames = 5 + static_cast<int>(next(40));
        moves[i].flags = (next(2) ? kHasHeatDashBlock : 0ull) | (next(2) ? kHasHeatDashHit : 0ull);
    }
    std::vector<DGate> gates(40);
    for (auto& g : gates) {
        std::memset(&g, 0, sizeof g);
        g.flags = next(1ull << 20) & next(1ull << 20);  // sparse requirement flags
        g.required_stance = static_cast<int>(next(3)) - 1;
        g.required_posture = static_cast<uint8_t>(next(2));
        g.heat_cost = static_cast<uint8_t>(next(4) == 0);
        g.move = static_cast<int16_t>(next(8) == 0 ? -1 : static_cast<int>(next(moves.size())));
    }
    cfg.back_to_wall_distance = 1.0; cfg.side_exposure_ratio = 0.3;
    DCharacter ch;
    std::memset(&ch, 0, sizeof ch);
    ch.moves = moves.data();
    ch.gates = gates.data();
    ch.move_count = static_cast<int>(moves.size());
    ch.candidate_count = 40;
    ch.move_candidate_inverse = 1.0 / (ch.candidate_count - kUniversalCount);
    const Match m{{&ch, &ch}, &cfg};
    unsigned long long checked = 0, bad = 0;
    for (int i = 0; i < 2000000; ++i) {
        Fight s;
        std::memset(&s, 0, sizeof s);
        s.winner = next(8) == 0 ? static_cast<int>(next(3)) : -1;
        for (int p = 0; p < 2; ++p) {
            Fighter& f = s.f[p];
            f.posture = static_cast<uint8_t>(next(6));
            f.universal = static_cast<uint8_t>(next(20));
            f.dash_from = static_cast<int8_t>(static_cast<int>(next(4)) - 1);
            f.flags = static_cast<uint32_t>(next(1u << 19));
            f.stun = next(3) == 0 ? static_cast<int>(next(5)) : 0;
            f.break_frames = next(3) == 0 ? static_cast<int>(next(4)) : 0;
            f.pending_throw_hit = next(4) == 0 ? static_cast<int>(next(3)) : -1;
            f.move = next(2) ? static_cast<int>(next(moves.size())) : -1;
            f.action_frame = static_cast<int>(next(50));
            f.grounded_elapsed = static_cast<int>(next(30));
            f.stance = static_cast<int>(next(3)) - 1;
            f.x = static_cast<double>(next(1000)) / 100.0 - 5.0;
            f.axis = static_cast<double>(next(1000)) / 100.0 - 5.0;
        }
        s.left_wall = -6.0;
        s.right_wall = 6.0;
        for (int p = 0; p < 2; ++p) {
            const uint32_t mask = universal_mask(m, s, p, can_act(m, s, p));
            for (int c = 0; c < kUniversalCount; ++c) {
                bad += (((mask >> c) & 1u) != 0u) != candidate_ok(m, s, p, c);
                ++checked;
            }
            const double aggression = static_cast<double>(next(1000)) / 999.0;
            const uint64_t prefix = mix64(state), counter = next(1u << 20);
            bad += random_opponent(m, s, p, aggression, prefix, counter) !=
                random_opponent_one_by_one(m, s, p, aggression, prefix, counter);
            ++checked;
            const Legality legal(m, s, p);
            for (int c = -1; c <= ch.candidate_count; ++c) {
                bad += legal(c) != candidate_ok(m, s, p, c);
                // no move candidate passes where moves_possible says none can
                bad += c >= kUniversalCount && !legal.moves_possible && candidate_ok(m, s, p, c);
                ++checked;
            }
        }
    }
    std::printf("%llu %llu\n", checked, bad);
    return bad == 0 ? 0 : 1;
}
"""


def test_universal_mask_equals_candidate_ok(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).exists():
        pytest.skip("nvcc is not available")
    src = tmp_path / "mask_check.cu"
    src.write_text(PROGRAM)
    exe = tmp_path / "mask_check"
    subprocess.run([nvcc, "-O2", "-std=c++17", f"-I{CSRC}", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)],
                   check=True, capture_output=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    checked, bad = (int(v) for v in out.stdout.split())
    assert checked == 2_000_000 * 2 * (22 + 1 + 42) and bad == 0 and out.returncode == 0
