"""Roster files: every fighter's compiled tables in the boundary layout of include/t8b.h.

A roster file is what the reference's loader (src/full_move_roster.cpp:51,
load_full_move_character) produces from data/generated, written once so that no CSV and
no reference code is needed where the hot path runs. Layout, little-endian:
  b"T8BRST01", u32 count, u32 0, t8b_engine_config_t,
  per character: i32 roster_id, move_count, hit_count, stance_count, candidate_count, 0;
  char slug[32]; t8b_rules_t; t8b_move_t[move_count]; t8b_hit_t[hit_count];
  t8b_stance_t[stance_count]; i32 candidate_moves[candidate_count];
  f32 candidate_features[candidate_count * 32].
"""
from __future__ import annotations

import ctypes as C
import lzma
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from ._lib import Character, EngineConfig, Hit, Move, Rules, Stance, FEATURE_SIZE, MAX_CANDIDATES


@dataclass
class RosterCharacter:
    slug: str
    roster_id: int
    moves: C.Array
    hits: C.Array
    stances: C.Array
    rules: Rules
    candidate_moves: np.ndarray  # int32 [candidates]
    candidate_features: np.ndarray  # float32 [candidates, 32]

    @property
    def candidate_count(self) -> int:
        return int(self.candidate_moves.shape[0])


@dataclass
class Roster:
    config: EngineConfig
    characters: list = field(default_factory=list)
    raw: bytes = b""

    def __len__(self) -> int:
        return len(self.characters)

    def c_array(self, indices=None):
        """t8b_character_t[] for t8b_sim_create; keeps the arrays alive on the returned object."""
        chars = self.characters if indices is None else [self.characters[i] for i in indices]
        array = (Character * len(chars))()
        for out, ch in zip(array, chars):
            out.moves = C.cast(ch.moves, C.POINTER(Move))
            out.hits = C.cast(ch.hits, C.POINTER(Hit))
            out.stances = C.cast(ch.stances, C.POINTER(Stance))
            out.candidate_moves = ch.candidate_moves.ctypes.data_as(C.POINTER(C.c_int32))
            out.candidate_features = ch.candidate_features.ctypes.data_as(C.POINTER(C.c_float))
            out.move_count = len(ch.moves)
            out.hit_count = len(ch.hits)
            out.stance_count = len(ch.stances)
            out.candidate_count = ch.candidate_count
            out.roster_id = ch.roster_id
            out.rules = ch.rules
        array._keepalive = chars
        return array

    def feature_tables(self, stride: int = MAX_CANDIDATES) -> np.ndarray:
        """[characters, stride, 32] float32, zero past each character's candidates
        (src/full_move_train.cpp:1176-1184)."""
        out = np.zeros((len(self.characters), stride, FEATURE_SIZE), np.float32)
        for index, ch in enumerate(self.characters):
            out[index, : ch.candidate_count] = ch.candidate_features
        return out


def parse(data: bytes) -> Roster:
    if data[:8] != b"T8BRST01":
        raise ValueError("not a roster file")
    count, _ = struct.unpack_from("<II", data, 8)
    offset = 16
    config = EngineConfig.from_buffer_copy(data, offset)
    offset += C.sizeof(EngineConfig)
    roster = Roster(config=config, raw=data)
    for _ in range(count):
        roster_id, moves, hits, stances, candidates, _pad = struct.unpack_from("<6i", data, offset)
        offset += 24
        slug = data[offset: offset + 32].split(b"\0")[0].decode()
        offset += 32
        rules = Rules.from_buffer_copy(data, offset)
        offset += C.sizeof(Rules)
        move_array = (Move * moves).from_buffer_copy(data, offset)
        offset += C.sizeof(Move) * moves
        hit_array = (Hit * hits).from_buffer_copy(data, offset)
        offset += C.sizeof(Hit) * hits
        stance_array = (Stance * max(stances, 0)).from_buffer_copy(data, offset) if stances else (Stance * 0)()
        offset += C.sizeof(Stance) * stances
        candidate_moves = np.frombuffer(data, np.int32, candidates, offset).copy()
        offset += 4 * candidates
        features = np.frombuffer(data, np.float32, candidates * FEATURE_SIZE, offset).reshape(candidates, FEATURE_SIZE).copy()
        offset += 4 * candidates * FEATURE_SIZE
        roster.characters.append(RosterCharacter(slug, roster_id, move_array, hit_array, stance_array, rules,
                                                 candidate_moves, features))
    if offset != len(data):
        raise ValueError("trailing bytes in roster file")
    return roster


def load(path) -> Roster:
    path = Path(path)
    data = path.read_bytes()
    if path.suffix == ".xz":
        data = lzma.decompress(data)
    return parse(data)
