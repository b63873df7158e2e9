"""TEST INFRASTRUCTURE: a Python mirror of the reference engine's State, its
test builders and its Action constructors, so the reference's own
known-answer tests (engine/tests/scenarios.rs, rebel_pbs.rs, ...) can be
restated here line by line against the product library.

The state crosses the C ABI in the reference's own write_state encoding
(engine/src/roots.rs:150-180); this module writes and reads that encoding
itself, independently of the library's C++ encoder, so a round trip through
the library also checks the encoder. Legal actions and apply run in the
product library (wc_state_legal_actions / wc_state_apply).

Field names and constants follow engine/src/state.rs, units.rs, actions.rs
and board.rs.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np

import warchest_b200 as wc

N_HEXES, N_UNITS, N_ZONES, N_PLAYERS = 37, 20, 7, 2
NONE = 255
WHITE, BLACK = 0, 1
Z_BAG, Z_HAND, Z_FACEUP, Z_FACEDOWN, Z_SUPPLY, Z_ELIM, Z_INFLIGHT = range(7)
CONT_CAP = 16

# unit indices (engine/src/units.rs:5-60)
(ARCHER, BERSERKER, CAVALRY, CROSSBOWMAN, ENSIGN, FOOTMAN, KNIGHT, LANCER, LIGHT_CAVALRY, MARSHAL, MERCENARY,
 PIKEMAN, SCOUT, SWORDSMAN, WARRIOR_PRIEST, ROYAL_GUARD, BERSERKER_V2, FOOTMAN_V2, WARRIOR_PRIEST_V2,
 ROYAL_COIN) = range(20)

# Cont tags (engine/src/roots.rs:49-104, the order of state.rs:121-164)
CONT_NAMES = ["Draw", "MainPlay", "RoyalGuardChoice", "SwordsmanMove", "BerserkerChain", "FootmanManeuver",
              "CavalryAttack", "MercenaryManeuver", "FootmanInstantDeploy", "WarriorPriestDraw",
              "WarriorPriestPlay", "_AttackPost"]
CONT_FIELDS = {"Draw": ["player"], "MainPlay": [], "RoyalGuardChoice": ["defender", "rg_hex"],
               "SwordsmanMove": ["hex"], "BerserkerChain": ["hex", "v2"], "FootmanManeuver": ["hexes"],
               "CavalryAttack": ["hex"], "MercenaryManeuver": ["hex"], "FootmanInstantDeploy": ["coin"],
               "WarriorPriestDraw": ["player", "rg_hex"], "WarriorPriestPlay": ["player"],
               "_AttackPost": ["atk_hex"]}


@dataclass
class Cont:
    """state.rs Cont: `kind` is the variant name, `f` its fields. For
    FootmanManeuver, f["hexes"] is the HexSet bit mask."""
    kind: str
    f: dict = field(default_factory=dict)

    def __getattr__(self, k):
        try:
            return self.__dict__["f"][k]
        except KeyError:
            raise AttributeError(k)

    def hexes_list(self) -> List[int]:
        """HexSet::to_vec: the hexes in ascending order."""
        m = self.f["hexes"]
        return [h for h in range(64) if m >> h & 1]


def main_play() -> Cont:
    return Cont("MainPlay")


class State:
    """engine/src/state.rs State, with the test builders of state.rs:495-560."""

    def __init__(self):
        self.hex_type = np.full(N_HEXES, NONE, np.uint8)
        self.hex_owner = np.full(N_HEXES, NONE, np.uint8)
        self.hex_height = np.zeros(N_HEXES, np.uint8)
        self.loc_marker = np.full(N_HEXES, NONE, np.uint8)
        self.zones = np.zeros((N_PLAYERS, N_ZONES, N_UNITS), np.uint8)
        self.markers_hand = np.zeros(N_PLAYERS, np.uint8)
        self.initiative = 0
        self.initiative_moved = False
        self.round = 1
        self.first_player = 0
        self.active = 0
        self.turns_taken = np.zeros(N_PLAYERS, np.uint8)
        self.main_plays = 0
        self.winner_ = NONE
        self.adjudicated_draw = False
        self.pending_ = main_play()
        self.conts: List[Cont] = []  # bottom of the stack first
        self.wp_v2_triggered = False
        self.interrupt = False

    # ---- test builders (state.rs:495-560)
    @staticmethod
    def blank(active: int) -> "State":
        s = State()
        s.initiative = active
        s.first_player = active
        s.active = active
        return s

    def set_unit(self, hex_, owner, unit, height):
        self.hex_type[hex_] = unit
        self.hex_owner[hex_] = owner
        self.hex_height[hex_] = height

    def set_marker(self, hex_, owner):
        self.loc_marker[hex_] = owner

    def add_zone(self, p, zone, unit, n):
        self.zones[p, zone, unit] += n

    def set_markers_hand(self, p, n):
        self.markers_hand[p] = n

    def set_initiative(self, holder, moved):
        self.initiative = holder
        self.initiative_moved = moved

    def pending(self) -> Cont:
        return self.pending_

    # ---- the write_state encoding (roots.rs:150-180)
    @staticmethod
    def _write_cont(out: bytearray, c: Cont):
        tag = CONT_NAMES.index(c.kind)
        out.append(tag)
        for name in CONT_FIELDS[c.kind]:
            v = c.f[name]
            if name == "hexes":
                out += struct.pack("<Q", v)
            else:
                out.append(int(bool(v)) if name == "v2" else int(v))

    @staticmethod
    def _read_cont(b: bytes, at: int):
        kind = CONT_NAMES[b[at]]
        at += 1
        f = {}
        for name in CONT_FIELDS[kind]:
            if name == "hexes":
                f[name] = struct.unpack_from("<Q", b, at)[0]
                at += 8
            else:
                f[name] = bool(b[at]) if name == "v2" else b[at]
                at += 1
        return Cont(kind, f), at

    def to_bytes(self) -> bytes:
        out = bytearray()
        for h in range(N_HEXES):
            out += bytes([self.hex_type[h], self.hex_owner[h], self.hex_height[h], self.loc_marker[h]])
        out += self.zones.astype(np.uint8).tobytes()
        out += bytes([self.markers_hand[0], self.markers_hand[1], self.initiative, int(self.initiative_moved)])
        out += struct.pack("<I", self.round)
        out += bytes([self.first_player, self.active, self.turns_taken[0], self.turns_taken[1]])
        out += struct.pack("<I", self.main_plays)
        out += bytes([self.winner_, int(self.adjudicated_draw)])
        State._write_cont(out, self.pending_)
        out.append(len(self.conts))
        for c in reversed(self.conts):  # pop order: the top first
            State._write_cont(out, c)
        out += bytes([int(self.wp_v2_triggered), int(self.interrupt)])
        return bytes(out)

    @staticmethod
    def from_bytes(b: bytes) -> "State":
        s, at = State.parse(b)
        assert at == len(b), "trailing bytes after the state"
        return s

    @staticmethod
    def parse(b: bytes, at: int = 0):
        """read_state (roots.rs:182-230) from offset `at`: (state, end offset)."""
        s = State()
        for h in range(N_HEXES):
            s.hex_type[h], s.hex_owner[h], s.hex_height[h], s.loc_marker[h] = b[at: at + 4]
            at += 4
        n = N_PLAYERS * N_ZONES * N_UNITS
        s.zones = np.frombuffer(b[at: at + n], np.uint8).reshape(N_PLAYERS, N_ZONES, N_UNITS).copy()
        at += n
        s.markers_hand = np.array([b[at], b[at + 1]], np.uint8)
        s.initiative, s.initiative_moved = b[at + 2], bool(b[at + 3])
        at += 4
        s.round = struct.unpack_from("<I", b, at)[0]
        at += 4
        s.first_player, s.active = b[at], b[at + 1]
        s.turns_taken = np.array([b[at + 2], b[at + 3]], np.uint8)
        at += 4
        s.main_plays = struct.unpack_from("<I", b, at)[0]
        at += 4
        s.winner_, s.adjudicated_draw = b[at], bool(b[at + 1])
        at += 2
        s.pending_, at = State._read_cont(b, at)
        k = b[at]
        at += 1
        items = []
        for _ in range(k):
            c, at = State._read_cont(b, at)
            items.append(c)
        s.conts = list(reversed(items))
        s.wp_v2_triggered, s.interrupt = bool(b[at]), bool(b[at + 1])
        at += 2
        return s, at

    # ---- the engine, through the product library
    def legal_actions(self) -> List[int]:
        return wc.legal_actions(self.to_bytes())

    def apply(self, code: int) -> "State":
        """Like the reference's State::apply, no legality test (the reference
        tests apply hand-picked actions)."""
        return State.from_bytes(wc.apply_action(self.to_bytes(), code, unchecked=True))

    def apply_checked(self, code: int) -> "State":
        return State.from_bytes(wc.apply_action(self.to_bytes(), code))

    def to_act(self) -> int:
        return wc.state_query(self.to_bytes())["to_act"]

    def winner(self) -> Optional[int]:
        return wc.state_query(self.to_bytes())["winner"]

    def is_terminal(self) -> bool:
        return wc.state_query(self.to_bytes())["terminal"]


# ------------------------------------------------------------------ roots
# write_root (roots.rs:247-262): the state, then per player u32 n, n configs
# (hand[5], fd[5], inflight or 0xff) and n f32 weights.

def encode_root(state: "State", beliefs) -> bytes:
    """beliefs: per player a list of ((hand5, fd5, inflight or None), weight)."""
    out = bytearray(state.to_bytes())
    for bel in beliefs:
        out += struct.pack("<I", len(bel))
        for (hand, fd, inflight), _ in bel:
            out += bytes(hand) + bytes(fd) + bytes([0xFF if inflight is None else inflight])
        for _, w in bel:
            out += struct.pack("<f", w)
    return bytes(out)


def decode_root(b: bytes):
    """read_root (roots.rs:265-284): (state, beliefs) as encode_root takes them."""
    s, at = State.parse(b)
    beliefs = []
    for _ in range(2):
        (n,) = struct.unpack_from("<I", b, at)
        at += 4
        cfgs = []
        for _ in range(n):
            hand, fd, inf = tuple(b[at: at + 5]), tuple(b[at + 5: at + 10]), b[at + 10]
            cfgs.append((hand, fd, None if inf == 0xFF else inf))
            at += 11
        ws = struct.unpack_from(f"<{n}f", b, at)
        at += 4 * n
        beliefs.append(list(zip(cfgs, ws)))
    assert at == len(b), "trailing bytes after the root"
    return s, beliefs


# --------------------------------------------------------------- actions
# Action::encode (actions.rs:252-295): kind | a << 6 | b << 12 | c << 18 with
# the variant's fields in declaration order, NONE as 63, absent fields 0.

KINDS = ["Deploy", "Bolster", "ClaimInitiative", "Recruit", "Pass", "Move", "Control", "Attack", "TacArcher",
         "TacCavalryMove", "TacCavalryAttack", "TacCrossbow", "TacEnsign", "TacLancer", "TacLightCav",
         "TacMarshal", "TacRoyalGuard", "FootMove", "FootControl", "FootAttack", "DrawCoin", "RGSoakSupply",
         "RGSoakStack", "SwordsmanMove", "SwordsmanDecline", "BerserkMove", "BerserkControl", "BerserkAttack",
         "BerserkStop", "MercMove", "MercControl", "MercAttack", "MercDecline", "FootmanInstantDeploy",
         "FootmanInstantDecline", "GrantMove", "GrantAttack", "GrantControl", "TacFootman"]
KIND = {n: i for i, n in enumerate(KINDS)}
NFIELDS = {"Deploy": 2, "Bolster": 2, "ClaimInitiative": 1, "Recruit": 2, "Pass": 1, "Move": 2, "Control": 1,
           "Attack": 2, "TacArcher": 2, "TacCavalryMove": 2, "TacCavalryAttack": 2, "TacCrossbow": 2,
           "TacEnsign": 2, "TacLancer": 3, "TacLightCav": 2, "TacMarshal": 2, "TacRoyalGuard": 2, "FootMove": 2,
           "FootControl": 1, "FootAttack": 2, "DrawCoin": 1, "RGSoakSupply": 0, "RGSoakStack": 0,
           "SwordsmanMove": 2, "SwordsmanDecline": 0, "BerserkMove": 2, "BerserkControl": 1, "BerserkAttack": 2,
           "BerserkStop": 0, "MercMove": 2, "MercControl": 1, "MercAttack": 2, "MercDecline": 0,
           "FootmanInstantDeploy": 1, "FootmanInstantDecline": 0, "GrantMove": 2, "GrantAttack": 2,
           "GrantControl": 1, "TacFootman": 1}


def encode(kind: str, *fields: int) -> int:
    assert len(fields) == NFIELDS[kind], kind
    code = KIND[kind]
    for i, v in enumerate(fields):
        code |= (63 if v == NONE else int(v)) << (6 + 6 * i)
    return code


def decode(code: int):
    """(kind name, fields) of an action code (Action::decode, actions.rs:297)."""
    kind = KINDS[code & 63]
    vals = [(code >> (6 + 6 * i)) & 63 for i in range(NFIELDS[kind])]
    return kind, tuple(NONE if v == 63 else v for v in vals)


class _Actions:
    """A.Attack(frm, target) -> the action's code, for every variant."""

    def __getattr__(self, kind):
        if kind not in KIND:
            raise AttributeError(kind)
        return lambda *f: encode(kind, *f)


A = _Actions()


def has(acts: List[int], code: int) -> bool:
    return code in acts


def count_kind(acts: List[int], kind: str, pred=None) -> int:
    n = 0
    for c in acts:
        k, f = decode(c)
        if k == kind and (pred is None or pred(*f)):
            n += 1
    return n
