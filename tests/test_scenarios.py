"""The reference's rules known-answer tests, restated: engine/tests/scenarios.rs
(38 hand-built positions with the exact legal and illegal actions and the
post-states the reference asserts). Each test names the reference test it
restates, with its line. The positions are built with the reference's own
test builders (State::blank / set_unit / add_zone / set_marker, mirrored in
tests/wc_state.py); legal actions and apply run in the product library
through the C ABI. These pin the rules engine that indexes every subgame
tree to the reference's expectations, independently of the oracle (which
compiles the same host sources).
"""
import pytest

from wc_state import (A, ARCHER, BERSERKER, BERSERKER_V2, BLACK, CAVALRY, CROSSBOWMAN, ENSIGN, FOOTMAN, FOOTMAN_V2,
                      KNIGHT, LANCER, LIGHT_CAVALRY, MARSHAL, MERCENARY, NONE, PIKEMAN, ROYAL_COIN, ROYAL_GUARD,
                      SCOUT, SWORDSMAN, WARRIOR_PRIEST, WARRIOR_PRIEST_V2, WHITE, Z_BAG, Z_ELIM, Z_FACEDOWN,
                      Z_FACEUP, Z_HAND, Z_INFLIGHT, Z_SUPPLY, State, count_kind, decode, encode, has)

# geometry cheatsheet (scenarios.rs:9-20)
CENTER, E1, E2, E3, W1 = 18, 19, 20, 21, 17
LOC_53, LOC_11, LOC_25 = 20, 11, 25


def one_unit(unit, hex_):
    """scenarios.rs:33-38: WHITE with one hand coin of `unit` and one unit at `hex_`."""
    s = State.blank(WHITE)
    s.set_unit(hex_, WHITE, unit, 1)
    s.add_zone(WHITE, Z_HAND, unit, 1)
    return s


def test_encoding_round_trips_through_the_library():
    """The Python mirror's write_state bytes and the library's agree: a state
    that goes out and comes back through apply keeps every untouched field."""
    s = one_unit(KNIGHT, CENTER)
    s.set_marker(LOC_11, BLACK)
    s2 = s.apply(A.Move(CENTER, W1))
    assert s2.hex_type[W1] == KNIGHT and s2.hex_type[CENTER] == NONE
    assert s2.loc_marker[LOC_11] == BLACK


# ---------------------------------------------------------------- ARCHER

def test_archer_cannot_normal_attack_but_tactic_hits_at_two():  # scenarios.rs:42
    s = one_unit(ARCHER, CENTER)
    s.set_unit(E1, BLACK, KNIGHT, 1)
    s.set_unit(E2, BLACK, SWORDSMAN, 1)
    acts = s.legal_actions()
    assert count_kind(acts, "Attack") == 0, "Archer must not offer a normal Attack"
    assert has(acts, A.TacArcher(CENTER, E2))
    assert not has(acts, A.TacArcher(CENTER, E1))


# ----------------------------------------------------------- CROSSBOWMAN

def test_crossbowman_straight_line_blocked_by_intervening_unit():  # scenarios.rs:75
    s = one_unit(CROSSBOWMAN, W1)
    s.set_unit(E1, BLACK, SWORDSMAN, 1)
    assert has(s.legal_actions(), A.TacCrossbow(W1, E1))
    s.set_unit(CENTER, BLACK, FOOTMAN, 1)
    acts = s.legal_actions()
    assert not has(acts, A.TacCrossbow(W1, E1)), "Crossbowman line must be blocked by an intervening unit"
    assert has(acts, A.Attack(W1, CENTER))


# -------------------------------------------------------- KNIGHT immunity

def test_knight_immune_to_unbolstered_and_hit_by_bolstered():  # scenarios.rs:118
    s = one_unit(SWORDSMAN, CENTER)
    s.set_unit(E1, BLACK, KNIGHT, 1)
    assert not has(s.legal_actions(), A.Attack(CENTER, E1))
    s.set_unit(CENTER, WHITE, SWORDSMAN, 2)
    assert has(s.legal_actions(), A.Attack(CENTER, E1))


def test_knight_immunity_applies_to_tactic_attacks():  # scenarios.rs:143
    s = one_unit(ARCHER, CENTER)
    s.set_unit(E2, BLACK, KNIGHT, 1)
    assert not has(s.legal_actions(), A.TacArcher(CENTER, E2))
    s.set_unit(CENTER, WHITE, ARCHER, 2)
    assert has(s.legal_actions(), A.TacArcher(CENTER, E2))


# ---------------------------------------------------------- PIKEMAN reflex

def test_pikeman_reflex_mutual_death_and_ignores_knight():  # scenarios.rs:169
    s = one_unit(SWORDSMAN, CENTER)
    s.set_unit(E1, BLACK, PIKEMAN, 1)
    s2 = s.apply(A.Attack(CENTER, E1))
    assert s2.hex_type[CENTER] == NONE, "attacker should die to reflex"
    assert s2.hex_type[E1] == NONE, "pikeman should die to the attack"
    assert s2.zones[WHITE][Z_ELIM][SWORDSMAN] == 1
    assert s2.zones[WHITE][Z_FACEUP][SWORDSMAN] == 1
    assert s2.zones[BLACK][Z_ELIM][PIKEMAN] == 1


# ------------------------------------------------------------ ROYAL GUARD

def test_royal_guard_defender_supply_choice():  # scenarios.rs:195
    s = one_unit(SWORDSMAN, CENTER)
    s.set_unit(E1, BLACK, ROYAL_GUARD, 1)
    s.add_zone(BLACK, Z_SUPPLY, ROYAL_GUARD, 1)
    s2 = s.apply(A.Attack(CENTER, E1))
    assert s2.to_act() == BLACK, "defender chooses RG soak"
    choices = s2.legal_actions()
    assert has(choices, A.RGSoakSupply())
    assert has(choices, A.RGSoakStack())
    s3 = s2.apply(A.RGSoakSupply())
    assert s3.hex_type[E1] == ROYAL_GUARD, "RG survives when soaked from supply"
    assert s3.zones[BLACK][Z_SUPPLY][ROYAL_GUARD] == 0
    assert s3.zones[BLACK][Z_ELIM][ROYAL_GUARD] == 1
    s3b = s2.apply(A.RGSoakStack())
    assert s3b.hex_type[E1] == NONE, "RG dies when soaked from stack"
    assert s3b.zones[BLACK][Z_SUPPLY][ROYAL_GUARD] == 1


def test_royal_guard_tactic_needs_royal_coin_and_ends_on_controlled_location():  # scenarios.rs:229
    s = one_unit(ROYAL_GUARD, CENTER)
    s.add_zone(WHITE, Z_HAND, ROYAL_COIN, 1)
    s.set_marker(LOC_53, WHITE)
    assert has(s.legal_actions(), A.TacRoyalGuard(CENTER, LOC_53))
    s2 = one_unit(ROYAL_GUARD, CENTER)
    s2.set_marker(LOC_53, WHITE)
    assert count_kind(s2.legal_actions(), "TacRoyalGuard") == 0
    s3 = one_unit(ROYAL_GUARD, CENTER)
    s3.add_zone(WHITE, Z_HAND, ROYAL_COIN, 1)
    assert count_kind(s3.legal_actions(), "TacRoyalGuard") == 0


# ------------------------------------------------------------------ SCOUT

def test_scout_deploy_adjacent_to_friendly():  # scenarios.rs:264
    s = State.blank(WHITE)
    s.set_unit(CENTER, WHITE, KNIGHT, 1)
    s.add_zone(WHITE, Z_HAND, SCOUT, 1)
    acts = s.legal_actions()
    assert has(acts, A.Deploy(SCOUT, E1))
    assert not has(acts, A.Deploy(SCOUT, E3))


# -------------------------------------------------------------- SWORDSMAN

def test_swordsman_optional_move_after_attack():  # scenarios.rs:291
    s = one_unit(SWORDSMAN, CENTER)
    s.set_unit(E1, BLACK, FOOTMAN, 2)
    s2 = s.apply(A.Attack(CENTER, E1))
    p = s2.pending()
    assert p.kind == "SwordsmanMove", f"expected SwordsmanMove pending, got {p}"
    assert p.hex == CENTER
    acts = s2.legal_actions()
    assert has(acts, A.SwordsmanDecline())
    assert has(acts, A.SwordsmanMove(CENTER, W1))


# -------------------------------------------------------------- BERSERKER

def test_berserker_v1_chain_via_any_maneuver_coin_to_faceup():  # scenarios.rs:317
    s = one_unit(BERSERKER, CENTER)
    s.set_unit(CENTER, WHITE, BERSERKER, 3)
    s2 = s.apply(A.Move(CENTER, W1))
    p = s2.pending()
    assert p.kind == "BerserkerChain", f"expected BerserkerChain, got {p}"
    assert p.hex == W1 and not p.v2
    assert has(s2.legal_actions(), A.BerserkStop())
    s3 = s2.apply(A.BerserkMove(W1, CENTER))
    assert s3.zones[WHITE][Z_FACEUP][BERSERKER] == 2, "chain coin recycles face-up, not eliminated"
    assert s3.zones[WHITE][Z_ELIM][BERSERKER] == 0, "chain coin is NOT eliminated"
    assert s3.hex_height[CENTER] == 2


def test_berserker_cannot_remove_final_coin():  # scenarios.rs:357
    s = one_unit(BERSERKER, CENTER)
    s2 = s.apply(A.Move(CENTER, W1))
    assert s2.pending().kind != "BerserkerChain"


def test_berserker_v2_only_attack_or_move_no_control():  # scenarios.rs:369
    s = State.blank(WHITE)
    s.set_unit(LOC_11, WHITE, BERSERKER_V2, 2)
    s.add_zone(WHITE, Z_HAND, BERSERKER_V2, 1)
    s.set_markers_hand(WHITE, 4)
    s2 = s.apply(A.Control(LOC_11))
    assert s2.pending().kind != "BerserkerChain", "V2 must not chain after control"
    s3 = State.blank(WHITE)
    s3.set_unit(CENTER, WHITE, BERSERKER_V2, 2)
    s3.add_zone(WHITE, Z_HAND, BERSERKER_V2, 1)
    s3.set_marker(LOC_25, BLACK)
    s4 = s3.apply(A.Move(CENTER, LOC_25))
    p = s4.pending()
    assert p.kind == "BerserkerChain" and p.v2, f"expected V2 chain, got {p}"
    assert count_kind(s4.legal_actions(), "BerserkControl") == 0, "V2 chain excludes control"


# ----------------------------------------------------------------- LANCER

def test_lancer_must_attack_and_knight_immunity_in_line():  # scenarios.rs:404
    s = one_unit(LANCER, W1)
    s.set_unit(E1, BLACK, SWORDSMAN, 1)
    acts = s.legal_actions()
    assert has(acts, A.TacLancer(W1, CENTER, E1))
    assert count_kind(acts, "Attack") == 0
    s2 = one_unit(LANCER, W1)
    s2.set_unit(E1, BLACK, KNIGHT, 1)
    assert count_kind(s2.legal_actions(), "TacLancer") == 0, "unbolstered Lancer cannot attack the Knight"
    s2.set_unit(W1, WHITE, LANCER, 2)
    assert has(s2.legal_actions(), A.TacLancer(W1, CENTER, E1))


# ---------------------------------------------------------------- CAVALRY

def test_cavalry_move_then_attack():  # scenarios.rs:444
    s = one_unit(CAVALRY, W1)
    s.set_unit(E1, BLACK, FOOTMAN, 2)
    assert has(s.legal_actions(), A.TacCavalryMove(W1, CENTER))
    s2 = s.apply(A.TacCavalryMove(W1, CENTER))
    p = s2.pending()
    assert p.kind == "CavalryAttack" and p.hex == CENTER, f"expected CavalryAttack, got {p}"
    assert has(s2.legal_actions(), A.TacCavalryAttack(CENTER, E1))


# ---------------------------------------------------------- LIGHT CAVALRY

def test_light_cavalry_moves_exactly_two_through_empty():  # scenarios.rs:479
    s = one_unit(LIGHT_CAVALRY, W1)
    assert has(s.legal_actions(), A.TacLightCav(W1, E1))
    s.set_unit(CENTER, BLACK, FOOTMAN, 1)
    assert not has(s.legal_actions(), A.TacLightCav(W1, E1))


# ------------------------------------------------------- ENSIGN / MARSHAL

def test_ensign_moves_friendly_within_two():  # scenarios.rs:506
    s = State.blank(WHITE)
    s.set_unit(CENTER, WHITE, ENSIGN, 1)
    s.add_zone(WHITE, Z_HAND, ENSIGN, 1)
    s.set_unit(W1, WHITE, FOOTMAN, 1)
    assert count_kind(s.legal_actions(), "TacEnsign", lambda frm, to: frm == W1) > 0


def test_marshal_grants_normal_attack_not_archer():  # scenarios.rs:522
    NB = 24
    s = State.blank(WHITE)
    s.set_unit(CENTER, WHITE, MARSHAL, 1)
    s.add_zone(WHITE, Z_HAND, MARSHAL, 1)
    s.set_unit(W1, WHITE, ARCHER, 1)
    s.set_unit(NB, BLACK, FOOTMAN, 1)
    assert count_kind(s.legal_actions(), "TacMarshal", lambda uh, t: uh == W1) == 0, \
        "Marshal must not grant an attack to an Archer"
    s2 = State.blank(WHITE)
    s2.set_unit(CENTER, WHITE, MARSHAL, 1)
    s2.add_zone(WHITE, Z_HAND, MARSHAL, 1)
    s2.set_unit(W1, WHITE, SWORDSMAN, 1)
    s2.set_unit(NB, BLACK, FOOTMAN, 1)
    assert has(s2.legal_actions(), A.TacMarshal(W1, NB)), "Marshal should grant the Swordsman a normal attack"


# ---------------------------------------------------------------- FOOTMAN

def test_footman_two_units_and_tactic_two_maneuvers():  # scenarios.rs:561
    s = State.blank(WHITE)
    s.set_unit(CENTER, WHITE, FOOTMAN, 1)
    s.set_unit(E1, BLACK, FOOTMAN, 1)
    s.set_unit(W1, WHITE, FOOTMAN, 1)
    s.add_zone(WHITE, Z_HAND, FOOTMAN, 1)
    assert has(s.legal_actions(), A.TacFootman(FOOTMAN))
    s2 = s.apply(A.TacFootman(FOOTMAN))
    assert s2.pending().kind == "FootmanManeuver"


def test_footman_deploy_two_allowed_others_capped_at_one():  # scenarios.rs:576
    s = State.blank(WHITE)
    s.set_unit(CENTER, WHITE, FOOTMAN, 1)
    s.set_marker(LOC_11, WHITE)
    s.set_marker(LOC_25, WHITE)
    s.add_zone(WHITE, Z_HAND, FOOTMAN, 1)
    assert count_kind(s.legal_actions(), "Deploy", lambda u, h: u == FOOTMAN) >= 1
    s2 = State.blank(WHITE)
    s2.set_unit(CENTER, WHITE, KNIGHT, 1)
    s2.set_marker(LOC_11, WHITE)
    s2.add_zone(WHITE, Z_HAND, KNIGHT, 1)
    assert count_kind(s2.legal_actions(), "Deploy", lambda u, h: u == KNIGHT) == 0


# -------------------------------------------------------------- MERCENARY

def test_mercenary_free_maneuver_only_when_deployed():  # scenarios.rs:599
    s = State.blank(WHITE)
    s.set_unit(CENTER, WHITE, MERCENARY, 1)
    s.add_zone(WHITE, Z_HAND, MERCENARY, 1)
    s.add_zone(WHITE, Z_SUPPLY, MERCENARY, 1)
    s2 = s.apply(A.Recruit(MERCENARY, MERCENARY))
    assert s2.pending().kind == "MercenaryManeuver"
    assert has(s2.legal_actions(), A.MercDecline())
    s3 = State.blank(WHITE)
    s3.add_zone(WHITE, Z_HAND, MERCENARY, 1)
    s3.add_zone(WHITE, Z_SUPPLY, MERCENARY, 1)
    s4 = s3.apply(A.Recruit(MERCENARY, MERCENARY))
    assert s4.pending().kind != "MercenaryManeuver"


# ------------------------------------------------ FOOTMAN V2 recruit-deploy

def test_footman_v2_recruit_instant_deploy():  # scenarios.rs:627
    s = State.blank(WHITE)
    s.set_unit(CENTER, WHITE, FOOTMAN_V2, 1)
    s.set_marker(LOC_11, WHITE)
    s.add_zone(WHITE, Z_HAND, FOOTMAN_V2, 1)
    s.add_zone(WHITE, Z_SUPPLY, FOOTMAN_V2, 1)
    s2 = s.apply(A.Recruit(FOOTMAN_V2, FOOTMAN_V2))
    assert s2.pending().kind == "FootmanInstantDeploy"
    acts = s2.legal_actions()
    assert has(acts, A.FootmanInstantDeploy(LOC_11))
    assert has(acts, A.FootmanInstantDecline())
    s3 = s2.apply(A.FootmanInstantDeploy(LOC_11))
    assert s3.hex_type[LOC_11] == FOOTMAN_V2


# --------------------------------------------------------- WARRIOR PRIEST

def test_warrior_priest_draws_and_forces_use():  # scenarios.rs:651
    s = State.blank(WHITE)
    s.set_unit(LOC_11, WHITE, WARRIOR_PRIEST, 1)
    s.add_zone(WHITE, Z_HAND, WARRIOR_PRIEST, 1)
    s.add_zone(WHITE, Z_BAG, ARCHER, 1)
    s.set_markers_hand(WHITE, 4)
    s2 = s.apply(A.Control(LOC_11))
    p = s2.pending()
    assert p.kind == "WarriorPriestDraw" and p.player == WHITE, f"expected WarriorPriestDraw, got {p}"
    assert has(s2.legal_actions(), A.DrawCoin(ARCHER))
    s3 = s2.apply(A.DrawCoin(ARCHER))
    assert s3.pending().kind == "WarriorPriestPlay"
    assert s3.zones[WHITE][Z_INFLIGHT][ARCHER] == 1
    assert has(s3.legal_actions(), A.Pass(ARCHER))


def test_warrior_priest_v2_once_per_turn():  # scenarios.rs:675
    s = State.blank(WHITE)
    s.set_unit(CENTER, WHITE, WARRIOR_PRIEST_V2, 1)
    s.add_zone(WHITE, Z_HAND, WARRIOR_PRIEST_V2, 1)
    s.set_unit(E1, BLACK, FOOTMAN, 3)
    s.add_zone(WHITE, Z_BAG, WARRIOR_PRIEST_V2, 1)
    s2 = s.apply(A.Attack(CENTER, E1))
    assert s2.pending().kind == "WarriorPriestDraw"
    s3 = s2.apply(A.DrawCoin(WARRIOR_PRIEST_V2))
    s4 = s3.apply(A.Attack(CENTER, E1))
    assert s4.pending().kind != "WarriorPriestDraw", "V2 caps at one trigger per turn"


def test_warrior_priest_v1_does_not_block_v2():  # scenarios.rs:703
    s = State.blank(WHITE)
    s.set_unit(LOC_11, WHITE, WARRIOR_PRIEST, 1)
    s.set_unit(CENTER, WHITE, WARRIOR_PRIEST_V2, 1)
    s.set_unit(E1, BLACK, FOOTMAN, 3)
    s.add_zone(WHITE, Z_HAND, WARRIOR_PRIEST, 1)
    s.add_zone(WHITE, Z_BAG, WARRIOR_PRIEST_V2, 1)
    s2 = s.apply(A.Attack(LOC_11, E1))
    assert s2.pending().kind == "WarriorPriestDraw"
    s3 = s2.apply(A.DrawCoin(WARRIOR_PRIEST_V2))
    s4 = s3.apply(A.Attack(CENTER, E1))
    assert s4.pending().kind == "WarriorPriestDraw", "V1's trigger must not block V2's"


def test_warrior_priest_forced_play_of_rg_coin_cannot_use_rg_tactic():  # scenarios.rs:738
    s = State.blank(WHITE)
    s.set_unit(W1, WHITE, WARRIOR_PRIEST, 1)
    s.set_unit(CENTER, WHITE, ROYAL_GUARD, 1)
    s.set_marker(LOC_25, WHITE)
    s.set_unit(E1, BLACK, FOOTMAN, 3)
    s.add_zone(WHITE, Z_HAND, WARRIOR_PRIEST, 1)
    s.add_zone(WHITE, Z_HAND, ROYAL_COIN, 1)
    s.add_zone(WHITE, Z_BAG, ROYAL_GUARD, 1)
    s2 = s.apply(A.Attack(W1, E1))
    s3 = s2.apply(A.DrawCoin(ROYAL_GUARD))
    plays = s3.legal_actions()
    assert has(plays, A.Pass(ROYAL_GUARD))
    assert not has(plays, A.TacRoyalGuard(CENTER, LOC_25)), \
        "an RG-coin forced play must not offer the Royal-Guard tactic"
    t = State.blank(WHITE)
    t.set_unit(W1, WHITE, WARRIOR_PRIEST, 1)
    t.set_unit(CENTER, WHITE, ROYAL_GUARD, 1)
    t.set_marker(LOC_25, WHITE)
    t.set_unit(E1, BLACK, FOOTMAN, 3)
    t.add_zone(WHITE, Z_HAND, WARRIOR_PRIEST, 1)
    t.add_zone(WHITE, Z_BAG, ROYAL_COIN, 1)
    t2 = t.apply(A.Attack(W1, E1))
    t3 = t2.apply(A.DrawCoin(ROYAL_COIN))
    assert has(t3.legal_actions(), A.TacRoyalGuard(CENTER, LOC_25)), \
        "a Royal-Coin forced play offers the Royal-Guard tactic"


# ------------------------------------------------------------- INITIATIVE

def test_initiative_claim_rules():  # scenarios.rs:794
    s = State.blank(WHITE)
    s.add_zone(WHITE, Z_HAND, ARCHER, 1)
    s.set_initiative(BLACK, False)
    assert has(s.legal_actions(), A.ClaimInitiative(ARCHER))
    s.set_initiative(WHITE, False)
    assert count_kind(s.legal_actions(), "ClaimInitiative") == 0
    s.set_initiative(BLACK, True)
    assert count_kind(s.legal_actions(), "ClaimInitiative") == 0


# --------------------------------------------------------- CONTROL / WIN

def test_control_returns_opponent_marker_and_wins_at_six():  # scenarios.rs:819
    s = State.blank(WHITE)
    for h in (1, 4, 8, 11, 16):
        s.set_marker(h, WHITE)
    s.set_markers_hand(WHITE, 1)
    s.set_marker(LOC_25, BLACK)
    s.set_markers_hand(BLACK, 5)
    s.set_unit(LOC_25, WHITE, KNIGHT, 1)
    s.add_zone(WHITE, Z_HAND, KNIGHT, 1)
    assert has(s.legal_actions(), A.Control(LOC_25))
    s2 = s.apply(A.Control(LOC_25))
    assert s2.winner() == WHITE, "6th marker wins"
    assert s2.markers_hand[BLACK] == 6


def test_control_illegal_on_already_controlled_location():  # scenarios.rs:841
    s = State.blank(WHITE)
    s.set_marker(LOC_11, WHITE)
    s.set_unit(LOC_11, WHITE, KNIGHT, 1)
    s.add_zone(WHITE, Z_HAND, KNIGHT, 1)
    assert count_kind(s.legal_actions(), "Control") == 0


# ----------------------------------------------------------- DEPLOY rules

def test_deploy_only_on_empty_controlled_locations():  # scenarios.rs:856
    s = State.blank(WHITE)
    s.set_marker(LOC_11, WHITE)
    s.set_marker(LOC_25, WHITE)
    s.set_unit(LOC_25, WHITE, KNIGHT, 1)
    s.add_zone(WHITE, Z_HAND, ARCHER, 1)
    acts = s.legal_actions()
    assert has(acts, A.Deploy(ARCHER, LOC_11))
    assert not has(acts, A.Deploy(ARCHER, LOC_25))
    assert not has(acts, A.Deploy(ARCHER, LOC_53))


# ------------------------------------------------------------- MOVE rules

def test_move_only_into_empty_hexes():  # scenarios.rs:900
    s = one_unit(KNIGHT, CENTER)
    s.set_unit(E1, BLACK, FOOTMAN, 1)
    acts = s.legal_actions()
    assert not has(acts, A.Move(CENTER, E1))
    assert has(acts, A.Move(CENTER, W1))


# -------------------------------------------------------- ACTION ENCODING

ENCODE_SAMPLES = [  # scenarios.rs:920-990
    A.Deploy(ARCHER, 5), A.Bolster(KNIGHT, 18), A.ClaimInitiative(ROYAL_COIN), A.Recruit(ARCHER, MARSHAL),
    A.Pass(ROYAL_COIN), A.Move(18, 19), A.Control(11), A.Attack(18, 19), A.TacArcher(18, 20),
    A.TacCavalryMove(18, 19), A.TacCavalryAttack(19, 20), A.TacCrossbow(17, 19), A.TacEnsign(18, 19),
    A.TacLancer(17, 18, 19), A.TacLightCav(17, 19), A.TacMarshal(17, 24), A.TacRoyalGuard(18, 20),
    A.TacFootman(FOOTMAN), A.FootMove(18, 19), A.FootControl(11), A.FootAttack(18, 19), A.DrawCoin(ARCHER),
    A.DrawCoin(NONE), A.RGSoakSupply(), A.RGSoakStack(), A.SwordsmanMove(18, 19), A.SwordsmanDecline(),
    A.BerserkMove(18, 19), A.BerserkControl(11), A.BerserkAttack(18, 19), A.BerserkStop(), A.MercMove(18, 19),
    A.MercControl(11), A.MercAttack(18, 19), A.MercDecline(), A.FootmanInstantDeploy(11),
    A.FootmanInstantDecline()]


def test_action_encode_decode_roundtrip():  # scenarios.rs:918
    """Every sampled variant decodes and re-encodes to the same code. The
    library's decoder is exercised by wc_state_apply, which refuses an
    undecodable code: a legal action applied by its code must be accepted."""
    for code in ENCODE_SAMPLES:
        kind, fields = decode(code)
        assert encode(kind, *fields) == code, kind
    # the library decodes exactly the codes it produces
    s = one_unit(KNIGHT, CENTER)
    for code in s.legal_actions():
        s.apply_checked(code)


# ------------------------------------------------------ census-replay fixes

def test_royal_guard_tactic_with_only_royal_coin_in_hand_discards_it_faceup():  # scenarios.rs:999
    s = State.blank(WHITE)
    s.set_unit(CENTER, WHITE, ROYAL_GUARD, 1)
    s.set_marker(LOC_11, WHITE)
    s.add_zone(WHITE, Z_HAND, ROYAL_COIN, 1)
    assert has(s.legal_actions(), A.TacRoyalGuard(CENTER, LOC_11)), \
        "RG tactic must be offered with only the Royal Coin in hand"
    s2 = s.apply(A.TacRoyalGuard(CENTER, LOC_11))
    assert s2.zones[WHITE][Z_FACEUP][ROYAL_COIN] == 1, "Royal Coin goes to the FACE-UP discard"
    assert s2.zones[WHITE][Z_FACEDOWN][ROYAL_COIN] == 0
    assert s2.hex_type[LOC_11] == ROYAL_GUARD


def test_footman_v2_recruit_coin_stays_in_discard_until_deployed():  # scenarios.rs:1031
    s = State.blank(WHITE)
    s.set_unit(CENTER, WHITE, FOOTMAN_V2, 1)
    s.set_marker(LOC_11, WHITE)
    s.add_zone(WHITE, Z_HAND, FOOTMAN_V2, 1)
    s.add_zone(WHITE, Z_SUPPLY, FOOTMAN_V2, 1)
    s2 = s.apply(A.Recruit(FOOTMAN_V2, FOOTMAN_V2))
    assert s2.pending().kind == "FootmanInstantDeploy"
    assert s2.zones[WHITE][Z_FACEUP][FOOTMAN_V2] == 1
    assert s2.zones[WHITE][Z_HAND][FOOTMAN_V2] == 0
    s3 = s2.apply(A.FootmanInstantDeploy(LOC_11))
    assert s3.hex_type[LOC_11] == FOOTMAN_V2
    assert s3.zones[WHITE][Z_FACEUP][FOOTMAN_V2] == 0
    s4 = s2.apply(A.FootmanInstantDecline())
    assert s4.zones[WHITE][Z_FACEUP][FOOTMAN_V2] == 1


def test_footman_tactic_covers_both_versions_in_any_order():  # scenarios.rs:1056
    s = State.blank(WHITE)
    s.set_unit(CENTER, WHITE, FOOTMAN, 1)
    s.set_unit(W1, WHITE, FOOTMAN_V2, 1)
    s.add_zone(WHITE, Z_HAND, FOOTMAN, 1)
    s2 = s.apply(A.TacFootman(FOOTMAN))
    p = s2.pending()
    assert p.kind == "FootmanManeuver", f"expected FootmanManeuver, got {p}"
    assert p.hexes_list() == [W1, CENTER], "both footman versions owe a maneuver"
    acts = s2.legal_actions()
    assert has(acts, A.FootMove(CENTER, E1))
    assert has(acts, A.FootMove(W1, 16))
    s3 = s2.apply(A.FootMove(W1, 16))
    p3 = s3.pending()
    assert p3.kind == "FootmanManeuver", f"expected FootmanManeuver for the remaining footman, got {p3}"
    assert p3.hexes_list() == [CENTER]


def test_berserker_chain_attack_uses_post_payment_height_for_knight_immunity():  # scenarios.rs:1104
    s = State.blank(WHITE)
    s.set_unit(CENTER, WHITE, BERSERKER, 2)
    s.set_unit(19, BLACK, KNIGHT, 1)
    s.add_zone(WHITE, Z_HAND, BERSERKER, 1)
    s2 = s.apply(A.Move(CENTER, 12))
    assert s2.pending().kind == "BerserkerChain"
    assert not has(s2.legal_actions(), A.BerserkAttack(12, 19)), \
        "height-2 chain attack resolves at height 1: Knight is immune"
    t = State.blank(WHITE)
    t.set_unit(CENTER, WHITE, BERSERKER, 3)
    t.set_unit(19, BLACK, KNIGHT, 1)
    t.add_zone(WHITE, Z_HAND, BERSERKER, 1)
    t2 = t.apply(A.Move(CENTER, 12))
    assert has(t2.legal_actions(), A.BerserkAttack(12, 19))


def test_warrior_priest_draw_resolves_before_rg_soak_choice():  # scenarios.rs:1145
    s = State.blank(WHITE)
    s.set_unit(CENTER, WHITE, WARRIOR_PRIEST, 1)
    s.set_unit(E1, BLACK, ROYAL_GUARD, 1)
    s.add_zone(BLACK, Z_SUPPLY, ROYAL_GUARD, 1)
    s.add_zone(WHITE, Z_HAND, WARRIOR_PRIEST, 1)
    s.add_zone(WHITE, Z_BAG, ARCHER, 1)
    s2 = s.apply(A.Attack(CENTER, E1))
    p = s2.pending()
    assert p.kind == "WarriorPriestDraw", f"expected WarriorPriestDraw before the soak, got {p}"
    assert p.player == WHITE and p.rg_hex == E1
    s3 = s2.apply(A.DrawCoin(ARCHER))
    assert s3.pending().kind == "RoyalGuardChoice", "defender's soak choice comes after the draw"
    s4 = s3.apply(A.RGSoakSupply())
    assert s4.zones[BLACK][Z_SUPPLY][ROYAL_GUARD] == 0
    assert s4.zones[BLACK][Z_ELIM][ROYAL_GUARD] == 1
    assert s4.hex_height[E1] == 1, "stack untouched after a supply soak"
    assert s4.pending().kind == "WarriorPriestPlay", f"the forced play comes after the soak, got {s4.pending()}"
    assert s4.zones[WHITE][Z_INFLIGHT][ARCHER] == 1


def test_ensign_cannot_move_itself():  # scenarios.rs:1190
    s = one_unit(ENSIGN, CENTER)
    s.set_unit(W1, WHITE, SWORDSMAN, 1)
    acts = s.legal_actions()
    assert count_kind(acts, "TacEnsign", lambda frm, to: frm == CENTER) == 0, "Ensign must not grant itself a move"
    assert count_kind(acts, "TacEnsign", lambda frm, to: frm == W1) > 0


def test_marshal_cannot_grant_itself_an_attack():  # scenarios.rs:1214
    s = one_unit(MARSHAL, CENTER)
    s.set_unit(E1, BLACK, SWORDSMAN, 1)
    s.set_unit(W1, WHITE, PIKEMAN, 1)
    s.set_unit(16, BLACK, SCOUT, 1)
    acts = s.legal_actions()
    assert count_kind(acts, "TacMarshal", lambda uh, t: uh == CENTER) == 0, "Marshal must not direct itself"
    assert has(acts, A.TacMarshal(W1, 16))
    assert has(acts, A.Attack(CENTER, E1))


def test_illegal_action_is_refused():
    """The boundary refuses an action the state does not allow (the
    reference would panic inside apply; the C ABI returns WC_E_ARG)."""
    import warchest_b200 as wc
    s = one_unit(KNIGHT, CENTER)
    with pytest.raises(wc.SolveError):
        s.apply_checked(A.Move(CENTER, 30))
    with pytest.raises(wc.SolveError):  # unchecked still refuses a move from an empty hex
        s.apply(A.Move(W1, 30))
    with pytest.raises(wc.SolveError):  # and a state whose fields are out of range
        bad = one_unit(KNIGHT, CENTER)
        bad.hex_type[3] = 40
        bad.legal_actions()
