"""Host rules and PBS code against the reference engine's own tests (CPU).

The rules engine, the belief machinery and the tree builder are shared by
the product library and the oracle, so these checks pin both:
  * engine/tests/invariants.rs:119-171 — random playouts (10,000 seeded
    games, Rng(0xA11CE)) keep every conservation and structural invariant;
  * engine/tests/scenarios.rs:923 — every legal action met on the way
    survives encode -> decode -> encode;
  * engine/tests/invariants.rs:182-205 — random drafts never share a card;
  * engine/tests/invariants.rs:211-241 — the board tables;
  * engine/src/rebel.rs:1494-1583 — DrawScratch::run equals the per-draw
    composition (five hand-built cases, 300 fuzz cases from Rng(0xD12A)).
"""
import ctypes as C


def _msg():
    return C.create_string_buffer(1024)


def test_random_playouts_keep_the_invariants(oracle):
    L, msg, st = oracle.lib(), _msg(), (C.c_uint64 * 4)()
    rc = L.oracle_check_playouts(C.c_uint64(0xA11CE), 10000, 1000, st, msg, 1024)
    assert rc == 0, msg.value.decode()
    games, applies, cap_hits, tripped = list(st)
    print(f"{games} games, avg length {applies / games:.1f}, cap hits {cap_hits}, {tripped} actions round-tripped")
    assert games == 10000 and tripped > applies


def test_random_drafts_are_disjoint(oracle):
    msg = _msg()
    assert oracle.lib().oracle_check_drafts(5000, msg, 1024) == 0, msg.value.decode()


def test_board_tables(oracle):
    msg = _msg()
    assert oracle.lib().oracle_check_board(msg, 1024) == 0, msg.value.decode()


def test_draw_runs_match_the_per_draw_composition(oracle):
    msg, n = _msg(), C.c_int()
    assert oracle.lib().oracle_check_draw_runs(300, C.byref(n), msg, 1024) == 0, msg.value.decode()
    assert n.value == 305
