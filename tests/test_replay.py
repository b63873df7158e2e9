"""The training batch's CPU side: replay rows, the oracle's restated
expansion and mirror, pinned by the reference's own checks.

  * expand_row (engine/src/rebel.rs:1353) of a state's packed row, with the
    state's own hand / face-down / bag sizes, equals the live encoder
    write_public_features (rebel.rs:1079) of the state, bit for bit;
  * the row mirror (train/mirror.py:60-85) agrees with the engine's own
    rotation, State::mirror, on coin-play states of seeded playouts
    (train/mirror.py:176-196 check_against_engine);
  * the mirror is an involution, swaps the unit ids, and expansion commutes
    with the feature-level mirror (train/mirror.py:127-173 self_check and
    self_check_rows, with mirror_x restated here from train/mirror.py:
    88-125).
"""
import ctypes as C

import numpy as np

ROW_BYTES, PUBFEAT = 215, 897
N_HEXES, HEX_CH, HEX_FACTS, NSLOT = 37, 16, 6, 5
PILE_COUNTS, CARD_FEATS, PLAYER_SCALARS = 4, 25, 6
OFF_PILES = N_HEXES * HEX_CH
OFF_CARDS = OFF_PILES + 2 * NSLOT * PILE_COUNTS
OFF_LOOSE = OFF_CARDS + 2 * NSLOT * CARD_FEATS
ROW_IDS, ROW_HEX_HEIGHT = 12, 22 + 2 * N_HEXES


def _lib(oracle):
    L = oracle.lib()
    L.oracle_replay_mirror_pairs.restype = C.c_size_t
    L.oracle_replay_mirror_pairs.argtypes = [C.c_uint32, C.c_uint64, C.c_void_p, C.c_size_t]
    return L


def mirror_rows(oracle, rows):
    rows = np.ascontiguousarray(rows, np.uint8)
    out = np.zeros_like(rows)
    oracle.lib().oracle_replay_mirror_rows(rows.ctypes.data_as(C.c_void_p), C.c_size_t(len(rows)),
                                           out.ctypes.data_as(C.c_void_p))
    return out


def expand(oracle, rows, hand, fd, bag):
    out = np.zeros((len(rows), PUBFEAT), np.float32)
    for i, r in enumerate(np.ascontiguousarray(rows, np.uint8)):
        h, f, b = (np.ascontiguousarray(a[i], np.uint8) for a in (hand, fd, bag))
        oracle.lib().oracle_replay_expand_row(r.ctypes.data_as(C.c_void_p), h.ctypes.data_as(C.c_void_p),
                                              f.ctypes.data_as(C.c_void_p), b.ctypes.data_as(C.c_void_p),
                                              out[i].ctypes.data_as(C.c_void_p))
    return out


def hexmap(oracle):
    """The rotation's hex permutation, read back through the row mirror: a
    row whose heights are the hex numbers mirrors to heights HEXMAP[h]."""
    row = np.full((1, ROW_BYTES), 255, np.uint8)
    row[0, ROW_HEX_HEIGHT:ROW_HEX_HEIGHT + N_HEXES] = np.arange(N_HEXES)
    return mirror_rows(oracle, row)[0, ROW_HEX_HEIGHT:ROW_HEX_HEIGHT + N_HEXES].astype(np.int64)


def feature_mirror(hm):
    """train/mirror.py:88-125: the permutation of the expanded encoding."""
    perm = np.arange(PUBFEAT)
    for h in range(N_HEXES):
        src, dst = h * HEX_CH, int(hm[h]) * HEX_CH
        perm[dst:dst + HEX_CH] = src + np.arange(HEX_CH)
        perm[dst + 0], perm[dst + 1] = src + 1, src + 0
        perm[dst + 3], perm[dst + 4] = src + 4, src + 3
        for k in range(NSLOT):
            perm[dst + HEX_FACTS + k] = src + HEX_FACTS + NSLOT + k
            perm[dst + HEX_FACTS + NSLOT + k] = src + HEX_FACTS + k
    for off, width in [(OFF_PILES, NSLOT * PILE_COUNTS), (OFF_CARDS, NSLOT * CARD_FEATS),
                       (OFF_LOOSE, PLAYER_SCALARS)]:
        for k in range(width):
            perm[off + k], perm[off + width + k] = off + width + k, off + k
    return perm, [OFF_LOOSE + 2 * PLAYER_SCALARS + 2]


def mirror_x(x, perm, flip):
    out = x[:, perm]
    out[:, flip] = 1.0 - out[:, flip]
    return out


def states(wc, n=24):
    out = []
    for s in range(n):
        try:
            out.append(wc.generate_root(s, plies=[0, 6, 20, 40][s % 4]))
        except wc.SolveError:
            continue
    return out


def test_row_header_and_live_encoder(wc, oracle):
    """pack_row writes format version 1 and the rules hash, and expanding it
    with the state's sizes gives the live encoder's features exactly."""
    roots = states(wc)
    rows = [wc.pack_row(r) for r in roots]
    hashes = {bytes(r[4:12]) for r in rows}
    assert len(hashes) == 1
    for root, row in zip(roots, rows):
        assert int.from_bytes(row[0:4], "little") == 1
        want = np.zeros(PUBFEAT, np.float32)
        sizes = np.zeros(6, np.uint8)
        assert oracle.lib().oracle_replay_live(root, C.c_size_t(len(root)), want.ctypes.data_as(C.c_void_p),
                                               sizes.ctypes.data_as(C.c_void_p)) == 0
        got = expand(oracle, np.frombuffer(row, np.uint8)[None], sizes[None, 0:2], sizes[None, 2:4], sizes[None, 4:6])
        np.testing.assert_array_equal(got[0], want)


def test_mirror_agrees_with_the_engine(oracle):
    L = _lib(oracle)
    cap = 600
    buf = np.zeros((2 * cap, ROW_BYTES), np.uint8)
    n = L.oracle_replay_mirror_pairs(8, 11, buf.ctypes.data_as(C.c_void_p), cap)
    assert n > 50
    rows, want = buf[0:2 * n:2], buf[1:2 * n:2]
    got = mirror_rows(oracle, rows)
    bad = np.flatnonzero((got != want).any(axis=1))
    assert not len(bad), f"{len(bad)} of {n} rows disagree with State::mirror"


def test_mirror_self_check(wc, oracle):
    L = _lib(oracle)
    cap = 256
    buf = np.zeros((2 * cap, ROW_BYTES), np.uint8)
    n = L.oracle_replay_mirror_pairs(4, 5, buf.ctypes.data_as(C.c_void_p), cap)
    rows = buf[0:2 * n:2]
    mr = mirror_rows(oracle, rows)
    np.testing.assert_array_equal(mirror_rows(oracle, mr), rows)  # an involution
    np.testing.assert_array_equal(rows[:, ROW_IDS:ROW_IDS + NSLOT], mr[:, ROW_IDS + NSLOT:ROW_IDS + 2 * NSLOT])
    rng = np.random.default_rng(3)
    hand, fd, bag = (rng.integers(0, 6, (n, 2)).astype(np.uint8) for _ in range(3))
    x = expand(oracle, rows, hand, fd, bag)
    a = expand(oracle, mr, hand[:, ::-1], fd[:, ::-1], bag[:, ::-1])
    perm, flip = feature_mirror(hexmap(oracle))
    mx = mirror_x(x, perm, flip)
    np.testing.assert_allclose(a, mx, atol=1e-6)  # row mirror and feature mirror commute
    np.testing.assert_allclose(mirror_x(mx, perm, flip), x)
    loc = slice(5, OFF_PILES, HEX_CH)
    np.testing.assert_array_equal(x[:, loc], mx[:, loc])  # the location map is rotation-invariant
    g = OFF_LOOSE + 2 * PLAYER_SCALARS
    np.testing.assert_array_equal(x[:, g:g + 2], mx[:, g:g + 2])  # plies and initiative-moved stay
    np.testing.assert_array_equal(x[:, g + 2], 1.0 - mx[:, g + 2])  # to-act flips
    np.testing.assert_array_equal(x[:, 1:OFF_PILES:HEX_CH].sum(1), mx[:, 0:OFF_PILES:HEX_CH].sum(1))


def test_replay_entry_points_refuse_bad_arguments(wc):
    """The device entry point checks its arguments before touching a device."""
    assert wc.lib().wc_replay_expand(None, 4, None, None, 8, None, None, None) == 1
    assert wc.lib().wc_replay_pack_row(b"\x00", 1, C.create_string_buffer(ROW_BYTES)) == 1
