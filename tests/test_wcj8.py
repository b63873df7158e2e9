"""The reference's job byte format, WCJ8 (engine/src/serialize.rs), through
the C ABI: wc_wcj8_from_root writes it, wc_job_from_wcj8 reads it.

Restates engine/tests/serialize_oracle.rs on this library's trees:
  * real_solver_round_trips (:21): bytes parse and re-serialise to the
    identical bytes, with the solver's node, iteration, row and cell counts;
  * tables_are_consistent (:83): CSR spans, config spans, soff monotonicity,
    the reverse tables' one block per non-root node in its parent's row
    space, ordered legal rows, child ids and transitions in range, the BFS
    order a permutation tiled by the levels, every leaf listed once;
  * starter_draft_round_trips (:196): seeded and starter drafts alike;
and adds the reader's own bar: the job read from the bytes is the job built
from the root, byte for byte (wc_job_digest), so a WCJ8 job solves exactly
as the root's own.
"""
import struct

import numpy as np
import pytest

FIELDS = [
    ("node_kind", "u8"), ("node_player", "u8"), ("node_child_start", "u32"), ("node_child", "u32"),
    ("obs_off", "u32"), ("obs_start", "u32"), ("obs_act", "u32"), ("obs_child", "u32"),
    ("legal_row_of", "u32"), ("legal_off", "u32"), ("legal_action", "u32"), ("legal_child", "u32"),
    ("legal_trans", "u32"), ("cell_row", "u32"), ("draw_off", "u32"), ("draw_to", "u32"), ("draw_p", "f32"),
    ("draw_row_off", "u32"), ("draw_row_start", "u32"), ("cfg_off", "u32"), ("reach_off", "u32"),
    ("soff", "u32"), ("node_parent", "u32"), ("rev_row_of", "u32"), ("rev_start", "u32"), ("rev_src", "u32"),
    ("rev_cell", "u32"), ("rvd_row_of", "u32"), ("rvd_start", "u32"), ("rvd_src", "u32"), ("rvd_p", "f32"),
    ("leaf_rows", "u32"), ("term_leaves", "u32"), ("terminal_utility", "f32"), ("leaf_coff", "u32"),
    ("leaf_cidx", "u32"), ("snap_coff", "u32"), ("leaf_raw", "u8"), ("card_feat", "f32"), ("cphi", "f32"),
    ("cplayer", "u8"), ("bfs_order", "u32"), ("level_start", "u32"),
]
NONE32 = 0xFFFFFFFF


class Bytes:
    """serialize.rs:993-1040 (R): little-endian, a u32 count before arrays."""

    def __init__(self, b):
        self.b, self.at = b, 0

    def u32(self):
        v = struct.unpack_from("<I", self.b, self.at)[0]
        self.at += 4
        return v

    def f32(self):
        v = struct.unpack_from("<f", self.b, self.at)[0]
        self.at += 4
        return v

    def arr(self, kind):
        n = self.u32()
        dt, w = {"u8": (np.uint8, 1), "u32": (np.dtype("<u4"), 4), "f32": (np.dtype("<f4"), 4)}[kind]
        v = np.frombuffer(self.b, dt, n, self.at).copy()
        self.at += n * w
        return v


def parse(b):
    r = Bytes(b)
    assert r.u32() == 0x57434A38 and r.u32() == 8
    j = {"depth": r.u32(), "iters": r.u32()}
    j["snapshots"] = b[r.at] != 0
    r.at += 1
    j["cfr"] = [r.f32() for _ in range(4)]
    j["snap_iters"], j["net_dims"] = r.arr("u32"), r.arr("u32")
    for k in ("nodes", "ncfg", "rows", "ncells"):
        j[k] = r.u32()
    for name, kind in FIELDS:
        j[name] = r.arr(kind)
    j["root"] = [r.arr("f32"), r.arr("f32")]
    j["carried"] = [[r.arr("f32"), r.arr("f32")] for _ in range(r.u32())]
    assert r.at == len(b), "trailing bytes"
    return j


def write(j):
    """serialize.rs:1051-1125 (to_bytes), the test's own writer."""
    out = [struct.pack("<II", 0x57434A38, 8), struct.pack("<II", j["depth"], j["iters"]),
           bytes([1 if j["snapshots"] else 0]), struct.pack("<4f", *j["cfr"])]

    def arr(v, kind):
        dt = {"u8": np.uint8, "u32": np.dtype("<u4"), "f32": np.dtype("<f4")}[kind]
        out.append(struct.pack("<I", len(v)) + np.asarray(v, dt).tobytes())

    arr(j["snap_iters"], "u32")
    arr(j["net_dims"], "u32")
    out.append(struct.pack("<4I", j["nodes"], j["ncfg"], j["rows"], j["ncells"]))
    for name, kind in FIELDS:
        arr(j[name], kind)
    arr(j["root"][0], "f32")
    arr(j["root"][1], "f32")
    out.append(struct.pack("<I", len(j["carried"])))
    for c in j["carried"]:
        arr(c[0], "f32")
        arr(c[1], "f32")
    return b"".join(out)


def cfg_of(wc, depth=2, snapshots=True, rule="PLUS"):
    return wc.Cfg(depth=depth, iters=8, snapshots=snapshots, cfr=getattr(wc.Cfr, rule), node_cap=200000)


def roots(wc, n, plies=20, random_draft=True):
    out = []
    for s in range(n):
        try:
            out.append(wc.generate_root(s, plies, random_draft=random_draft))
        except wc.SolveError:
            continue
    return out


def test_real_solver_round_trips(wc):
    cfg = cfg_of(wc)
    checked = 0
    for root in roots(wc, 8):
        b = wc.wcj8_bytes(root, cfg)
        j = parse(b)
        assert write(j) == b, "byte-identical round trip"
        job = wc.PackedJob.from_root(root, cfg)
        assert j["nodes"] == job.info["nodes"] and j["iters"] == cfg.iters
        assert j["rows"] == len(j["leaf_rows"]) == job.info["net_rows"]
        assert j["ncells"] == job.info["cells"]
        assert list(j["snap_iters"]) == wc.snapshot_iters(cfg.iters) and list(j["net_dims"]) == [5]
        checked += 1
    assert checked >= 4


def tables_consistent(j):
    n = j["nodes"]
    assert len(j["node_child_start"]) == n + 1 and j["node_child_start"][n] == len(j["node_child"])
    assert len(j["soff"]) == n + 1 and j["soff"][n] == j["ncells"]
    assert j["legal_off"][0] == 0 and j["legal_off"][-1] == j["ncells"]
    assert np.all(np.diff(j["legal_off"].astype(np.int64)) >= 0)
    for k in ("legal_action", "legal_child", "legal_trans", "cell_row"):
        assert len(j[k]) == j["ncells"]
    assert len(j["cfg_off"]) == 2 * n + 1
    assert j["reach_off"][n] == j["reach_off"][-1]
    assert j["rev_start"][-1] == len(j["rev_src"]) == len(j["rev_cell"])
    assert j["rvd_start"][-1] == len(j["rvd_src"]) == len(j["rvd_p"])
    par, kind = j["node_parent"], j["node_kind"]
    assert par[0] == NONE32
    for c in range(1, n):
        p = int(par[c])
        assert p < c, "parent after child"
        dec = kind[p] == 0
        assert (j["rev_row_of"][c] != NONE32) == dec and (j["rvd_row_of"][c] != NONE32) == (not dec)
    cfg_off = j["cfg_off"]
    for i in range(n):
        if kind[i] != 0:
            assert j["legal_row_of"][i] == NONE32
            continue
        me = int(j["node_player"][i])
        nc = int(cfg_off[2 * i + me + 1] - cfg_off[2 * i + me])
        row0 = int(j["legal_row_of"][i])
        assert row0 + nc < len(j["legal_off"])
        na = int(j["obs_start"][j["obs_off"][i + 1] - 1])
        for c in range(nc):
            cells = range(int(j["legal_off"][row0 + c]), int(j["legal_off"][row0 + c + 1]))
            prev = -1
            for cell in cells:
                assert j["cell_row"][cell] == c
                a = int(j["legal_action"][cell])
                assert prev < a < na, "actions not ordered in row"
                prev = a
                ch = int(j["legal_child"][cell])
                assert ch < n and par[ch] == i
                tr = int(j["legal_trans"][cell])
                if tr != NONE32:
                    assert tr < cfg_off[2 * ch + me + 1] - cfg_off[2 * ch + me]
    assert len(j["leaf_coff"]) == 2 * j["rows"] + 1 and j["leaf_coff"][-1] == len(j["leaf_cidx"])
    assert sorted(j["bfs_order"]) == list(range(n))
    ls = j["level_start"]
    assert ls[0] == 0 and ls[-1] == n
    marks = np.zeros(n, np.int64)
    np.add.at(marks, j["leaf_rows"], 1)
    np.add.at(marks, j["term_leaves"], 1)
    assert np.array_equal(marks > 0, kind == 2) and marks.max() <= 1
    assert np.all(np.isfinite(j["terminal_utility"]))


def test_tables_are_consistent(wc):
    cfg = cfg_of(wc)
    for root in roots(wc, 6):
        tables_consistent(parse(wc.wcj8_bytes(root, cfg)))


@pytest.mark.parametrize("depth,snapshots,rule", [(2, True, "PLUS"), (2, False, "LINEAR"), (3, False, "PLUS")])
def test_job_from_bytes_is_the_job_from_the_root(wc, depth, snapshots, rule):
    cfg = cfg_of(wc, depth, snapshots, rule)
    for root in roots(wc, 3 if depth == 3 else 6):
        try:
            direct = wc.PackedJob.from_root(root, cfg)
        except wc.SolveError:  # over the node cap
            continue
        b = wc.wcj8_bytes(root, cfg)
        assert wc.PackedJob.from_wcj8(b, cfg).digest == direct.digest


def test_carried_roots_travel(wc):
    cfg = cfg_of(wc)
    root = wc.generate_root(4)
    job = wc.PackedJob.from_root(root, cfg)
    w = len(job.root_belief())
    rng = np.random.default_rng(1)
    carried = rng.random((3, w)).astype(np.float32)
    b = wc.wcj8_bytes(root, cfg, carried)
    j = parse(b)
    assert len(j["carried"]) == 3
    np.testing.assert_array_equal(np.concatenate(j["carried"][1]), carried[1])
    assert wc.PackedJob.from_wcj8(b, cfg).digest == wc.PackedJob.from_root(root, cfg, carried).digest


def test_starter_draft_round_trips(wc):
    for draft in (True, False):
        for plies in (0, 6, 30):
            for root in roots(wc, 3, plies, draft):
                b = wc.wcj8_bytes(root, cfg_of(wc))
                assert write(parse(b)) == b


def test_reader_refuses_malformed_bytes(wc):
    b = wc.wcj8_bytes(wc.generate_root(0), cfg_of(wc))
    bad = [b"WCJ8" + b[4:], b[:4] + struct.pack("<I", 7) + b[8:], b[:-1], b + b"\x00"]
    j = parse(b)
    j["cplayer"] = j["cplayer"][:-1]  # a count that disagrees with ncfg
    bad.append(write(j))
    for x in bad:
        with pytest.raises(wc.SolveError) as e:
            wc.PackedJob.from_wcj8(x, cfg_of(wc))
        assert e.value.code == 1


def _first(mask):
    idx = np.flatnonzero(mask)
    assert idx.size, "the tree has no such entry"
    return int(idx[0])


@pytest.mark.parametrize("what", [
    "node_child", "legal_child", "legal_trans", "cell_row", "obs_act", "obs_child", "draw_to",
    "leaf_rows", "term_leaves", "leaf_cidx", "cplayer", "soff", "leaf_coff", "legal_off", "draw_row_start",
    "cfg_span", "cfg_total", "legal_row_of",
])
def test_reader_refuses_indices_out_of_range(wc, what):
    """Bytes whose every count agrees but one index points outside its
    table: the reader returns an argument error (code 1) rather than handing
    the flattener an index to follow."""
    cfg = cfg_of(wc)
    # roots with chance nodes (seed 6) and with game-ending leaves (seed 23,
    # 260 plies in) for the tables only those hold
    seed, plies = {"draw_to": (6, 20), "draw_row_start": (6, 20), "term_leaves": (23, 260)}.get(what, (0, 20))
    b = wc.wcj8_bytes(wc.generate_root(seed, plies), cfg)
    j = parse(b)
    n, big = j["nodes"], 1 << 30
    if what in ("node_child", "leaf_rows", "term_leaves"):
        j[what][0] = n
    elif what == "legal_child":
        j[what][0] = n + 5
    elif what == "legal_trans":
        j[what][_first(j[what] != NONE32)] = big
    elif what == "cell_row":
        j[what][0] = big
    elif what in ("obs_act", "obs_child"):
        j[what][0] = big
    elif what == "draw_to":
        j[what][0] = big
    elif what == "leaf_cidx":
        j[what][0] = j["ncfg"]
    elif what == "cplayer":
        j[what][0] = 2
    elif what == "soff":  # a decreasing step that keeps both ends
        k = _first(np.diff(j["soff"].astype(np.int64)) > 0)
        j[what][k + 1] = j[what][k] - 1 if j[what][k] else j[what][k + 2] + 1
    elif what == "leaf_coff":  # a row whose config span no longer fits its node
        k = _first(np.diff(j["leaf_coff"].astype(np.int64)) > 0)
        j[what][k + 1] += 1
    elif what == "legal_off":  # a legal row reaching past its node's cells
        j[what][1] = big
    elif what == "draw_row_start":
        j[what][j["draw_row_off"][_first(j["node_kind"] == 1)]] += 1
    elif what in ("cfg_span", "cfg_total"):  # spans no solvable job has, refused before anything is sized by them
        add = (1 << 20) + 1 if what == "cfg_span" else 1 << 28
        j["cfg_off"][-2:] += np.uint32(add)
    elif what == "legal_row_of":  # a first legal row whose end would wrap 32 bits
        j[what][_first(j["node_kind"] == 0)] = NONE32 - 1
    x = write(j)
    assert x != b
    with pytest.raises(wc.SolveError) as e:
        wc.PackedJob.from_wcj8(x, cfg)
    assert e.value.code == 1
