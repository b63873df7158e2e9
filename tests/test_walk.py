"""Continual re-solving (engine/src/selfplay.rs:466-905): a game of two
solving seats that walks each solved subgame with the real play and
re-solves where the walk leaves the tree, carrying the exit beliefs into
the next solve's Phase 2.

CPU: the walk driven by the CPU solver (oracle_walk) plays whole games with
every lockstep check of the reference walk holding (the tree's supports
equal the Bayes-filtered beliefs at every decision and after every draw run,
the true config never leaves the belief). GPU (test_gpu_walk.py): the same
games solved on the device give the same trajectory.
"""
import pytest


@pytest.mark.parametrize("seed,depth", [(1, 1), (2, 2)])
def test_cpu_walk_plays_whole_games(wc, oracle, seed, depth):
    cfg = wc.Cfg(depth=depth, iters=8, snapshots=True, cfr=wc.Cfr.PLUS, node_cap=20000)
    ctr, root = oracle.walk(seed, cfg, None, max_solves=0)
    print(ctr)
    assert ctr["ended"] == 1 and ctr["solves"] >= 2
    # every solved tree is walked from its root; deeper trees hold several decisions
    assert ctr["walk_decisions"] >= ctr["solves"] + ctr["capped"] * 0
    if depth > 1:
        assert ctr["walk_decisions"] > ctr["solves"]
    assert ctr["winner"] in (-1, 0, 1)


def test_cpu_walk_with_network_stops_after_max_solves(wc, oracle):
    weights = wc.seeded_weights("test", 0xD15EA5E)
    cfg = wc.Cfg(depth=2, iters=8, snapshots=True, cfr=wc.Cfr.PLUS, node_cap=20000)
    ctr, root = oracle.walk(3, cfg, weights, max_solves=3)
    print(ctr)
    assert ctr["solves"] == 3 and ctr["ended"] == 1 and ctr["walking"] == 0
    assert len(root) > 0


def test_oracle_takes_weights_above_4gb(wc, oracle):
    """The oracle entry points without declared argument types get their
    weight pointers as c_void_p: weights placed above 4 GB (an anonymous
    mapping at a high hint address) reach the walk intact."""
    import ctypes as C

    import numpy as np

    dims, w, b, ln = wc.seeded_weights("test", 0xD15EA5E)
    n = w.size + b.size + ln.size
    libc = C.CDLL(None)
    libc.mmap.restype = C.c_void_p
    libc.mmap.argtypes = [C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_int, C.c_long]
    libc.munmap.argtypes = [C.c_void_p, C.c_size_t]
    nbytes = 4 * n
    addr = libc.mmap(C.c_void_p(0x5F0000000000), nbytes, 0x3, 0x22, -1, 0)  # RW, private anonymous
    assert addr not in (None, C.c_void_p(-1).value)
    try:
        assert addr >= 1 << 32, "the mapping did not land above 4 GB"
        big = np.ctypeslib.as_array((C.c_float * n).from_address(addr))
        hw, hb, hl = big[: w.size], big[w.size: w.size + b.size], big[w.size + b.size:]
        hw[:], hb[:], hl[:] = w, b, ln
        cfg = wc.Cfg(depth=2, iters=8, snapshots=True, cfr=wc.Cfr.PLUS, node_cap=20000)
        assert oracle.walk(3, cfg, (dims, hw, hb, hl), max_solves=1) == oracle.walk(3, cfg, (dims, w, b, ln),
                                                                                     max_solves=1)
    finally:
        libc.munmap(C.c_void_p(addr), nbytes)  # the views die with this call's frame, unread
