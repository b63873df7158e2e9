"""Continual re-solving on the device: the game of tests/test_walk.py with
every subgame solved by wc_solve_batch (GpuClient.play, many games per
batch) walks the same trajectory as with the CPU solver. With the fp32
network the device's average strategies are bit-identical to the CPU
solver's, so every sampled action, draw and Bayes update is the same; the
carried beliefs differ only in their f16 carry-store rounding, which feeds
Phase 2's root values and not the play."""
import pytest

pytestmark = pytest.mark.gpu


def test_device_walk_matches_cpu_walk(wc, oracle):
    weights = wc.seeded_weights("test", 0xD15EA5E)
    cfg = wc.Cfg(depth=2, iters=16, snapshots=True, cfr=wc.Cfr.PLUS, node_cap=20000)
    seeds = [3, 4, 5, 6]
    games = [wc.Game(cfg, seed=s, max_solves=6) for s in seeds]
    c = wc.spawn(0, *weights, net="exact")
    try:
        solved = c.play(games)
    finally:
        c.close()
    assert solved == sum(g.counters()["solves"] for g in games)
    for s, g in zip(seeds, games):
        want, want_root = oracle.walk(s, cfg, weights, max_solves=6)
        got = g.counters()
        print(s, got)
        assert got == want
        assert g.root() == want_root


def test_belief_heavy_roots_resolve_repeatedly(wc):
    """BASELINE configs[4]'s loop in miniature: belief-heavy roots (up to 256
    consistent configs per player, Dirichlet(1) weights), re-solved after
    each walk, 8 solves per game, on the tensor-core network."""
    weights = wc.seeded_weights("he", 0)
    cfg = wc.Cfg(depth=2, iters=32, snapshots=True, cfr=wc.Cfr.PLUS, node_cap=200000)
    games = [wc.Game(cfg, seed=s, root=wc.generate_wide_root(s, 256), max_solves=8) for s in range(8)]
    c = wc.spawn(0, *weights, net="f16")
    try:
        c.play(games)
    finally:
        c.close()
    for g in games:
        ctr = g.counters()
        print(ctr)
        assert ctr["ended"] == 1
        assert ctr["solves"] + ctr["capped"] >= 1
