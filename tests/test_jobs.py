"""Tree flattening on the host (CPU): the job image the device solves has
the shape of the tree the builder made, and its per-level task lists cover
that tree exactly once. The oracle links the same host builder sources, so
the shape equality below is a consistency check of the flattener (job image
against the unflattened tree), not a parity pin: the tree and the legal-move
order are pinned to the reference by the restated reference tests
(test_scenarios.py, test_rebel_pbs.py, test_solver_oracle.py), and the
flattened job by the bit-identical GPU solves against the oracle, which
solves the unflattened tree."""
import numpy as np
import pytest


@pytest.mark.parametrize("depth,seeds", [(1, range(4)), (2, range(4)), (3, [0])])
def test_job_image_matches_its_tree(wc, oracle, depth, seeds):
    for seed in seeds:
        root = wc.generate_root(seed)
        cfg = wc.Cfg(depth=depth, iters=4, snapshots=True, cfr=wc.Cfr.PLUS)
        job = wc.PackedJob.from_root(root, cfg)
        o = oracle.Oracle(root, cfg)
        s = o.shape
        for k in ("nodes", "cells", "net_rows", "terminal_leaves", "configs", "levels"):
            assert job.info[k] == s[k], (seed, k, job.info[k], s[k])
        assert job.info["root_nc0"] == o.nc0 and job.info["root_nc1"] == o.nc1
        assert o.lib_ncells() == job.info["cells"] if hasattr(o, "lib_ncells") else True
        # both players' root beliefs are distributions
        rb = job.root_belief()
        assert rb.size == o.nc0 + o.nc1
        assert abs(rb[: o.nc0].sum() - 1) < 1e-5 and abs(rb[o.nc0:].sum() - 1) < 1e-5
        # exit nodes: the carry layout lists the oracle's exit leaves in order
        off, ids = job.carry_layout()
        np.testing.assert_array_equal(ids, o.exit_leaves())
        assert np.all(np.diff(off.astype(np.int64)) >= 0)


def test_task_counts_cover_the_tree(wc):
    """wc_job_counts: every legal cell is in exactly one regret-matching row
    range, and each player's row count is its share of the decision rows."""
    for seed in range(3):
        job = wc.PackedJob.from_root(wc.generate_root(seed), wc.Cfg(depth=2, iters=4, snapshots=False,
                                                                   cfr=wc.Cfr.PLUS))
        c = job.counts()
        assert c[0] + c[1] == job.info["cells"]
        assert c[2] > 0 and c[3] > 0
        assert c[4] + c[5] > 0  # value gather entries


def test_node_cap_is_reported(wc):
    root = wc.generate_root(0)
    with pytest.raises(wc.SolveError) as e:
        wc.PackedJob.from_root(root, wc.Cfg(depth=3, iters=4, snapshots=False, cfr=wc.Cfr.PLUS, node_cap=50))
    assert e.value.code == 3  # WC_E_CAPPED


def test_batch_build_equals_one_at_a_time(wc):
    """wc_job_build_batch (the parallel tape builder) gives, root for root, the
    job wc_job_build gives: the same bytes (digest), including the capped
    roots, which come back empty as the reference's tape builder skips them
    (wave_tape.rs:48-61)."""
    roots = [wc.generate_root(s) for s in range(12)]
    for cap in (0, 3000):
        cfg = wc.Cfg(depth=3, iters=8, snapshots=False, cfr=wc.Cfr.PLUS, node_cap=cap)
        one = []
        for r in roots:
            try:
                one.append(wc.PackedJob.from_root(r, cfg))
            except wc.SolveError as e:
                assert e.code == 3  # WC_E_CAPPED
                one.append(None)
        for threads in (1, 4):
            many = wc.PackedJob.build_many(roots, cfg, threads=threads)
            assert [j is None for j in many] == [j is None for j in one]
            for a, b in zip(one, many):
                if a is not None:
                    assert a.digest == b.digest
                    assert a.info == b.info
        if cap:
            assert any(j is None for j in one) and any(j is not None for j in one)


def test_batch_build_reports_a_bad_root(wc):
    cfg = wc.Cfg(depth=2, iters=4, snapshots=False, cfr=wc.Cfr.PLUS)
    good = wc.generate_root(0)
    with pytest.raises(wc.SolveError) as e:
        wc.PackedJob.build_many([good, b"\x00\x01"], cfg, threads=2)
    assert "root 1" in str(e.value)
    assert wc.PackedJob.build_many([], cfg) == []


def test_digest_separates_different_jobs(wc):
    cfg = wc.Cfg(depth=2, iters=4, snapshots=False, cfr=wc.Cfr.PLUS)
    d = {wc.PackedJob.from_root(wc.generate_root(s), cfg).digest for s in range(6)}
    assert len(d) == 6


def test_batch_build_with_carried_beliefs(wc):
    """Per-root carried root pairs (the tape builder carries the live belief,
    wave_tape.rs:57-58) give the job from_root gives with the same pairs; a
    root without any values its live belief as the one Phase-2 root."""
    cfg = wc.Cfg(depth=2, iters=4, snapshots=True, cfr=wc.Cfr.PLUS)
    roots = [wc.generate_root(s) for s in range(5)]
    rng = np.random.default_rng(7)
    carried = []
    for i, r in enumerate(roots):
        if i == 2:
            carried.append(None)
            continue
        j = wc.PackedJob.from_root(r, cfg)
        w = j.info["root_nc0"] + j.info["root_nc1"]
        carried.append(rng.random((i + 1, w), dtype=np.float32))
    many = wc.PackedJob.build_many(roots, cfg, threads=3, carried=carried)
    for r, c, b in zip(roots, carried, many):
        a = wc.PackedJob.from_root(r, cfg, c)
        assert a.digest == b.digest
        assert b.info["ncarried"] == (1 if c is None else c.shape[0])


def test_wide_roots(wc, oracle):
    """Belief-heavy roots: each player's belief covers
    min(ncfg, |consistent configs|) configs with positive weights summing to
    one, the same seed gives the same bytes, and the oracle builds the same
    tree from them."""
    cfg = wc.Cfg(depth=2, iters=4, snapshots=True, cfr=wc.Cfr.PLUS)
    for seed in range(3):
        full = wc.PackedJob.from_root(wc.generate_wide_root(seed, 100000), cfg)
        n_all = (full.info["root_nc0"], full.info["root_nc1"])
        for ncfg in (4, 256):
            r = wc.generate_wide_root(seed, ncfg)
            assert r == wc.generate_wide_root(seed, ncfg)
            job = wc.PackedJob.from_root(r, cfg)
            n = (job.info["root_nc0"], job.info["root_nc1"])
            assert n == tuple(min(ncfg, a) for a in n_all)
            rb = job.root_belief()
            for part in (rb[: n[0]], rb[n[0]:]):
                assert np.all(part > 0) and abs(part.sum() - 1) < 1e-5
            o = oracle.Oracle(r, cfg)
            for k in ("nodes", "cells", "net_rows", "configs"):
                assert job.info[k] == o.shape[k]


def test_distinct_public_rows_are_the_distinct_boards(wc, oracle):
    """The tensor-core trunk runs once per distinct public row of a job
    (wc_job_counts slot 20) and copies the board pieces to the other rows.
    That is sound only if the grouping is the one the board network itself
    makes: the number of distinct rows must equal the number of distinct P
    rows the CPU oracle's fp32 network computes (engine/src/net.rs:558-731)
    for the job's network rows."""
    weights = wc.seeded_weights("he", 0)
    cfg = wc.Cfg(depth=2, iters=4, snapshots=False, cfr=wc.Cfr.PLUS)
    shared = 0
    for seed in range(6):
        root = wc.generate_root(seed)
        job = wc.PackedJob.from_root(root, cfg)
        c = job.counts()
        pb, _, _, _ = oracle.Oracle(root, cfg, weights).net_pieces()
        distinct = np.unique(pb.view(np.uint32), axis=0).shape[0]
        assert c[20] == distinct, (seed, c[20], distinct, job.info["net_rows"])
        shared += c[20] < job.info["net_rows"]
    assert shared >= 2  # the same public position, reached along different public paths


def test_jobs_match_the_pinned_digests(wc):
    """The builder's output byte for byte (wc_job_digest) on seeded roots of
    depths 1-3 and belief-heavy depth-4 roots, against the digests pinned in
    tests/golden/job_digests.json (written by tests/golden/make_job_digests.py;
    the builder before its draw-transition and leaf-run reuse wrote the same
    digests)."""
    import importlib.util
    import json
    import os

    here = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    spec = importlib.util.spec_from_file_location("make_job_digests", os.path.join(here, "make_job_digests.py"))
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    want = json.load(open(os.path.join(here, "job_digests.json")))
    got = gen.digests(wc)
    assert [c["digest"] for c in got] == [c["digest"] for c in want]
