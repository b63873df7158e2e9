"""bench.py's accounting on the CPU: the per-class algorithmic work follows
the job counts it is stated in, the roofline arithmetic divides that work by
the measured class time, and the workload builder skips capped roots the way
the reference's tape builder does (wave_tape.rs:51-56) while keeping every
kept job paired with its root."""
import json
import os

import numpy as np
import pytest

import bench


@pytest.fixture(scope="module")
def jobs(wc):
    cfg = wc.Cfg(depth=2, iters=8, snapshots=False, cfr=wc.Cfr.PLUS)
    return [wc.PackedJob.from_root(wc.generate_root(s), cfg) for s in range(3)]


def test_algorithmic_work_follows_the_counts(jobs):
    w = bench.algorithmic_work(jobs)
    assert set(w) == {"rows", "vgather", "reach", "pool", "join", "head", "trunk"}
    c = np.sum([j.counts() for j in jobs], axis=0).astype(np.float64)
    pairs = jobs[0].cfg.iters / 2.0
    rows = sum(j.info["net_rows"] for j in jobs)
    calls = jobs[0].cfg.iters + 2  # one carried root (the live belief)
    assert w["rows"] == ("hbm", (24 * (c[0] + c[1]) + 8 * (c[2] + c[3])) * pairs)
    assert w["join"] == ("tensor", 4 * 2 * 128 * 128 * rows * calls)
    assert w["trunk"] == ("tensor", 17.0e6 * c[20])
    # the regret-matching cells are every legal cell of the trees
    assert c[0] + c[1] == sum(j.info["cells"] for j in jobs)
    for bound, amount in w.values():
        assert bound in ("hbm", "tensor") and amount > 0


def test_roofline_arithmetic():
    hbm, tflops, src = bench.peaks()
    work = {"rows": ("hbm", 2.0e9), "join": ("tensor", 3.0e12), "pool": ("hbm", 1.0e9)}
    prof = {"rows": 1000.0, "join": 500.0, "pool": 0.0}  # ms; a class without time is left out
    out, src2 = bench.rooflines(prof, work)
    assert src2 == src and set(out) == {"rows", "join"}
    assert out["rows"]["achieved"] == pytest.approx(2.0)            # GB/s
    assert out["rows"]["frac"] == pytest.approx(2.0 / hbm)
    assert out["join"]["achieved"] == pytest.approx(6.0)            # TFLOP/s
    assert out["join"]["frac"] == pytest.approx(6.0 / tflops)
    peaks_file = os.path.join(os.path.dirname(bench.__file__), "MEASURED_PEAKS.json")
    if os.path.exists(peaks_file):
        with open(peaks_file) as f:
            p = json.load(f)
        assert hbm == p["hbm_gbs"] and src.startswith("measured")


def test_workload_builder_skips_capped_roots(wc):
    seeds = list(range(8))
    cfg = wc.Cfg(depth=3, iters=8, snapshots=False, cfr=wc.Cfr.PLUS, node_cap=3000)
    roots, jobs = bench.build_jobs(wc, seeds, cfg, 3)
    assert len(roots) == len(jobs) < len(seeds)
    for r, j in zip(roots, jobs):
        assert j.root == r
        assert j.info["nodes"] <= 3000
    # the kept roots are exactly the uncapped ones, in seed order
    kept = []
    for s in seeds:
        try:
            wc.PackedJob.from_root(wc.generate_root(s, bench.PLIES), cfg)
            kept.append(wc.generate_root(s, bench.PLIES))
        except wc.SolveError as e:
            assert e.code == 3
    assert roots == kept

