"""CUDA batch solves against the CPU oracle, through the C ABI.

Fixtures follow the reference's GPU tests (engine/src/gpu/tests.rs:17-118):
seeded solve-site roots, a few CFR iterations with snapshots, three skewed
carried roots (tests.rs:56-70), and the test weight blob (tests.rs:34-48).
Every CFR rule of search.rs:133-185 runs (linear, plus, dcfr, and the
predictive pcfr / sapcfr, whose regret-matching step adds predict x delta).
Tolerances:
  * no network / zero network: bit-exact strategies, root values and carries
    (the kernels keep the oracle's operation order and rounding);
  * fp32 network ("precise"): bit-exact as well — the kernels keep the
    oracle's sequential GEMM order and share its deterministic tanh.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SEEDS = [0, 1, 2, 3]


def skew(live, n0, i):
    """tests.rs:56-70: add 0.5 to every (i + 2)-th weight, renormalise."""
    out = []
    for v in (live[:n0], live[n0:]):
        x = np.array([p + (0.5 if c % (i + 2) == 0 else 0.0) for c, p in enumerate(v)], np.float32)
        out.append(x / x.sum())
    return np.concatenate(out)


def roots_for(wc, seeds, plies=20):
    return [wc.generate_root(s, plies) for s in seeds]


def solve_and_compare(wc, oracle, client, roots, cfg, weights, exact, strat_tol=1e-4, root_tol=1e-3,
                      carry_tol=6e-4, ncarried=3):
    built = []
    for root in roots:
        live_job = wc.PackedJob.from_root(root, cfg)
        live = live_job.root_belief()
        n0 = live_job.info["root_nc0"]
        carried = np.stack([skew(live, n0, k) for k in range(ncarried)])
        built.append((wc.PackedJob.from_root(root, cfg, carried), carried, root))
    results = client.solve_batch([b[0] for b in built])
    worst = {"strategy": 0.0, "roots": 0.0, "carries": 0.0}
    for (job, carried, root), res in zip(built, results):
        o = oracle.Oracle(root, cfg, weights)
        assert o.shape["cells"] == job.info["cells"] and o.shape["nodes"] == job.info["nodes"]
        o.multistep(cfg.iters)
        want_strat = o.snapshot(-1)
        want_roots = o.value_under(carried)
        got_roots = np.stack([np.concatenate(rv) for rv in res.root_values])
        if exact:
            np.testing.assert_array_equal(res.strategy, want_strat)
            np.testing.assert_array_equal(got_roots, want_roots)
        else:
            np.testing.assert_allclose(res.strategy, want_strat, rtol=0, atol=strat_tol)
            np.testing.assert_allclose(got_roots, want_roots, rtol=0, atol=root_tol)
        worst["strategy"] = max(worst["strategy"], float(np.abs(res.strategy - want_strat).max()))
        worst["roots"] = max(worst["roots"], float(np.abs(got_roots - want_roots).max()))
        if cfg.snapshots:
            offs, exits = job.carry_layout()
            assert res.carries.shape == (o.nsnaps() - 1, offs[-1])
            for e in sorted({0, len(exits) // 2, len(exits) - 1}):
                want = o.carried_beliefs(int(exits[e]), int(offs[e + 1] - offs[e]))
                got = res.carries[:, offs[e]:offs[e + 1]].astype(np.float32)
                if exact:
                    np.testing.assert_array_equal(got, want.astype(np.float16).astype(np.float32))
                else:
                    np.testing.assert_allclose(got, want, rtol=0, atol=carry_tol)
                worst["carries"] = max(worst["carries"], float(np.abs(got - want).max()))
        # every probability row sums to 1 inside [-2e-6, 1 + 2e-6] (tests.rs:147-172)
        assert np.all(res.strategy >= -2e-6) and np.all(res.strategy <= 1 + 2e-6)
    print("worst abs error", worst)
    return worst


@pytest.fixture(scope="module")
def client_nonet(wc):
    c = wc.spawn(0)
    yield c
    c.close()


@pytest.mark.parametrize("rule", ["plus", "linear", "dcfr", "pcfr", "sapcfr"])
def test_no_network_bit_exact(wc, oracle, client_nonet, rule):
    cfg = wc.Cfg(depth=2, iters=16, snapshots=True, cfr=wc.Cfr.NAMED[rule])
    solve_and_compare(wc, oracle, client_nonet, roots_for(wc, SEEDS), cfg, None, exact=True)


def test_no_network_depth3_bit_exact(wc, oracle, client_nonet):
    cfg = wc.Cfg(depth=3, iters=32, snapshots=False, cfr=wc.Cfr.PLUS)
    solve_and_compare(wc, oracle, client_nonet, roots_for(wc, [0, 3]), cfg, None, exact=True)


def test_zero_network_bit_exact(wc, oracle):
    dims, w, b, ln = wc.seeded_weights("test", 0xD15EA5E)
    w[:] = 0
    client = wc.spawn(0, dims, w, b, ln, precise=True)
    try:
        cfg = wc.Cfg(depth=2, iters=8, snapshots=True, cfr=wc.Cfr.LINEAR)
        solve_and_compare(wc, oracle, client, roots_for(wc, SEEDS[:2]), cfg, (dims, w, b, ln), exact=True)
    finally:
        client.close()


@pytest.mark.parametrize("rule", ["linear", "plus", "dcfr", "pcfr", "sapcfr"])
def test_precise_network_parity(wc, oracle, rule):
    weights = wc.seeded_weights("test", 0xD15EA5E)
    client = wc.spawn(0, *weights, precise=True)
    try:
        cfg = wc.Cfg(depth=2, iters=8, snapshots=True, cfr=wc.Cfr.NAMED[rule])
        solve_and_compare(wc, oracle, client, roots_for(wc, SEEDS), cfg, weights, exact=True)
    finally:
        client.close()


def test_batch_composition_is_exact(wc, client_nonet):
    """A tree alone and beside 15 others solves identically (tests.rs:328)."""
    cfg = wc.Cfg(depth=2, iters=16, snapshots=False, cfr=wc.Cfr.PLUS)
    jobs = [wc.PackedJob.from_root(r, cfg) for r in roots_for(wc, range(16))]
    together = client_nonet.solve_batch(jobs)
    for i in [0, 7, 15]:
        alone = client_nonet.solve_batch([jobs[i]])[0]
        np.testing.assert_array_equal(alone.strategy, together[i].strategy)
        np.testing.assert_array_equal(np.concatenate(alone.root_values[0]),
                                      np.concatenate(together[i].root_values[0]))


def test_submit_wait_matches_batch(wc, client_nonet):
    cfg = wc.Cfg(depth=2, iters=8, snapshots=False, cfr=wc.Cfr.PLUS)
    jobs = [wc.PackedJob.from_root(r, cfg) for r in roots_for(wc, range(4))]
    handles = [client_nonet.submit(j) for j in jobs]
    got = [h.wait() for h in handles]
    want = client_nonet.solve_batch(jobs)
    for g, w in zip(got, want):
        np.testing.assert_array_equal(g.strategy, w.strategy)


def test_memory_bounded_waves_match_one_batch(wc, monkeypatch):
    """wc_solve_batch in waves (WC_WAVE_BYTES forces several; each wave's
    upload overlaps the previous wave's solve, in two arenas reused across
    calls) gives, job for job, the results of one resident batch; the
    reference's route flags stay clear for jobs this small."""
    weights = wc.seeded_weights("test", 0xD15EA5E)
    cfg = wc.Cfg(depth=2, iters=8, snapshots=True, cfr=wc.Cfr.PLUS)
    jobs = [wc.PackedJob.from_root(r, cfg) for r in roots_for(wc, range(12))]
    ref = wc.spawn(0, *weights, net="f16")
    try:
        b = ref.upload(jobs)
        b.solve()
        want = [b.result(j) for j in range(len(jobs))]
        b.free()
    finally:
        ref.close()
    total = sum(j.info["table_bytes"] for j in jobs)
    monkeypatch.setenv("WC_WAVE_BYTES", str(max(1, 4 * total // 12)))  # a few jobs per wave
    c = wc.spawn(0, *weights, net="f16")
    try:
        for _ in range(2):  # the second call reuses the arenas
            got = c.solve_batch(jobs)
            for g, w in zip(got, want):
                np.testing.assert_array_equal(g.strategy, w.strategy)
                np.testing.assert_array_equal(np.concatenate(g.root_values[0]), np.concatenate(w.root_values[0]))
                np.testing.assert_array_equal(g.carries, w.carries)
                assert not g.oversize_route and not g.card_exclusive_route
    finally:
        c.close()
