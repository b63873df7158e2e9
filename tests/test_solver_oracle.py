"""The oracle solver against the reference's solver tests (CPU).

  * engine/tests/rebel_solver.rs:167-289 — on micro endgames whose whole
    remaining game fits in the subgame, every regret rule (linear, plus,
    dcfr, pcfr, sapcfr) lands within 0.03 of the tabular-CFR game value, the
    two root values cancel within 0.02, and NashConv is non-negative and
    falls between iteration 2 and 500;
  * engine/tests/rebel_solver.rs:576-600 — the kept iterations are 0, the
    powers of two and the final one, increasing; the job image keeps the same
    list (one carry block per kept snapshot but the last).
"""
import numpy as np
import pytest


def test_subgame_solver_matches_tabular_cfr_on_micro_endgames(wc, oracle):
    checked = 0
    for seed in range(3000):
        root = oracle.micro_root(seed, 60 + seed % 120, 3)
        if root is None:
            continue
        probe = oracle.Oracle(root, wc.Cfg(depth=8, iters=500, snapshots=True, cfr=wc.Cfr.LINEAR))
        if probe.nc0 * probe.nc1 > 64:
            continue
        assert probe.shape["all_terminal"] == 1, "the whole remaining game must fit inside the subgame"
        if probe.shape["nodes"] > 8000 or oracle.lib().oracle_solver_outcomes(probe.h) < 2:
            continue
        nc0, nc1 = probe.nc0, probe.nc1
        del probe
        exact = oracle.tabular_value(root, 100)
        bel = np.concatenate([np.full(nc0, 1.0 / nc0), np.full(nc1, 1.0 / nc1)]).astype(np.float32)
        for name, rule in wc.Cfr.NAMED.items():
            sv = oracle.Oracle(root, wc.Cfg(depth=8, iters=500, snapshots=True, cfr=rule))
            sv.multistep(2)
            early = sv.nash_conv()[0]
            sv.multistep(498)
            late = sv.nash_conv()[0]
            vals = sv.value_under(bel[None, :])[0]
            v0 = float(np.dot(bel[:nc0], vals[:nc0]))
            v1 = float(np.dot(bel[nc0:], vals[nc0:]))
            print(f"seed {seed} {name}: value {v0:+.4f} (exact {exact:+.4f}) zero-sum {v0 + v1:+.4f} "
                  f"NashConv {early:.4f} -> {late:.4f}")
            assert abs(v0 + v1) < 0.02, (seed, name, v0, v1)
            assert abs(v0 - exact) < 0.03, (seed, name, v0, exact)
            assert late > -1e-3, (seed, name, late)
            assert late < max(early, 1e-3), (seed, name, early, late)
        checked += 1
        if checked >= 4:
            break
    assert checked >= 4


@pytest.mark.parametrize("iters", [1, 2, 8, 64, 512])
def test_snapshot_iterations_are_log_spaced_plus_final(wc, iters):
    v = wc.snapshot_iters(iters)
    assert v[0] == 0 and v[-1] == iters
    assert v == [t for t in range(iters + 1) if t == 0 or (t & (t - 1)) == 0 or t == iters]
    assert all(a < b for a, b in zip(v, v[1:]))


def test_job_keeps_the_snapshot_list(wc):
    root = wc.generate_root(0)
    for iters in (1, 8, 64):
        job = wc.PackedJob.from_root(root, wc.Cfg(depth=1, iters=iters, snapshots=True, cfr=wc.Cfr.PLUS))
        assert job.info["carry_snapshots"] == len(wc.snapshot_iters(iters)) - 1


# ---- structural tests of the tree, restated from engine/tests/rebel_solver.rs
# (oracle/solver_checks.cpp drives the host tree builder and the CPU solver)

def _check(fn, *args):
    import ctypes as C

    msg = C.create_string_buffer(2048)
    rc = fn(*args, msg, 2048)
    assert rc == 0, msg.value.decode()


def test_draw_pass_through_consistency(oracle):  # rebel_solver.rs:449
    import ctypes as C

    st = (C.c_int * 5)()
    _check(oracle.lib().oracle_check_draw_pass_through, st)
    print(f"draw pass-through: rejected={st[0]} built={st[1]} toolarge={st[2]} nochance={st[3]} solved={st[4]}")


def test_warrior_priest_draw_walks_through_the_tree(oracle):  # rebel_solver.rs:612
    _check(oracle.lib().oracle_check_warrior_priest_draw_walk)


def test_depth_is_spent_on_coin_plays_not_micro_choices(oracle):  # rebel_solver.rs:753
    _check(oracle.lib().oracle_check_depth_counts_coin_plays)
