"""The reference's public-belief-state tests, restated: engine/tests/rebel_pbs.rs
(17 tests). Each test here names the reference test and line it restates; the
checks themselves are written in C++ over the host sources (oracle/
pbs_checks.cpp) because they drive the engine's internals (configs, beliefs,
draw transitions, features, the CPU solver) exactly as the Rust tests do.

`a_solve_reads_only_the_beliefs` is also checked on the product: the jobs the
product library builds from two worlds with the same public state and
beliefs must be identical byte for byte (wc_job_digest), so the GPU solve is
a function of the beliefs alone.
"""
import ctypes as C


def _run(fn, *args):
    msg = C.create_string_buffer(2048)
    rc = fn(*args, msg, 2048)
    assert rc == 0, msg.value.decode()


def test_features_do_not_leak_private_information(oracle):  # rebel_pbs.rs:165
    st = (C.c_int * 2)()
    _run(oracle.lib().oracle_check_features_do_not_leak, 0, st)
    print(f"{st[0]} positions checked")


def test_features_do_not_leak_private_information_random_draft(oracle):  # rebel_pbs.rs:171
    st = (C.c_int * 2)()
    _run(oracle.lib().oracle_check_features_do_not_leak, 1, st)
    print(f"{st[0]} positions checked, pending-maneuver mask fired in {st[1]}")


def test_belief_tracker_matches_brute_force(oracle):  # rebel_pbs.rs:198
    n = C.c_int()
    _run(oracle.lib().oracle_check_belief_tracker, 0, C.byref(n))
    print(f"{n.value} steps verified against exhaustive world enumeration")


def test_belief_tracker_matches_brute_force_with_warrior_priests(oracle):  # rebel_pbs.rs:215
    n = C.c_int()
    _run(oracle.lib().oracle_check_belief_tracker, 1, C.byref(n))
    print(f"{n.value} steps verified (Warrior Priest draft)")


def test_config_key_packing_has_headroom(oracle):  # rebel_pbs.rs:418
    _run(oracle.lib().oracle_check_config_key_headroom)


def test_reachable_config_census_with_warrior_priests(oracle):  # rebel_pbs.rs:464 (reported, not asserted)
    out = (C.c_uint64 * 4)()
    assert oracle.lib().oracle_check_config_census(out) == 0
    print(f"census: {out[3]} positions, median {out[0]} mean {out[1] / 10:.1f} p99 {out[2]}")
    assert out[3] > 0


def test_roots_round_trip(oracle):  # rebel_pbs.rs:501
    n = C.c_int()
    _run(oracle.lib().oracle_check_roots_round_trip, C.byref(n))
    assert n.value > 0


def test_packed_row_expands_to_the_same_features(oracle):  # rebel_pbs.rs:551
    n = C.c_int()
    _run(oracle.lib().oracle_check_packed_row_expands, C.byref(n))


def test_config_features_separate_every_config(oracle):  # rebel_pbs.rs:586
    n = C.c_int()
    _run(oracle.lib().oracle_check_config_features_separate, C.byref(n))


def test_a_subgame_of_only_terminal_leaves_solves(oracle):  # rebel_pbs.rs:640
    n = C.c_int()
    _run(oracle.lib().oracle_check_terminal_leaf_subgame, C.byref(n))


def test_card_features_separate_every_draftable_unit(oracle):  # rebel_pbs.rs:697
    _run(oracle.lib().oracle_check_card_features_separate)


def test_config_counts_are_hand_facedown_bag(oracle):  # rebel_pbs.rs:732
    _run(oracle.lib().oracle_check_config_counts)


def test_a_solve_reads_only_the_beliefs(oracle):  # rebel_pbs.rs:771
    n = C.c_int()
    _run(oracle.lib().oracle_check_solve_reads_only_beliefs, C.byref(n))
    print(f"{n.value} positions solved bit-identically in two worlds")


def test_product_jobs_read_only_the_beliefs(oracle, wc):
    """rebel_pbs.rs:771 for the product: the job tables built from the two
    worlds are identical, so every solve of them is too."""
    L = oracle.lib()
    checked = 0
    for seed in range(1, 80):
        b0, b1 = C.create_string_buffer(1 << 20), C.create_string_buffer(1 << 20)
        n0, n1 = C.c_size_t(), C.c_size_t()
        if L.oracle_ambiguous_worlds(C.c_uint64(seed), b0, b1, C.c_size_t(1 << 20), C.byref(n0), C.byref(n1)):
            continue
        cfg = wc.Cfg(depth=2, iters=8, snapshots=True)
        r0, r1 = b0.raw[: n0.value], b1.raw[: n1.value]
        assert r0 != r1, "the two worlds should differ in their hidden coins"
        j0, j1 = wc.PackedJob.from_root(r0, cfg), wc.PackedJob.from_root(r1, cfg)
        assert j0.digest == j1.digest, f"seed {seed}: the job moved with the true world"
        checked += 1
    assert checked > 20, f"only {checked} positions exercised"


def test_the_value_function_separates_configs_sharing_a_hand(oracle):  # rebel_pbs.rs:831
    st = (C.c_int * 3)()
    _run(oracle.lib().oracle_check_value_separates_configs, st)
    print(f"{st[0]} same-hand pairs: values differ in {st[1]}, strategies in {st[2]}")


def test_normalized_weights_match_belief_normalize(oracle):  # rebel_pbs.rs:898
    n = C.c_int()
    _run(oracle.lib().oracle_check_normalized_weights, C.byref(n))


def test_from_pairs_keeps_zero_weight_configs(oracle):  # rebel_pbs.rs:929
    _run(oracle.lib().oracle_check_from_pairs_keeps_zero_weight)


def test_zero_weight_config_survives_the_walk_update(oracle):  # rebel_pbs.rs:960
    _run(oracle.lib().oracle_check_zero_weight_walk_update)
