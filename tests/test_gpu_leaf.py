"""Leaf evaluation alone (value-net leaf inference).

Every network row of seeded depth-2/3 trees is valued at the initial
(uniform-strategy) reaches, through the C ABI:
  * fp32 network path: bit-identical to the CPU oracle's leaf_values
    (engine/src/search.rs:1550-1636 with net.rs);
  * tensor-core path: within 1e-2 relative to the fp32 values, norm-wise
    (||v_fast - v_fp32|| / ||v_fp32|| per job and traverser), the bf16 bar
    of the north_star, for both operand types (f16 measured 1.9e-3 worst;
    bf16 runs the per-iteration chain on bf16 operands and the trunk and
    the readout on f16, since bf16 everywhere measured 1.9e-2). The
    readout <f(c), h> of a random-weight
    network is nearly orthogonal (median |cos| 0.02-0.08), so the relative
    error of a value is several times the relative error of h; the largest
    single deviation relative to the job's largest value is printed beside it.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def weights(wc):
    return wc.seeded_weights("he", 0)


def leaf_values(wc, client, jobs, p):
    batch = client.upload(jobs)
    batch.leaf_values(p)
    out = [batch.leaf_values_of(j, p) for j in range(len(jobs))]
    batch.free()
    return out


@pytest.mark.parametrize("depth,seeds", [(2, [0, 1, 2]), (3, [0])])
def test_precise_leaf_values_are_bit_exact(wc, oracle, weights, depth, seeds):
    cfg = wc.Cfg(depth=depth, iters=4, snapshots=False, cfr=wc.Cfr.PLUS)
    roots = [wc.generate_root(s) for s in seeds]
    jobs = [wc.PackedJob.from_root(r, cfg) for r in roots]
    client = wc.spawn(0, *weights, precise=True)
    try:
        got = [leaf_values(wc, client, jobs, p) for p in (0, 1)]
        for k, r in enumerate(roots):
            o = oracle.Oracle(r, cfg, weights)
            for p in (0, 1):
                np.testing.assert_array_equal(got[p][k], o.leaf_values(p))
    finally:
        client.close()


@pytest.mark.parametrize("net,bar", [("f16", 1e-2), ("bf16", 1e-2)])
def test_tensor_leaf_values_within_bar(wc, weights, net, bar):
    cfg = wc.Cfg(depth=3, iters=4, snapshots=False, cfr=wc.Cfr.PLUS)
    jobs = [wc.PackedJob.from_root(wc.generate_root(s), cfg) for s in range(4)]
    exact = wc.spawn(0, *weights, net="exact")
    fast = wc.spawn(0, *weights, net=net)
    try:
        worst = 0.0
        for p in (0, 1):
            a = leaf_values(wc, exact, jobs, p)
            b = leaf_values(wc, fast, jobs, p)
            for x, y in zip(a, b):
                rel = float(np.linalg.norm(x - y) / max(np.linalg.norm(x), 1e-30))
                worst = max(worst, rel)
                mx = float(np.abs(x - y).max() / max(np.abs(x).max(), 1e-30))
                print(f"{net} p{p}: {x.size} values, norm-wise rel err {rel:.3e}, max dev / max |v| {mx:.3e}")
        assert worst <= bar, worst
    finally:
        exact.close()
        fast.close()


@pytest.mark.parametrize("net", ["f16", "bf16"])
def test_board_rows_of_shared_public_rows(wc, oracle, weights, net):
    """The tensor-core board trunk runs once per distinct public row of a job
    and the other rows take that row's P and jp (k_board_dup). Every row's
    stored board pieces must still be its own: P (stored as P + bout minus
    the row mean) against the oracle's fp32 P (engine/src/net.rs:558-731)
    up to the column offset bout, and jp (stored minus its row mean) against
    the oracle's jp, per row within 5e-2 of the row's norm (a row given
    another row's pieces is off by about its whole norm); rows with the same
    public bytes hold bit-identical pieces."""
    cfg = wc.Cfg(depth=2, iters=4, snapshots=False, cfr=wc.Cfr.PLUS)
    roots = [wc.generate_root(s) for s in (1, 2, 4)]
    jobs = [wc.PackedJob.from_root(r, cfg) for r in roots]
    assert sum(int(j.counts()[20]) < j.info["net_rows"] for j in jobs) >= 2
    client = wc.spawn(0, *weights, net=net)
    try:
        batch = client.upload(jobs)
        batch.leaf_values(0)
        got = [batch.board_rows(j) for j in range(len(jobs))]
        batch.free()
    finally:
        client.close()
    for k, r in enumerate(roots):
        pb_o, jp_o, _, _ = oracle.Oracle(r, cfg, weights).net_pieces()
        pb_f, jp_f = got[k]
        pc = pb_o - pb_o.mean(axis=1, keepdims=True)
        d = pb_f - pc
        d -= d.mean(axis=0, keepdims=True)  # the common offset: bout minus its mean
        p_err = np.linalg.norm(d, axis=1) / np.linalg.norm(pc, axis=1)
        jc = jp_o - jp_o.mean(axis=1, keepdims=True)
        j_err = np.linalg.norm(jp_f - jc, axis=1) / np.linalg.norm(jc, axis=1)
        print(f"{net} root {k}: {pb_o.shape[0]} rows, {int(jobs[k].counts()[20])} distinct, worst row error "
              f"P {p_err.max():.2e} jp {j_err.max():.2e}")
        assert p_err.max() <= 5e-2 and j_err.max() <= 5e-2
        _, first, inverse = np.unique(pb_o.view(np.uint32), axis=0, return_index=True, return_inverse=True)
        rep = first[inverse.ravel()]
        np.testing.assert_array_equal(pb_f, pb_f[rep])
        np.testing.assert_array_equal(jp_f, jp_f[rep])
