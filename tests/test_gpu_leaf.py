"""Leaf evaluation alone (value-net leaf inference).

Every network row of seeded depth-2/3 trees is valued at the initial
(uniform-strategy) reaches, through the C ABI:
  * fp32 network path: bit-identical to the CPU oracle's leaf_values
    (engine/src/search.rs:1550-1636 with net.rs);
  * tensor-core path: within 1e-2 relative to the fp32 values, norm-wise
    (||v_fast - v_fp32|| / ||v_fp32|| per job and traverser) with f16
    operands (measured: 1.9e-3 worst); bf16 operands get a 4e-2 bar
    (measured: 1.9e-2 worst). The readout <f(c), h> of a random-weight
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


@pytest.mark.parametrize("net,bar", [("f16", 1e-2), ("bf16", 4e-2)])
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
