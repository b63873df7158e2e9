"""The tensor-core network paths against the fp32 network path.

Same trees, same CFR schedule; only the network arithmetic differs (16-bit
operands with fp32 accumulation on tcgen05, fast GELU). Two operand types:
  * f16, the default: the precision class of the reference GPU service's
    fast mode (cuBLAS COMPUTE_32F_FAST_16F, engine/src/gpu/device.rs:2306-2330);
  * bf16: the per-iteration chain (pooling, join layers, join output) on
    bf16 operands, the once-per-solve board trunk and the readout
    <f(c), h> on f16 operands (the readout multiplies operand error several
    times). Held to the same bars; the numbers it reaches are printed.

Checks (the bf16 value-net bar is "within 1e-2 relative, with the
exploitability of the small config reported"):
  * seeded He-normal weights, zero CFR iterations: root values (the uniform
    strategy's value of every leaf's network output) within 1e-2 relative,
    norm-wise per job;
  * the reference's tensor-core test weights (engine/src/gpu/tests.rs:34-48,
    393-444): root values within 1e-2 absolute plus 2e-3 relative; every
    strategy row a distribution;
  * exploitability: the oracle (fp32 network) measures the NashConv of the
    fast path's average strategy, which must stay within 5% of the NashConv
    of the exact path's strategy (measured: 1.5% worst for f16).
Per-cell strategy agreement is not a bar here: with random weights sibling
actions get near-equal values, regrets are differences of those, and
independent per-row rounding of ~3e-4 reorders them (a coherent 5e-4 weight
perturbation of the exact network moves strategies 10x less).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# per operand type: (relative root-value bar, absolute root-value bar,
# relative NashConv excess bar)
BARS = {"f16": (1e-2, 1e-2, 0.05), "bf16": (1e-2, 1e-2, 0.05)}


@pytest.fixture(scope="module")
def he_weights(wc):
    return wc.seeded_weights("he", 0)


@pytest.fixture(scope="module")
def test_weights(wc):
    return wc.seeded_weights("test", 0xD15EA5E)


def solve(wc, weights, net, jobs):
    c = wc.spawn(0, *weights, net=net)
    try:
        return c.solve_batch(jobs)
    finally:
        c.close()


@pytest.mark.parametrize("net", ["f16", "bf16"])
def test_tensor_network_values_at_the_uniform_strategy(wc, he_weights, net):
    cfg = wc.Cfg(depth=2, iters=0, snapshots=False, cfr=wc.Cfr.PLUS)
    jobs = [wc.PackedJob.from_root(wc.generate_root(s), cfg) for s in range(6)]
    exact, fast = solve(wc, he_weights, "exact", jobs), solve(wc, he_weights, net, jobs)
    worst = 0.0
    for e, f in zip(exact, fast):
        a = np.concatenate(e.root_values[0])
        b = np.concatenate(f.root_values[0])
        worst = max(worst, float(np.linalg.norm(a - b) / max(np.linalg.norm(a), 1e-30)))
    print(f"{net}: worst relative root-value error {worst:.3e}")
    assert worst <= BARS[net][0]


@pytest.mark.parametrize("net", ["f16", "bf16"])
@pytest.mark.parametrize("depth,iters,rule", [(2, 8, "LINEAR"), (3, 16, "PLUS")])
def test_tensor_network_tracks_exact_math(wc, test_weights, net, depth, iters, rule):
    cfg = wc.Cfg(depth=depth, iters=iters, snapshots=False, cfr=getattr(wc.Cfr, rule))
    jobs = [wc.PackedJob.from_root(wc.generate_root(s), cfg) for s in range(4)]
    exact, fast = solve(wc, test_weights, "exact", jobs), solve(wc, test_weights, net, jobs)
    _, abs_bar, _ = BARS[net]
    for e, f in zip(exact, fast):
        a, b = np.concatenate(e.root_values[0]), np.concatenate(f.root_values[0])
        np.testing.assert_allclose(b, a, rtol=2e-3, atol=abs_bar)
        assert np.all(f.strategy >= -2e-6) and np.all(f.strategy <= 1 + 2e-6)
        print(f"{net} depth {depth}: mean |strategy diff| {np.abs(f.strategy - e.strategy).mean():.2e}")


@pytest.mark.parametrize("net", ["f16", "bf16"])
@pytest.mark.parametrize("kind", ["test", "he"])
def test_tensor_network_exploitability(wc, oracle, he_weights, test_weights, net, kind):
    weights = test_weights if kind == "test" else he_weights
    cfg = wc.Cfg(depth=2, iters=8, snapshots=False, cfr=wc.Cfr.LINEAR)
    roots = [wc.generate_root(s) for s in range(4)]
    jobs = [wc.PackedJob.from_root(r, cfg) for r in roots]
    exact, fast = solve(wc, weights, "exact", jobs), solve(wc, weights, net, jobs)
    for r, e, f in zip(roots, exact, fast):
        o = oracle.Oracle(r, cfg, weights)
        o.set_strategy(e.strategy)
        nc_exact = o.nash_conv()[0]
        o.set_strategy(f.strategy)
        nc_fast = o.nash_conv()[0]
        print(f"{net} {kind}: NashConv exact {nc_exact:.4e}, {net} {nc_fast:.4e}")
        assert nc_fast <= nc_exact * (1 + BARS[net][2])
