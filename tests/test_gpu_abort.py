"""The tensor-core kernels' bounded waits, made to run out on purpose.

Every mbarrier wait in the tensor-core kernels (trunk, pooling, join, head)
is bounded by %globaltimer; when one gives up, the kernel takes a
block-uniform stop decision, issues nothing more, drains the copies and
products it had issued, releases its tensor memory and records a code that
the host reads after the solve. With the limit set to one nanosecond
(wc_debug_set_wait_limit) nearly every wait gives up at its first check,
while the copies and products it waits on still complete: the solve must
fail with the kernels' status (no fault), every drain must finish (codes
below 10), and the same context must then solve the same jobs exactly as
before once the limit is restored. No flag is left unset and nothing is
made to fault; the waits only stop early.
"""
import re

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_waits_that_give_up_leave_the_context_usable(wc):
    weights = wc.seeded_weights("he", 0)
    cfg = wc.Cfg(depth=2, iters=4, snapshots=False, cfr=wc.Cfr.PLUS)
    jobs = [wc.PackedJob.from_root(wc.generate_root(s), cfg) for s in range(4)]
    client = wc.spawn(0, *weights, net="f16")
    try:
        batch = client.upload(jobs)
        batch.solve()
        want = [batch.result(j).strategy for j in range(len(jobs))]
        wc._check(wc.lib().wc_debug_set_wait_limit(client._ctx, 1))
        with pytest.raises(wc.SolveError) as e:
            batch.solve()
        assert e.value.code == 2, e.value
        m = re.search(r"time limit \(code (\d+)", str(e.value))
        assert m, str(e.value)
        code = int(m.group(1))
        print(f"solve with 1 ns waits: {e.value}")
        assert 1 <= code <= 4, "in-flight work did not drain"
        wc._check(wc.lib().wc_debug_set_wait_limit(client._ctx, 0))
        batch.solve()
        for j in range(len(jobs)):
            np.testing.assert_array_equal(batch.result(j).strategy, want[j])
        batch.free()
    finally:
        client.close()
