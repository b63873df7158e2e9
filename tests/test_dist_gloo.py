"""The multi-GPU host logic on two CPU ranks (gloo, world size 2): the
bench's sharding (disjoint contiguous seed blocks, weak scaling), the
one-time weight broadcast from rank 0, and the max-over-ranks step time and
whole-job sums. The device path is the same code with the nccl backend."""
import os
import socket
import sys

import numpy as np
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    sys.path.insert(0, ROOT)
    import bench
    import warchest_b200 as wc

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        seeds = bench.seed_range(rank, 3)
        dims, w, b, ln = wc.seeded_weights("he", 0)
        mine = (dims, w, b, ln) if rank == 0 else (dims, np.zeros_like(w), np.zeros_like(b), np.zeros_like(ln))
        tw = bench.broadcast_weights(mine, "cpu")
        same = all(np.array_equal(t.numpy(), a) for t, a in zip(tw, (w, b, ln)))
        cfg = wc.Cfg(depth=1, iters=8, snapshots=False, cfr=wc.Cfr.PLUS)
        nodes = sum(wc.PackedJob.from_root(wc.generate_root(s), cfg).info["nodes"] for s in seeds)
        out.put((rank, seeds, same, nodes, bench.allsum(world, float(nodes)),
                 bench.max_over_ranks(world, float(rank + 1))))
        bench.barrier(world)
    finally:
        dist.destroy_process_group()


def test_two_rank_sharding_broadcast_and_reductions():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, s0, same0, n0, tot0, mx0), (r1, s1, same1, n1, tot1, mx1) = res
    assert s0 == [0, 1, 2] and s1 == [3, 4, 5]  # disjoint contiguous blocks
    assert same0 and same1  # rank 1 received rank 0's weights
    assert tot0 == tot1 == n0 + n1  # whole-job totals
    assert mx0 == mx1 == 2.0  # step time = max over ranks
