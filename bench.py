"""Benchmark: batched depth-limited CFR+ solves with value-network leaves.

Workload: per GPU, 4096 independent subgames whose
roots are seeded solve sites (seeded draft, 20 uniform decisions, on to the
next MainPlay; seeds rank*4096 .. rank*4096+4095), depth 3, 512 CFR+
iterations, the v5 value network at every iteration, Phase 2 on the live
root belief. One step = one full batched solve of that batch: per-solve
network pieces, init, 512 iterations, the average strategy, root values.

Metric: CFR node-updates/s = sum over subgames of public nodes x iterations,
divided by the device time of the step (CUDA events on the solver's stream,
max over ranks). Whole-job value = all ranks' node-updates / that time.
Weak scaling: every rank solves its own 4096 subgames; the value-net weights
are broadcast once from rank 0 over NCCL; there is no per-iteration
collective.

--impl reference times the CPU restatement of the reference solver (the
oracle under oracle/, the reference's own Rust cannot be built here) on a
bounded sample of the same workload with every host thread.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "war-chest-bot-9000-_b200"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

METRIC = "CFR node-updates/sec"
UNIT = "node-updates/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--subgames", type=int, default=4096, help="subgames per GPU")
    ap.add_argument("--subgames-total", type=int, default=0,
                    help="configs[3]: this many subgames split over the ranks (strong scaling), each rank's shard "
                         "solved through wc_solve_batch's memory-bounded waves; a separate line, not the bench line")
    ap.add_argument("--depth", type=int, default=3)
    ap.add_argument("--iters", type=int, default=512)
    ap.add_argument("--plies", type=int, default=20)
    ap.add_argument("--net", default="bf16", choices=["bf16", "f16", "exact", "none"],
                    help="value network: tcgen05 with bf16 operands for the per-iteration chain (trunk and "
                         "readout f16), f16 operands throughout, fp32 exact, or none")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline leg (profiling runs)")
    ap.add_argument("--build-threads", type=int, default=0)
    ap.add_argument("--games", type=int, default=64, help="--workload resolve: games (belief-heavy roots)")
    ap.add_argument("--workload", default="solve", choices=["solve", "leaf", "batch", "resolve"],
                    help="solve: the configs[2] batched solve (the bench line); leaf: configs[1], value-net leaf "
                         "inference alone at 1K / 16K / 256K rows; batch: the training-batch expansion of replay "
                         "rows at 1K / 256K rows (one JSON line per batch size, not bench lines); resolve: "
                         "configs[4]'s continual re-solving loop (8 solves per game) at --depth / --iters")
    return ap.parse_args()


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        # short: ranks that wait on a missing peer end with an error; the longest
        # legitimate gap between collectives is the warm-up solves (~2 min)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def cfr_plus(wc):
    return wc.Cfr.PLUS


def build_jobs(wc, seeds, cfg, threads):
    """Seeded roots on host threads (the C calls release the GIL), then the
    jobs by the library's parallel builder (wc_job_build_batch: native
    threads, roots taken from a shared queue). Roots whose tree hits the node
    cap are counted and skipped, as the reference's tape builder does
    (wave_tape.rs:51-56)."""
    roots = [None] * len(seeds)

    def work(lo, hi):
        for i in range(lo, hi):
            roots[i] = wc.generate_root(seeds[i], PLIES)

    n = len(seeds)
    th = [threading.Thread(target=work, args=(n * k // threads, n * (k + 1) // threads)) for k in range(threads)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    jobs = wc.PackedJob.build_many(roots, cfg, threads=threads)
    keep = [i for i in range(n) if jobs[i] is not None]
    return [roots[i] for i in keep], [jobs[i] for i in keep]


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = os.path.join(tempfile.gettempdir(), f"wcb200_clocks_{os.getpid()}_{index}.csv")

    def start(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        self.proc.wait()
        self.f.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons)}


def algorithmic_work(jobs):
    """Per kernel class, the work one solve must do (every value read or
    written once; indices u32): HBM bytes for the CFR and pooling kernels,
    tensor FLOPs for the network kernels. Per unit:
      rows     24 B per legal cell (regret R/W, current W, child value, index) + 8 B per row
      vgather  12 B per entry (index, weight, source value) + 8 B per output
      reach    24 B per cell entry, 16 B per draw entry, 8 B per output
      pool     8 B per leaf-config entry (reach, column) + 128 B per row (the f16 pooled atom)
      join     4 x 2*128*128 FLOP per network row
      head     2*128*256 FLOP per network row + 2*256 per leaf-config entry of the traverser
      trunk    17.0 MFLOP per distinct public row of a job (once per solve; rows
               that repeat a public row share its board pieces, so the work
               the solve must do is per distinct row)
    CFR classes run once per iteration for one player, so a solve does each
    player's share iters/2 times; the leaf classes run once per iteration and
    twice per carried root in Phase 2."""
    c = np.sum([j.counts() for j in jobs], axis=0).astype(np.float64)
    iters = jobs[0].cfg.iters
    pairs = iters / 2.0
    rows = sum(j.info["net_rows"] for j in jobs)
    carried = max(max(j.info["ncarried"], 1) for j in jobs)
    calls = iters + 2 * carried
    entries = (c[14] + c[15]) / 2.0  # leaf-config entries per call (players alternate)
    return {
        "rows": ("hbm", (24 * (c[0] + c[1]) + 8 * (c[2] + c[3])) * pairs),
        "vgather": ("hbm", (12 * (c[4] + c[5]) + 8 * (c[6] + c[7])) * pairs),
        "reach": ("hbm", (24 * (c[8] + c[9]) + 16 * (c[10] + c[11]) + 8 * (c[12] + c[13])) * pairs),
        "pool": ("hbm", (8 * entries + 128 * rows) * calls),
        "join": ("tensor", 4 * 2 * 128 * 128 * rows * calls),
        "head": ("tensor", (2 * 128 * 256 * rows + 2 * 256 * entries) * calls),
        "trunk": ("tensor", 17.0e6 * c[20]),
    }


def peaks():
    """Measured HBM GB/s and bf16 TFLOP/s of this pool's B200s: the burst
    figure for a kernel timed alone, the sustained one for kernels timed
    inside a long step (the classes here are timed inside whole solves)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p.get("bf16_tflops_sustained", p["bf16_tflops"]), "measured (tensor: sustained)"
    except Exception:
        return 6650.0, 1400.0, "fallback"


def rooflines(prof, work):
    """Achieved rate and fraction of peak per kernel class, from the
    per-class CUDA-event times of the timed solves."""
    hbm, tflops, src = peaks()
    out = {}
    for k, (bound, amount) in work.items():
        ms = prof.get(k, 0.0)
        if ms <= 0:
            continue
        if bound == "hbm":
            a = amount / (ms / 1e3) / 1e9
            out[k] = {"bound": "hbm", "achieved": a, "peak": hbm, "unit": "GB/s", "frac": a / hbm, "ms": ms}
        else:
            a = amount / (ms / 1e3) / 1e12
            out[k] = {"bound": "tensor", "achieved": a, "peak": tflops, "unit": "TFLOP/s", "frac": a / tflops, "ms": ms}
    return out, src


def cpu_sample_roots(oracle, cfg, seeds, threads):
    """The bounded CPU sample: among the first 4 x threads workload seeds,
    the `threads` roots whose trees have the median number of network rows
    (one per host thread; the per-subgame rate barely depends on size, and a
    median-sized depth-3 solve's network setup takes ~30 s on one core).
    Tree sizes come from the oracle's own builder."""
    import ctypes as C

    cand = seeds[: 4 * threads]
    roots = []
    for s in cand:
        buf = C.create_string_buffer(1 << 20)
        n = C.c_size_t()
        if oracle.lib().oracle_root_generate(C.c_uint64(s), PLIES, 1, buf, C.c_size_t(1 << 20), C.byref(n)) != 0:
            raise RuntimeError("root generation failed")
        roots.append(buf.raw[: n.value])
    sizes = [0] * len(cand)

    def size(lo, hi):
        for i in range(lo, hi):
            try:
                sizes[i] = oracle.Oracle(roots[i], cfg).shape["net_rows"]
            except RuntimeError:  # node cap: skipped like the GPU workload
                sizes[i] = -1

    th = [threading.Thread(target=size, args=(len(cand) * k // threads, len(cand) * (k + 1) // threads))
          for k in range(threads)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    ok = [i for i in range(len(cand)) if sizes[i] >= 0]
    med = sorted(sizes[i] for i in ok)[len(ok) // 2]
    pick = sorted(ok, key=lambda i: (abs(sizes[i] - med), i))[:threads]
    return [roots[i] for i in pick], [cand[i] for i in pick], [sizes[i] for i in pick]


def cpu_baseline(oracle, cfg, weights, seeds):
    """The oracle (CPU restatement of the reference solver) on a bounded
    sample of the workload, one subgame per host thread: each thread times
    its solver build, the per-solve network and 2 CFR+ iterations, then 4
    more iterations, and extrapolates its full solve (oracle_bench); the rate
    is the sum of the threads' node-updates/s."""
    threads = os.cpu_count() or 1
    roots, picked, sizes = cpu_sample_roots(oracle, cfg, seeds, threads)
    rate, wall, m = oracle.bench(roots, cfg, weights, threads, 2, 4)
    return {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{m} workload subgames (seeds {min(picked)}..{max(picked)}, the median network-row count "
                      f"{sorted(sizes)[len(sizes) // 2]} of the first {4 * threads} seeds), one per thread: build + "
                      f"network + 2 CFR+ iterations and 4 more timed, each {cfg.iters}-iteration solve "
                      f"extrapolated; {wall:.1f} s wall"}


def batch_workload(args):
    """The training batch (train/gpu_batch.py make_batch): replay rows packed
    from seeded positions (0-60 plies, the distinct rows repeated to the batch
    size), 1-4 configs per (row, seat) with seeded counts. Device: CUDA events
    around wc_replay_expand on torch's stream, inputs already on the device,
    L2 flushed (a 256 MB write) before each timed call; e2e adds the host to
    device copies of the compact arrays (make_batch as a trainer calls it).
    Algorithmic bytes: the row (215 B) and both views' features (2 x 897 x
    4 B) per row, 15 B of counts in and 60 B of phi out per config, each
    config's span id (8 B). CPU: the oracle's restatement of the CPU batch
    (train/train.py:249-270) on one thread, on the 1K batch."""
    import ctypes as Cc

    import torch

    import oracle_lib
    import warchest_b200 as wc
    from warchest_b200 import gpu_batch

    hbm, _, src = peaks()
    dev = torch.device("cuda:0")
    distinct = []
    for s in range(512):
        try:
            distinct.append(np.frombuffer(wc.pack_row(wc.generate_root(s, plies=int(s % 61))), np.uint8))
        except wc.SolveError:
            pass
    distinct = np.stack(distinct)
    gpu_batch.warmup(dev)
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)
    for n in (1024, 262144):
        rng = np.random.default_rng(n)
        rows = distinct[rng.integers(0, len(distinct), n)]
        seg = np.repeat(np.arange(2 * n, dtype=np.int64), rng.integers(1, 5, 2 * n))
        m = len(seg)
        cc = rng.integers(0, 4, (m, 15)).astype(np.uint8)
        parts = (rows, np.zeros((n, 10), np.uint8), cc, (seg % 2).astype(np.uint8), np.ones(m, np.float32),
                 np.zeros(m, np.float32), seg)
        rows_t = torch.as_tensor(rows, device=dev)
        cc_t = torch.as_tensor(cc, device=dev)
        seg_t = torch.as_tensor(seg, device=dev)
        x = torch.empty((2 * n, wc.PUBFEAT), dtype=torch.float32, device=dev)
        phi = torch.empty((m, 15), dtype=torch.float32, device=dev)
        stream = torch.cuda.current_stream(dev)
        times, e2e = [], []
        for it in range(8):
            flush.fill_(float(it))
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            wc._check(wc.lib().wc_replay_expand(rows_t.data_ptr(), n, cc_t.data_ptr(), seg_t.data_ptr(), m,
                                                x.data_ptr(), phi.data_ptr(), stream.cuda_stream))
            b.record(stream)
            torch.cuda.synchronize(dev)
            if it >= 3:
                times.append(a.elapsed_time(b))
            t0 = time.perf_counter()
            out = gpu_batch.make_batch(parts, None, dev)
            torch.cuda.synchronize(dev)
            if it >= 3:
                e2e.append((time.perf_counter() - t0) * 1e3)
            del out
        ms = float(np.median(times))
        nbytes = 215.0 * n + 2 * 897 * 4.0 * n + (15 + 60 + 8) * float(m)
        line = {"workload": f"training batch: {n} replay rows, {m} configs", "rows": n, "configs": m,
                "ms": ms, "rows_per_s": n / (ms / 1e3),
                "roofline": {"bound": "hbm", "achieved": nbytes / (ms / 1e3) / 1e9, "peak": hbm, "unit": "GB/s",
                             "frac": nbytes / (ms / 1e3) / 1e9 / hbm, "peak_source": src},
                "e2e_ms": float(np.median(e2e)), "e2e_rows_per_s": n / (float(np.median(e2e)) / 1e3)}
        if n == 1024:
            L = oracle_lib.lib()
            xo = np.zeros((2 * n, wc.PUBFEAT), np.float32)
            po = np.zeros((m, 15), np.float32)
            t0 = time.perf_counter()
            L.oracle_replay_make_batch(rows.ctypes.data_as(Cc.c_void_p), Cc.c_size_t(n), cc.ctypes.data_as(Cc.c_void_p),
                                       seg.ctypes.data_as(Cc.c_void_p), Cc.c_size_t(m), xo.ctypes.data_as(Cc.c_void_p),
                                       po.ctypes.data_as(Cc.c_void_p))
            cpu_ms = (time.perf_counter() - t0) * 1e3
            line["cpu_baseline"] = {"value": n / (cpu_ms / 1e3), "unit": "rows/s", "cores": 1, "kind": "port",
                                    "sample": f"the {n}-row batch, once"}
            line["equal_to_cpu_batch"] = bool(np.array_equal(x.cpu().numpy(), xo) and
                                              np.array_equal(phi.cpu().numpy(), po))
        print(json.dumps(line), flush=True)


def leaf_workload(args):
    """the value network alone on rows from seeded random
    playouts of 10-60 plies. Positions: the roots of seeds 0.. with a seeded
    ply count in [10, 60] (wc_root_generate: seeded draft, uniform decisions,
    on to the next MainPlay); rows: the network rows of their depth-1
    subgames (each a position one coin play later, with both players' belief
    supports as the configs), taken until the batch size is reached. A leaf
    inference of a row is the trunk once plus both seat queries (join and
    readout over the row's configs), as the reference evaluates it
    (search.rs:1464-1636); the per-config encoder runs once per subgame.
    Times are CUDA events of wc_batch_leaf_values (per-solve network once,
    then the two seat queries). Accuracy: leaf values of the 16-bit paths
    against the fp32 path, norm-wise relative, over the whole batch."""
    import warchest_b200 as wc

    wc.set_cap_marker_value(0.0)
    weights = wc.seeded_weights("he", 0)
    cfg = wc.Cfg(depth=1, iters=0, snapshots=False, cfr=wc.Cfr.PLUS)
    rng = np.random.default_rng(2024)
    hbm, tflops, src = peaks()
    threads = os.cpu_count() or 1
    pool, seed = [], 0  # depth-1 jobs of seeds 0, 1, ... in seed order (built natively, in chunks)
    for target in (1024, 16384, 262144):
        while sum(j.info["net_rows"] for j in pool) < target:
            roots = []
            for s in range(seed, seed + 2048):
                try:
                    roots.append(wc.generate_root(s, int(rng.integers(10, 61))))
                except wc.SolveError:  # the game ended before the root
                    pass
            seed += 2048
            pool += [j for j in wc.PackedJob.build_many(roots, cfg, threads=threads)
                     if j is not None and j.info["net_rows"] > 0]
        jobs, rows = [], 0
        for j in pool:
            if rows >= target:
                break
            jobs.append(j)
            rows += j.info["net_rows"]
        counts = np.sum([j.counts() for j in jobs], axis=0)
        configs = sum(j.info["configs"] for j in jobs)
        flops = 17.0e6 * counts[20] + 2 * 197.6e3 * rows + 512 * (counts[14] + counts[15]) + 170e3 * configs
        line = {"workload": f"configs[1]: leaf inference alone, {rows} rows (target {target}) from {len(jobs)} "
                            f"positions of 10-60 seeded playout plies", "rows": rows, "configs": int(configs)}
        vals = {}
        for net in ("exact", "bf16", "f16"):
            c = wc.spawn(0, *weights, net=net)
            try:
                b = c.upload(jobs)
                for _ in range(3):  # warm-up
                    b.leaf_values(0)
                t = []
                for _ in range(5):
                    a = b.leaf_values(0, profile=True)
                    z = b.leaf_values(1, profile=True)
                    t.append(a["net_solve"] + a["leaf"] + z["leaf"])
                ms = float(np.median(t))
                parts = []
                for p in (0, 1):
                    b.leaf_values(p)
                    parts.append(np.concatenate([b.leaf_values_of(j, p) for j in range(len(jobs))]))
                vals[net] = np.concatenate(parts)
                b.free()
            finally:
                c.close()
            line[net] = {"ms": ms, "rows_per_s": rows / (ms / 1e3), "tflops": flops / (ms / 1e3) / 1e12,
                         "frac_of_bf16_peak": flops / (ms / 1e3) / 1e12 / tflops}
        for net in ("bf16", "f16"):
            line[net]["rel_err_vs_fp32"] = float(np.linalg.norm(vals[net] - vals["exact"]) /
                                                 np.linalg.norm(vals["exact"]))
        line["peak_source"] = src
        print(json.dumps(line), flush=True)


def main():
    global PLIES
    args = parse()
    PLIES = args.plies
    if args.workload == "leaf":
        leaf_workload(args)
        return
    if args.workload == "batch":
        batch_workload(args)
        return
    if args.workload == "resolve":
        resolve_workload(args)
        return
    if args.subgames_total:
        total_workload(args)
        return
    if args.impl == "reference":
        # the CPU reference runs on rank 0 alone; other ranks exit without work
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return
        local = 0
    else:
        world, rank, local = dist_setup(args)
    import oracle_lib
    import warchest_b200 as wc

    wc.set_cap_marker_value(0.0)  # the reference bench pins the horizon payoff at 0 (rebelbench.rs:35)
    oracle_lib.lib().oracle_set_cap_marker_value(0.0)
    cfg = wc.Cfg(depth=args.depth, iters=args.iters, snapshots=False, cfr=cfr_plus(wc), node_cap=200000)
    seeds = seed_range(rank, args.subgames)
    weights = wc.seeded_weights("he", 0) if args.net != "none" else None
    workload = {"workload": f"configs[2]: {args.subgames} subgames/GPU, depth {args.depth}, {args.iters} CFR+ iters, "
                            f"v5 net every iteration, {args.plies}-ply seeded roots",
                "subgames_per_gpu": args.subgames, "depth": args.depth, "iters": args.iters,
                "net": args.net, "parallelism": f"shards{world}",
                "l2": "working set (GBs of tree tables and state) far above the 126 MB L2"}

    if args.impl == "reference":
        if rank == 0:
            samples = [cpu_baseline(oracle_lib, cfg, weights, seeds) for _ in range(max(1, args.steps))]
            base = sorted(samples, key=lambda b: b["value"])[len(samples) // 2]
            base["sample"] += f"; median of {len(samples)} repetitions"
            line = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": UNIT, "n_gpus": world,
                    "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                    "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded roots)", "config": workload,
                    "cpu_baseline": base,
                    "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
            print(json.dumps(line), flush=True)
        return

    # host threads per rank: the ranks of one node share its cores
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    threads = args.build_threads or max(1, (os.cpu_count() or 1) // max(1, local_world))
    t0 = time.perf_counter()
    roots, jobs = build_jobs(wc, seeds, cfg, threads)
    build_s = time.perf_counter() - t0
    workload["capped_skipped"] = len(seeds) - len(jobs)
    workload["subgames_solved_per_gpu"] = len(jobs)

    # weights: rank 0's seeded blob, broadcast once over NCCL when sharded
    if weights is not None and world > 1:
        import torch

        tw = broadcast_weights(weights, torch.device("cuda", local))
        torch.cuda.synchronize()
        client = wc.spawn(local, net=args.net)
        client.set_weights_device(0, tw[0].data_ptr(), tw[1].data_ptr(), tw[2].data_ptr())
    elif weights is not None:
        client = wc.spawn(local, *weights, net=args.net)
    else:
        client = wc.spawn(local)

    batch = client.upload(jobs)
    stats = batch.stats()
    for _ in range(args.warmup):
        batch.solve()
    barrier(world)
    clocks = Clocks(local)
    clocks.start()
    times, profiles = [], []
    for _ in range(args.steps):
        prof = batch.solve_profiled()
        times.append(prof["total"] / 1e3)
        profiles.append(prof)
    launches = batch.launches()  # counted by the runtime as it launches
    clocks_rec = clocks.stop()
    barrier(world)
    step_s = max_over_ranks(world, float(np.mean(times)))
    total_nu = allsum(world, stats["node_updates"])
    total_leaf = allsum(world, stats["leaf_evals"])  # every collective runs on every rank, in the same order
    value = total_nu / step_s

    # end to end through the public API: pinned host blobs in, results out
    batch.free()
    e2e_times = []
    h2d = sum(j.info["table_bytes"] for j in jobs)
    d2h = sum(4 * j.info["cells"] + 4 * (j.info["root_nc0"] + j.info["root_nc1"]) for j in jobs)
    # wc_solve_batch keeps its two wave arenas across calls: one untimed call
    # sizes them, as a serving process does once at start-up
    client.solve_batch(jobs)
    for _ in range(1):
        barrier(world)
        t0 = time.perf_counter()
        res = client.solve_batch(jobs)
        e2e_times.append(time.perf_counter() - t0)
        del res
    e2e_s = max_over_ranks(world, min(e2e_times))
    e2e = {"value": total_nu / e2e_s, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
           "timing": "host wall clock around the synchronous wc_solve_batch (pinned host tables in, memory-bounded "
                     "waves with each wave's upload overlapping the previous wave's solve, results out), after "
                     "one untimed call that sizes the wave arenas"}

    # rooflines per kernel class; the headline object is the dominant one
    prof = {k: float(np.mean([p[k] for p in profiles])) for k in profiles[0]}
    per_class, src = rooflines(prof, algorithmic_work(jobs))
    dom = max(per_class, key=lambda k: per_class[k]["ms"])
    roofline = dict(per_class[dom])
    net_rows = sum(j.info["net_rows"] for j in jobs)
    traffic = TRAFFIC_PER_ROW[dom] * net_rows if dom in TRAFFIC_PER_ROW else None
    roofline.update({"kernel": KERNELS.get(dom, dom), "traffic": traffic, "peak_source": src,
                     "traffic_basis": "ncu DRAM bytes per network row (256-subgame capture, images above the L2) "
                                      "x this workload's rows",
                     "per_class": per_class, "per_class_ms": prof})

    if rank == 0:
        base = None if args.no_cpu_baseline else cpu_baseline(oracle_lib, cfg, weights, seeds)
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": DTYPES[args.net],
                "data": "synthetic (seeded roots, seeded He-normal weights)", "config": workload,
                "e2e": e2e, "gpu_launches": launches,
                "roofline": roofline, "cpu_baseline": base, "clocks": clocks_rec,
                "leaf_evals_per_sec": total_leaf / step_s,
                "host_build_s": build_s, "device_bytes": stats["device_bytes"]}
        print(json.dumps(line), flush=True)
    client.close()
    if world > 1:
        import torch.distributed as dist

        barrier(world)  # the other ranks wait here while rank 0 timed the CPU baseline
        dist.destroy_process_group()


def resolve_workload(args):
    """BASELINE configs[4]'s loop: --games games from belief-heavy roots
    (each player's belief over up to 256 consistent configs, Dirichlet(1)
    weights), each solving a subgame, walking it with the real play and
    re-solving with the carried beliefs, 8 solves per game, CFR+ at --iters
    (configs[4]: 1024) and --depth (configs[4]: 4), through the public
    GpuClient.play: continuous batching, as the reference's game actors feed
    its GPU service (every game builds its next subgame on a host thread as
    soon as its walk resumes; whenever the device is idle the subgames ready
    then are solved in one wc_solve_batch). Node-updates/s is over the solve
    calls' wall clock; solves/s over the whole loop's."""
    import warchest_b200 as wc

    wc.set_cap_marker_value(0.0)
    cfg = wc.Cfg(depth=args.depth, iters=args.iters, snapshots=True, cfr=cfr_plus(wc), node_cap=200000)
    weights = wc.seeded_weights("he", 0)
    client = wc.spawn(0, *weights, net=args.net)
    games = [wc.Game(cfg, seed=s, root=wc.generate_wide_root(s, 256), max_solves=8) for s in range(args.games)]
    threads = args.build_threads or (os.cpu_count() or 1)
    stats = {}
    wall0 = time.perf_counter()
    solved = client.play(games, threads=threads, stats=stats)
    wall_s = time.perf_counter() - wall0
    counters = [g.counters() for g in games]
    nodes = stats["nodes"] * float(args.iters)
    gpu_s = stats["solve_s"]
    line = {"workload": f"configs[4] loop: {args.games} belief-heavy games (256 configs per player), depth "
                        f"{args.depth}, {args.iters} CFR+ iters, 8 solves per game, one GPU, continuous batching",
            "games": args.games, "batches": stats["batches"], "largest_batch": stats["largest_batch"],
            "solves": solved,
            "walk_decisions": sum(c["walk_decisions"] for c in counters),
            "capped": sum(c["capped"] for c in counters),
            "wall_s": wall_s, "gpu_s": gpu_s, "solves_per_s": solved / wall_s,
            "node_updates_per_s_gpu": nodes / gpu_s if gpu_s else None, "host_threads": threads}
    print(json.dumps(line), flush=True)
    client.close()


def total_workload(args):
    """--subgames-total subgames (seeds 0 ..) split
    evenly over the ranks (strong scaling), depth 3, 512 CFR+ iterations,
    the net every iteration. A shard larger than one device batch is solved
    in memory-bounded waves by wc_solve_batch (each wave's host tables
    uploaded while the previous wave solves), so a step is one
    wc_solve_batch call timed on the host clock (uploads and the result
    download inside), max over ranks; one untimed call first sizes the wave
    arenas."""
    world, rank, local = dist_setup(args)
    import warchest_b200 as wc

    wc.set_cap_marker_value(0.0)
    cfg = wc.Cfg(depth=args.depth, iters=args.iters, snapshots=False, cfr=cfr_plus(wc), node_cap=200000)
    per = args.subgames_total // world
    seeds = list(range(rank * per, (rank + 1) * per if rank + 1 < world else args.subgames_total))
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    threads = args.build_threads or max(1, (os.cpu_count() or 1) // max(1, local_world))
    t0 = time.perf_counter()
    _, jobs = build_jobs(wc, seeds, cfg, threads)
    build_s = time.perf_counter() - t0
    weights = wc.seeded_weights("he", 0)
    if world > 1:
        import torch

        tw = broadcast_weights(weights, torch.device("cuda", local))
        torch.cuda.synchronize()
        client = wc.spawn(local, net=args.net)
        client.set_weights_device(0, tw[0].data_ptr(), tw[1].data_ptr(), tw[2].data_ptr())
    else:
        client = wc.spawn(local, *weights, net=args.net)
    nu = sum(j.info["nodes"] for j in jobs) * float(args.iters)
    for _ in range(max(1, args.warmup)):
        client.solve_batch(jobs)
    times = []
    for _ in range(args.steps):
        barrier(world)
        t0 = time.perf_counter()
        res = client.solve_batch(jobs)
        times.append(time.perf_counter() - t0)
        del res
    step_s = max_over_ranks(world, float(np.mean(times)))
    total_nu = allsum(world, nu)
    solved = allsum(world, float(len(jobs)))
    if rank == 0:
        line = {"metric": METRIC, "value": total_nu / step_s, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": max(1, args.warmup), "ms_per_step": step_s * 1e3, "higher_is_better": True,
                "scaling": "strong", "dtype": DTYPES[args.net], "data": "synthetic (seeded roots, seeded He-normal weights)",
                "config": {"workload": f"configs[3]: {args.subgames_total} subgames over {world} GPU(s), depth "
                                       f"{args.depth}, {args.iters} CFR+ iters, v5 net every iteration",
                           "subgames_total": args.subgames_total, "subgames_solved": int(solved),
                           "parallelism": f"shards{world}", "timing": "host clock around wc_solve_batch "
                           "(memory-bounded waves, tables uploaded inside the step), max over ranks"},
                "host_build_s": build_s}
        print(json.dumps(line), flush=True)
    client.close()
    if world > 1:
        import torch.distributed as dist

        barrier(world)
        dist.destroy_process_group()


def batch_levels(jobs):
    return max(j.info["levels"] for j in jobs)


def seed_range(rank, subgames):
    """The contiguous seed block of one rank (weak scaling: every rank solves
    its own `subgames` roots)."""
    return list(range(rank * subgames, (rank + 1) * subgames))


def broadcast_weights(weights, device):
    """Rank 0's (w, b, ln) to every rank, once, as device tensors (the only
    collective on the data path's setup; none per iteration)."""
    import torch
    import torch.distributed as dist

    tw = [torch.from_numpy(a).to(device) for a in weights[1:]]
    for t in tw:
        dist.broadcast(t, src=0)
    return tw


def _dist_device():
    import torch.distributed as dist

    return "cuda" if dist.get_backend() == "nccl" else "cpu"


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(world, x):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=_dist_device())
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def allsum(world, x):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=_dist_device())
    dist.all_reduce(t)
    return float(t.item())


PLIES = 20
KERNELS = {"rows": "k_rows", "vgather": "k_vgather", "reach": "k_rgather", "pool": "k_pool_fast",
           "join": "k_join_fast", "head": "k_head_fast", "trunk": "k_trunk_fast"}
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per network row
# per launch, from one ncu capture of each kernel on 256 subgames (1,441,491
# rows, seeds 0..255, depth 3, 4 GB on the device, its images far above the
# L2); a launch's traffic grows with its rows, so the full launch's traffic
# is this times the workload's rows. The pooling figure is of a launch that
# pooled both players.
TRAFFIC_PER_ROW = {"head": 1015.6, "join": 915.5, "pool": 451.6, "trunk": 438.4}
DTYPES = {"f16": "f32 CFR state, f16 tensor-core value net (fp32 accumulate)",
          "bf16": "f32 CFR state, tensor-core value net (fp32 accumulate): bf16 operands for the per-iteration "
                  "pooling / join / join-output chain, f16 for the once-per-solve trunk and the readout",
          "exact": "f32", "none": "f32"}

if __name__ == "__main__":
    main()
