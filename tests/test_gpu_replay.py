"""The training batch on the device (wc_replay_expand through
warchest_b200.gpu_batch.make_batch, the interface of the reference's
train/gpu_batch.py) against the CPU oracle's restatement of the CPU batch
(train/train.py:249-270). The reference's own gate (train/test_gpu_batch.py)
holds floats to atol 1e-6 and the rest exact; every feature here is one IEEE
division of a small integer or a table entry, so the bar is bit equality.

Rows are packed from real positions (seeded games 0 to 40 plies deep, and
the coin-play states of seeded playouts), each row with a ragged span of
configs per seat whose counts are drawn at random.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROW_BYTES, PUBFEAT = 215, 897


def replay_parts(wc, oracle, n_roots, pairs, seed):
    rows = []
    for s in range(n_roots):
        try:
            rows.append(np.frombuffer(wc.pack_row(wc.generate_root(s, plies=[0, 6, 20, 40][s % 4])), np.uint8))
        except wc.SolveError:
            continue
    if pairs:
        L = oracle.lib()
        L.oracle_replay_mirror_pairs.restype = C.c_size_t
        L.oracle_replay_mirror_pairs.argtypes = [C.c_uint32, C.c_uint64, C.c_void_p, C.c_size_t]
        buf = np.zeros((2 * pairs, ROW_BYTES), np.uint8)
        k = L.oracle_replay_mirror_pairs(64, seed, buf.ctypes.data_as(C.c_void_p), pairs)
        rows += list(buf[0:2 * k:2])
    rows = np.stack(rows)
    n = len(rows)
    rng = np.random.default_rng(seed)
    per = rng.integers(1, 5, 2 * n)
    seg = np.repeat(np.arange(2 * n, dtype=np.int64), per)
    m = len(seg)
    cc = rng.integers(0, 4, (m, 15)).astype(np.uint8)
    aux = rng.integers(0, 3, (n, 10)).astype(np.uint8)
    cp = (seg % 2).astype(np.uint8)
    cw = rng.random(m).astype(np.float32)
    cy = rng.standard_normal(m).astype(np.float32)
    return rows, aux, cc, cp, cw, cy, seg


def oracle_batch(oracle, rows, cc, seg):
    n, m = len(rows), len(cc)
    x = np.zeros((2 * n, PUBFEAT), np.float32)
    phi = np.zeros((m, 15), np.float32)
    rows, cc, seg = (np.ascontiguousarray(a) for a in (rows, cc, seg))
    rc = oracle.lib().oracle_replay_make_batch(rows.ctypes.data_as(C.c_void_p), C.c_size_t(n),
                                               cc.ctypes.data_as(C.c_void_p), seg.ctypes.data_as(C.c_void_p),
                                               C.c_size_t(m), x.ctypes.data_as(C.c_void_p),
                                               phi.ctypes.data_as(C.c_void_p))
    assert rc == 0
    return x, phi


@pytest.mark.parametrize("n_roots,pairs,seed", [(1, 0, 1), (24, 400, 2), (64, 4000, 3)])
def test_device_batch_equals_cpu_batch(wc, oracle, n_roots, pairs, seed):
    import torch

    from warchest_b200 import gpu_batch

    parts = replay_parts(wc, oracle, n_roots, pairs, seed)
    rows, aux, cc, cp, cw, cy, seg = parts
    dev = torch.device("cuda:0")
    gpu_batch.warmup(dev)
    for _ in range(2):  # twice: the second call reuses the loaded tables
        x, phi, w, sg, y, owner, nseg = gpu_batch.make_batch(parts, None, dev)
        torch.cuda.synchronize(dev)
        want_x, want_phi = oracle_batch(oracle, rows, cc, seg)
        np.testing.assert_array_equal(x.cpu().numpy(), want_x)
        np.testing.assert_array_equal(phi.cpu().numpy(), want_phi)
        np.testing.assert_array_equal(w.cpu().numpy(), cw)
        np.testing.assert_array_equal(sg.cpu().numpy(), seg)
        np.testing.assert_array_equal(y.cpu().numpy(), cy)
        np.testing.assert_array_equal(owner.cpu().numpy(), aux.astype(np.int64))
        assert nseg == 2 * len(rows)
    print(f"{len(rows)} rows, {len(seg)} configs: device batch == CPU batch")


def test_device_batch_refuses_missing_spans(wc, oracle):
    from warchest_b200 import gpu_batch

    rows, aux, cc, cp, cw, cy, seg = replay_parts(wc, oracle, 4, 0, 5)
    keep = seg != seg.max()  # the last row's second seat has no configs: its lookup runs past the end
    with pytest.raises(wc.SolveError):
        gpu_batch.make_batch((rows, aux, cc[keep], cp[keep], cw[keep], cy[keep], seg[keep]), None, "cuda:0")
