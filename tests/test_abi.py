"""The C ABI without a GPU: the library loads, exports every function that
include/wc_b200.h declares, and its device entry points fail loudly (an
error status and message, no CPU fallback) when no CUDA device is present.
Host-only entry points (roots, jobs, weights) work on the CPU."""
import ctypes as C
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "wc_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?(?:int|void|uint64_t|size_t|char)\s*\*?\s*(wc_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_header_declares_the_service_surface():
    names = declared_functions()
    for must in ["wc_init", "wc_publish", "wc_publish_device", "wc_solve_batch", "wc_submit", "wc_wait",
                 "wc_result_free", "wc_job_build", "wc_last_error", "wc_queued_work", "wc_shutdown"]:
        assert must in names


def test_library_exports_every_declared_function(wc):
    lib = wc.lib()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_device_entry_points_fail_loudly_without_a_gpu(wc):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    with pytest.raises(wc.SolveError) as e:
        wc.spawn(0)
    assert e.value.code == 2  # WC_E_CUDA
    buf = C.create_string_buffer(4096)
    wc.lib().wc_last_error(buf, 4096)
    assert buf.value


def test_reference_root_encoding_at_the_boundary(wc):
    """wc_job_build reads the reference's own root encoding (write_root,
    engine/src/roots.rs:247-313, format v3). A root written here field by
    field, as the Rust engine writes it (tests/wc_state.py, independent of
    the library's encoder), builds a job; a roots file of such roots splits
    back into them (read_roots); and the library's generated roots decode
    with the same independent reader and re-encode byte for byte."""
    import struct

    from wc_state import (BLACK, CAVALRY, CROSSBOWMAN, FOOTMAN, LANCER, PIKEMAN, ROYAL_COIN, SWORDSMAN,
                          WARRIOR_PRIEST, WHITE, ARCHER, Z_BAG, Z_HAND, State, decode_root, encode_root)

    s = State.blank(WHITE)
    s.set_unit(17, WHITE, WARRIOR_PRIEST, 1)
    s.set_unit(19, BLACK, FOOTMAN, 3)
    for u in (WARRIOR_PRIEST, SWORDSMAN, PIKEMAN, CROSSBOWMAN, ROYAL_COIN):
        s.add_zone(WHITE, Z_BAG, u, 1)
    for u in (FOOTMAN, ARCHER, CAVALRY, LANCER, ROYAL_COIN):
        s.add_zone(BLACK, Z_BAG, u, 1)
    s.add_zone(WHITE, Z_HAND, WARRIOR_PRIEST, 1)
    # slots are the owned unit types in index order: white's WP is slot 3
    root = encode_root(s, [[(((0, 0, 0, 1, 0), (0,) * 5, None), 1.0)], [(((0,) * 5, (0,) * 5, None), 1.0)]])
    job = wc.PackedJob.from_root(root, wc.Cfg(depth=2, iters=4, snapshots=True, cfr=wc.Cfr.PLUS))
    assert job.info["nodes"] > 1 and job.info["root_nc0"] == 1 and job.info["root_nc1"] == 1
    with pytest.raises(wc.SolveError):  # truncated: refused, not read past the end
        wc.PackedJob.from_root(root[:-3], wc.Cfg(depth=2, iters=4))
    # a coin in flight in no slot (any byte but 0xff and 0-4) is refused as an
    # argument (WC_E_ARG)
    for bad in ((((0, 0, 0, 1, 0), (0,) * 5, 7), 1.0), (((0, 0, 0, 1, 0), (0,) * 5, 0x80), 1.0)):
        with pytest.raises(wc.SolveError) as e:
            wc.PackedJob.from_root(encode_root(s, [[bad], [(((0,) * 5, (0,) * 5, None), 1.0)]]),
                                   wc.Cfg(depth=2, iters=4))
        assert e.value.code == 1
    g = wc.generate_root(0)
    assert g == wc.generate_root(0)  # deterministic
    st, bel = decode_root(g)
    assert encode_root(st, bel) == g
    for b in bel:
        assert abs(sum(w for _, w in b) - 1.0) < 1e-5
    roots_file = struct.pack("<III", 0x57107207, 3, 2) + root + g
    assert wc.split_roots_file(roots_file) == [root, g]
    with pytest.raises(wc.SolveError):
        wc.split_roots_file(struct.pack("<III", 0x57107207, 1, 0))  # a version-1 file is refused


def test_weight_blobs(wc, oracle):
    dims, w, b, ln = wc.seeded_weights("test", 0xD15EA5E)
    assert dims == [5]
    assert np.all(np.abs(w) <= 0.05) and abs(float(w.mean())) < 1e-3
    assert np.all(b == 0)
    L = oracle.lib()
    n = L.oracle_norms(None, None)
    g_off = (C.c_uint64 * n)()
    width = (C.c_uint64 * n)()
    L.oracle_norms(g_off, width)
    gam = np.zeros_like(ln, dtype=bool)
    for o, k in zip(g_off, width):
        assert np.all(ln[o:o + k] == 1.0)  # LayerNorm gamma = 1
        gam[o:o + k] = True
    assert np.all(ln[~gam] == 0.0)  # beta = 0
    _, w2, b2, _ = wc.seeded_weights("he", 0)
    assert np.all(b2 == 0) and np.isfinite(w2).all() and 0.01 < float(w2.std()) < 1.0
    _, w3, _, _ = wc.seeded_weights("he", 0)
    assert np.array_equal(w2, w3)
