"""wc_debug_umma_gemm_static: the tensor-core GEMM self-test without device
allocation, for callers that cannot call cudaMalloc (their device memory is
owned by another allocator, or an allocation's device-wide synchronisation is
not acceptable on their path). Its device staging lives in one static array
that every call shares.

Checked through the C ABI against the allocating entry point,
wc_debug_umma_gemm, on the same operands: the two run the same kernel, so the
results must be identical (the GEMM tests' host-product tolerance is far
looser). Two calls in a row with different operands and shapes show that
nothing stale from the first call leaks into the second. A k beyond the static
array's capacity must be refused before anything runs.

This file sorts last so that a stop-at-first-failure run has run every other
test before it; it also passes alone in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def bf16_bits(x):
    u = np.asarray(x, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def last_error(lib):
    buf = C.create_string_buffer(4096)
    lib.wc_last_error(buf, 4096)
    return buf.value.decode()


def gemm(lib, fn, a, b):
    a = np.ascontiguousarray(a, np.uint16)
    b = np.ascontiguousarray(b, np.uint16)
    d = np.full((128, b.shape[0]), np.nan, np.float32)
    rc = getattr(lib, fn)(a.ctypes.data, b.ctypes.data, a.shape[1], b.shape[0], d.ctypes.data)
    return rc, d


def test_static_scratch_gemm_matches_allocating_entry_point(wc):
    lib = wc.lib()
    rng = np.random.default_rng(2024)
    # the largest accepted problem first, then a smaller one over its leftovers
    for k, n in [(256, 256), (128, 96)]:
        a = bf16_bits(rng.standard_normal((128, k)))
        b = bf16_bits(rng.standard_normal((n, k)))
        rc_ref, want = gemm(lib, "wc_debug_umma_gemm", a, b)
        assert rc_ref == 0, last_error(lib)
        rc, got = gemm(lib, "wc_debug_umma_gemm_static", a, b)
        assert rc == 0, last_error(lib)
        np.testing.assert_array_equal(got, want)


def test_static_scratch_gemm_small_then_large(wc):
    """A small static call, a small allocating call, then the largest static
    call: each launch must be allowed the shared memory it needs whatever ran
    before it, so the large call returns its own product, not the small
    call's leftovers in the shared array."""
    lib = wc.lib()
    rng = np.random.default_rng(7)
    order = [("wc_debug_umma_gemm_static", 64, 16), ("wc_debug_umma_gemm", 64, 16),
             ("wc_debug_umma_gemm_static", 256, 256)]
    for fn, k, n in order:
        a = bf16_bits(rng.standard_normal((128, k)))
        b = bf16_bits(rng.standard_normal((n, k)))
        rc_ref, want = gemm(lib, "wc_debug_umma_gemm", a, b)
        assert rc_ref == 0, last_error(lib)
        rc, got = gemm(lib, fn, a, b)
        assert rc == 0, last_error(lib)
        np.testing.assert_array_equal(got, want)


def test_static_scratch_gemm_refuses_oversize(wc):
    lib = wc.lib()
    a = np.zeros((128, 320), np.uint16)
    b = np.zeros((64, 320), np.uint16)
    rc, _ = gemm(lib, "wc_debug_umma_gemm_static", a, b)
    assert rc != 0
    assert "exceeds 256" in last_error(lib)
