"""tcgen05 self-test: descriptors, 128-byte swizzle and TMEM read-out of the
tensor-core kernels, checked against a float64 product of the same bf16
operands (fp32 accumulation over K <= 256: relative error ~1e-6)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def bf16_bits(x):
    u = np.asarray(x, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_value(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("k,n", [(64, 16), (128, 128), (192, 96), (128, 256), (256, 112)])
def test_umma_gemm_matches_host(wc, k, n):
    rng = np.random.default_rng(k * 1000 + n)
    a = bf16_bits(rng.standard_normal((128, k)))
    b = bf16_bits(rng.standard_normal((n, k)))
    got = wc.debug_umma_gemm(a, b)
    want = bf16_value(a).astype(np.float64) @ bf16_value(b).astype(np.float64).T
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-4)
