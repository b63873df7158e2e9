// A deterministic single-precision tanh, identical on the host and on the
// GPU.
//
// The network's GELU is the tanh form (engine/src/net.rs:126-129). The
// reference takes tanh from the platform libm, so its own results already
// differ between platforms by an ulp or so; here one implementation built
// only from IEEE +, -, *, / and exact scaling is used by both the CUDA
// kernels and the CPU oracle, so the fp32 network path reproduces the oracle
// bit for bit. Both sides must be compiled without floating-point
// contraction (-ffp-contract=off / -fmad=false).
//
// Method: S. L. Moshier's Cephes single-precision tanhf (Cephes Mathematical
// Library, tanhf.c): an odd polynomial in x^2 for |x| <= 0.625, otherwise
// 1 - 2 / (exp(2|x|) + 1) with Cephes' expf (Cody-Waite reduction by ln 2 in
// two parts, then a degree-6 polynomial). The error against a correctly
// rounded tanh is checked by tests/test_detmath.py.
#pragma once

#ifdef __CUDACC__
#define WC_HD __host__ __device__ __forceinline__
#else
#define WC_HD inline
#endif

namespace wc {

// 2^n for integer n in [-126, 127], built from its exponent bits.
WC_HD float det_pow2(int n) {
    union {
        unsigned u;
        float f;
    } v;
    v.u = (unsigned)(n + 127) << 23;
    return v.f;
}

// Round to the nearest integer, ties toward +inf, for |x| < 2^22 (what the
// reduction needs: floor(y + 0.5)).
WC_HD float det_floor(float x) {
    int i = (int)x;  // truncation toward zero is exact for |x| < 2^31
    float f = (float)i;
    return f > x ? f - 1.0f : f;
}

// e^x for x in [0, 88] (the only range tanh needs).
WC_HD float det_exp(float x) {
    const float LOG2EF = 1.44269504088896341f;
    const float C1 = 0.693359375f;
    const float C2 = -2.12194440e-4f;
    float z = det_floor(LOG2EF * x + 0.5f);
    int n = (int)z;
    x = x - z * C1;
    x = x - z * C2;
    z = x * x;
    float p = 1.9875691500E-4f;
    p = p * x + 1.3981999507E-3f;
    p = p * x + 8.3334519073E-3f;
    p = p * x + 4.1665795894E-2f;
    p = p * x + 1.6666665459E-1f;
    p = p * x + 5.0000001201E-1f;
    float e = p * z + x + 1.0f;
    // scale in two steps so n up to 127 stays representable
    int h = n / 2;
    return e * det_pow2(h) * det_pow2(n - h);
}

WC_HD float det_tanh(float x) {
    float ax = x < 0.0f ? -x : x;
    if (ax > 0.625f) {
        if (ax > 44.0f) return x < 0.0f ? -1.0f : 1.0f;
        float s = det_exp(ax + ax);
        float t = 1.0f - 2.0f / (s + 1.0f);
        return x < 0.0f ? -t : t;
    }
    if (x == 0.0f) return x;
    float s = x * x;
    float p = -5.70498872745E-3f;
    p = p * s + 2.06390887954E-2f;
    p = p * s - 5.37397155531E-2f;
    p = p * s + 1.33314422036E-1f;
    p = p * s - 3.33332819422E-1f;
    return p * s * x + x;
}

// GELU, tanh form (net.rs:126-129), with the operation order of the reference.
WC_HD float det_gelu(float x) {
    float inner = 0.79788456f * (x + 0.044715f * x * x * x);
    return 0.5f * x * (1.0f + det_tanh(inner));
}

}  // namespace wc
