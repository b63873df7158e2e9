// Thin sm_100a helpers for the 5th-generation tensor cores (tcgen05):
// shared-memory matrix descriptors, the bf16 instruction descriptor, MMA
// issue and completion through an mbarrier, TMEM allocation and loads.
//
// Operand layout used everywhere here: K-major, 128-byte swizzled. A tile of
// R rows (R a multiple of 8) and K columns of bf16 is stored as K/64 "atoms";
// atom a holds columns [64a, 64a + 64) of every row, row r at byte
// a * R * 128 + r * 128, its 16-byte chunk c at position c ^ (r % 8). Tiles
// start on 1024-byte boundaries. One MMA consumes K = 16 (32 bytes): the
// descriptor start address advances by 32 bytes within an atom.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

namespace umma {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Byte offset of element (r, k) inside a swizzled K-major tile of R rows.
__device__ __forceinline__ uint32_t sw128_offset(uint32_t R, uint32_t r, uint32_t k) {
    uint32_t atom = k >> 6, kk = k & 63;
    uint32_t chunk = (kk >> 3) ^ (r & 7);
    return atom * R * 128u + r * 128u + chunk * 16u + (kk & 7) * 2u;
}

// Shared-memory descriptor of a swizzled K-major operand (SWIZZLE_128B:
// layout type 2, SBO = 1024 bytes between 8-row groups, version 1).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}

// Descriptor of the K-step `k0` (a multiple of 16) of a tile of R rows.
__device__ __forceinline__ uint64_t desc_at(uint32_t tile_saddr, uint32_t R, uint32_t k0) {
    return desc_sw128(tile_saddr + (k0 >> 6) * R * 128u + (k0 & 63) * 2u);
}

// Instruction descriptor, kind::f16 with K-major A and B of one 16-bit type
// (fmt: 0 = f16, 1 = bf16) and an f32 D.
__host__ __device__ constexpr uint32_t idesc16(uint32_t M, uint32_t N, uint32_t fmt) {
    return (1u << 4) | (fmt << 7) | (fmt << 10) | ((N >> 3) << 17) | ((M >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_bf16(uint32_t M, uint32_t N) { return idesc16(M, N, 1u); }

// The 16-bit operand type of the tensor-core network: HALF = true is IEEE
// binary16 (11 significant bits), false is bfloat16 (8 significant bits, the
// fp32 exponent range). Both run at the same tcgen05 rate.
template <bool HALF>
struct Op16;
template <>
struct Op16<false> {
    static constexpr uint32_t fmt = 1;
    static __device__ __forceinline__ uint32_t pack(float a, float b) {
        __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    }
    static __device__ __forceinline__ uint16_t one(float a) {
        __nv_bfloat16 v = __float2bfloat16_rn(a);
        return *reinterpret_cast<uint16_t*>(&v);
    }
    static __device__ __forceinline__ float lo(uint32_t w) { return __uint_as_float(w << 16); }
    static __device__ __forceinline__ float hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
    static __device__ __forceinline__ float at(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }
};
template <>
struct Op16<true> {
    static constexpr uint32_t fmt = 0;
    static __device__ __forceinline__ uint32_t pack(float a, float b) {
        __half2 v = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    }
    static __device__ __forceinline__ uint16_t one(float a) { return __half_as_ushort(__float2half_rn(a)); }
    static __device__ __forceinline__ float lo(uint32_t w) { return __half2float(__ushort_as_half((uint16_t)(w & 0xffffu))); }
    static __device__ __forceinline__ float hi(uint32_t w) { return __half2float(__ushort_as_half((uint16_t)(w >> 16))); }
    static __device__ __forceinline__ float at(uint16_t v) { return __half2float(__ushort_as_half(v)); }
};

// D[tmem] (+)= A * B^T, one elected thread.
__device__ __forceinline__ void mma16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
        :
        : "r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

// The same product with A read from tensor memory: tmem_a is A's first
// column (lane field 0), one row per lane, two 16-bit K elements per 32-bit
// column (low half the even element), so each K step of 16 is 8 columns.
__device__ __forceinline__ void mma16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
        :
        : "r"(tmem_d), "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

// Arrive on `mbar` when every MMA issued so far by this thread has completed.
__device__ __forceinline__ void commit(uint64_t* mbar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(mbar))
                 : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* mbar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(mbar)), "r"(count) : "memory");
}

// Wait limits, in nanoseconds of %globaltimer. A product or a bulk copy takes
// microseconds, so a wait that runs for WAIT_NS has met a partner that will
// never arrive; the caller records an error and stops issuing work. DRAIN_NS
// bounds the waits at a kernel's exit for work that is already in flight
// (an issued product or copy, which completes on its own).
constexpr uint64_t WAIT_NS = 2000000000ull;
constexpr uint64_t DRAIN_NS = 4000000000ull;

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// One test of phase `parity` of the barrier at shared address `addr`.
__device__ __forceinline__ bool mbar_test(uint32_t addr, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait on phase `parity`: returns false if the phase has not
// completed after `limit_ns` (the caller records an error and skips its
// dependent work instead of hanging). The limit is wall time, so it does not
// depend on try_wait's suspend time or on profiler instrumentation.
__device__ __forceinline__ bool mbar_wait(uint64_t* mbar, uint32_t parity, uint64_t limit_ns = WAIT_NS) {
    const uint32_t addr = smem_u32(mbar);
    if (mbar_test(addr, parity)) return true;
    const uint64_t t0 = now_ns();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 16; ++i)
            if (mbar_test(addr, parity)) return true;
        if (now_ns() - t0 >= limit_ns) return false;
    }
}

// Self-check of a pointer used by 16-byte vector or bulk accesses.
__device__ __forceinline__ bool misaligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; }

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// TMEM allocation by one whole warp; the address lands in *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

// 32 consecutive f32 columns of this thread's TMEM lane (warp w reads lanes
// 32w..32w+31): taddr already includes the lane offset (32w << 16).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// The same load without the wait, into raw registers: issue several, then
// one tmem_wait_ld before reading any of them.
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Store 32 consecutive f32 columns of this thread's TMEM lane (the inverse of
// tmem_ld32), then wait until the stores have landed.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
    uint32_t r[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(v[i]);
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        :
        : "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
          "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
          "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 raw 32-bit words into consecutive columns of this thread's TMEM lane,
// without the wait (follow with tmem_wait_st before the data is consumed).
__device__ __forceinline__ void tmem_st32_nowait(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        :
        : "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
          "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
          "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Prefetch [p, p + bytes) into L2 without waiting (the bulk copy engine
// fetches it). The copy wants 16-byte boundaries: the start is rounded down
// (still inside the 16-byte aligned allocation that holds p) and the end is
// rounded down too, so nothing past the range's end is touched.
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, size_t bytes) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p) & ~uintptr_t(15);
    const uintptr_t e = (reinterpret_cast<uintptr_t>(p) + bytes) & ~uintptr_t(15);
    if (e > a)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"((uint32_t)(e - a)) : "memory");
}

// Bulk asynchronous copy global -> shared (16-byte aligned, size a multiple
// of 16), completing `bytes` of transaction count on `bar`; and the arrive
// that announces how many bytes the phase expects.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// 8 consecutive floats as one 16-byte chunk of 16-bit operands.
template <bool HALF = false>
__device__ __forceinline__ uint4 pack_chunk(const float* x) {
    return make_uint4(Op16<HALF>::pack(x[0], x[1]), Op16<HALF>::pack(x[2], x[3]), Op16<HALF>::pack(x[4], x[5]),
                      Op16<HALF>::pack(x[6], x[7]));
}

// GELU (tanh form) for the tensor-core path, through the identity
// 0.5 x (1 + tanh(u)) = x / (1 + exp(-2u)), u = sqrt(2/pi) (x + 0.044715 x^3),
// with the hardware base-2 exponential (relative error about 2^-22) and a fast
// divide: about 1e-6 relative error everywhere, well under the 16-bit operand
// rounding, and no cancellation for negative x. The exponent is clamped at
// 126 so the divisor stays finite (x / (1 + 2^126) is 0 to fp32 precision).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float gelu_fast(float x) {
    const float u = 0.79788456f * (x + 0.044715f * x * x * x);
    const float e = ex2_approx(fminf(-2.8853900817779268f * u, 126.0f));
    return __fdividef(x, 1.0f + e);
}

// LayerNorm affine + GELU (tanh form) of two already-normalised values
// n = (x - mean) / sd at columns c, c + 1, packed as two 16-bit operands.
// gb2 holds the (gamma, beta) pairs of the columns as packed f16x2 words:
// [2 * (c / 2)] the gammas, [2 * (c / 2) + 1] the betas. Computed in f16x2
// arithmetic with the hardware f16x2 tanh (one conversion, one FMA for gamma /
// beta, the tanh form x (1 + tanh(u)) / 2 with x^2 capped at 1024 inside u,
// where tanh has long saturated; 7 packed ops and one tanh per pair): its
// error is of the order of the f16 rounding of the result. For bf16 operands
// the f16 pair is then rounded to bf16 (3 fewer mantissa bits, so the f16
// steps add little), which keeps the epilogue at the f16 path's instruction
// count.
__device__ __forceinline__ __half2 ln_gelu2_h(float n0, float n1, int c, const uint32_t* gb2) {
    const uint2 gb = *reinterpret_cast<const uint2*>(gb2 + 2 * (c >> 1));
    const __half2 n = __floats2half2_rn(n0, n1);
    const __half2 x = __hfma2(n, *reinterpret_cast<const __half2*>(&gb.x), *reinterpret_cast<const __half2*>(&gb.y));
    const __half2 x2 = __hmin2(__hmul2(x, x), __float2half2_rn(1024.0f));
    const __half2 u = __hmul2(x, __hfma2(x2, __float2half2_rn(0.035677408f), __float2half2_rn(0.79788456f)));
    uint32_t ub = *reinterpret_cast<const uint32_t*>(&u), tb;
    asm("tanh.approx.f16x2 %0, %1;" : "=r"(tb) : "r"(ub));
    const __half2 t = *reinterpret_cast<const __half2*>(&tb);
    return __hmul2(x, __hfma2(t, __float2half2_rn(0.5f), __float2half2_rn(0.5f)));
}
template <bool HALF>
__device__ __forceinline__ uint32_t ln_gelu2(float n0, float n1, int c, const uint32_t* gb2) {
    const __half2 g = ln_gelu2_h(n0, n1, c, gb2);
    if constexpr (HALF) {
        return *reinterpret_cast<const uint32_t*>(&g);
    } else {
        const float2 f = __half22float2(g);
        return Op16<false>::pack(f.x, f.y);
    }
}

// Pairs of fp32 values in one 64-bit register for the sm_100 packed fp32
// forms (add / fma .f32x2: two IEEE fp32 operations per instruction, each
// rounded as the scalar one): low word the first value.
__device__ __forceinline__ unsigned long long f2(uint32_t lo, uint32_t hi) {
    unsigned long long d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo), "r"(hi));
    return d;
}
__device__ __forceinline__ unsigned long long f2(float lo, float hi) { return f2(__float_as_uint(lo), __float_as_uint(hi)); }
__device__ __forceinline__ float f2_lo(unsigned long long v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(unsigned long long v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// (gamma, beta) of columns c, c + 1 as the packed words ln_gelu2 reads.
__device__ __forceinline__ void pack_gb2(const float* gam, const float* bet, int c, uint32_t* out2) {
    const __half2 g = __floats2half2_rn(gam[c], gam[c + 1]), b = __floats2half2_rn(bet[c], bet[c + 1]);
    out2[0] = *reinterpret_cast<const uint32_t*>(&g);
    out2[1] = *reinterpret_cast<const uint32_t*>(&b);
}

}  // namespace umma
