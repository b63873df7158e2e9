// The tensor-core ("fast") value network: tcgen05 MMAs with operands in
// 128-byte-swizzled shared memory and fp32 accumulators in TMEM, epilogues on
// the CUDA cores (bias, residual, LayerNorm, tanh-GELU).
//
// Operand types. The kernels' template flag H is the type of the
// per-iteration chain, which carries nearly all of a solve's network work:
// the pooling product, the four join layers and the join output product
// (H = true: f16, false: bf16). The readout product V = H * F^T always
// takes f16 operands (the LayerNorm output h and f(c); both well inside
// f16's range), and so do the stored board rows P and jp that the chain adds
// in: the readout <f(c), h> is nearly orthogonal for these networks, so it
// multiplies the relative error of its operands several times, and bf16's
// 8-bit mantissa there alone costs about 1e-2 relative error in the leaf
// values, where f16's 11 bits cost about 1e-3.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <map>
#include <mutex>
#include <set>

#include "device.h"
#include "kernels.h"
#include "umma.cuh"

namespace wcdev {

// ---------------------------------------------------------------- selftest
// D[128, N] = A[128, K] * B[N, K]^T through one CTA's tcgen05 path: checks the
// descriptors, the swizzle and the TMEM read-out against a host product.
__global__ void k_umma_selftest(const __nv_bfloat16* __restrict__ A, const __nv_bfloat16* __restrict__ B, int K,
                                int N, float* __restrict__ D, int* __restrict__ status) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t mbar;
    __shared__ uint32_t tmem_slot;
    uint8_t* smem = smem_raw + ((1024u - (umma::smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sA = smem;
    uint8_t* sB = smem + 128 * K * 2;
    const int tid = threadIdx.x, warp = tid / 32;
    // stage operands, 8 bf16 (16 bytes) at a time
    for (int q = tid; q < 128 * K / 8; q += blockDim.x) {
        int r = q / (K / 8), k = (q % (K / 8)) * 8;
        *reinterpret_cast<uint4*>(sA + umma::sw128_offset(128, r, k)) =
            *reinterpret_cast<const uint4*>(A + (size_t)r * K + k);
    }
    for (int q = tid; q < N * K / 8; q += blockDim.x) {
        int r = q / (K / 8), k = (q % (K / 8)) * 8;
        *reinterpret_cast<uint4*>(sB + umma::sw128_offset(N, r, k)) =
            *reinterpret_cast<const uint4*>(B + (size_t)r * K + k);
    }
    if (tid == 0) {
        umma::mbar_init(&mbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    uint32_t ncols = 32;
    while (ncols < (uint32_t)N) ncols <<= 1;
    if (warp == 0) umma::tmem_alloc(&tmem_slot, ncols);
    umma::fence_async_smem();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = tmem_slot;
    if (tid == 0) {
        const uint32_t idesc = umma::idesc_bf16(128, N);
        for (int k0 = 0; k0 < K; k0 += 16)
            umma::mma16(tmem, umma::desc_at(umma::smem_u32(sA), 128, k0), umma::desc_at(umma::smem_u32(sB), N, k0),
                           idesc, k0 > 0);
        umma::commit(&mbar);
    }
    __shared__ int drained;
    const bool ok = umma::mbar_wait(&mbar, 0);
    umma::fence_before_sync();
    const bool bad = __syncthreads_or(!ok) != 0;
    umma::fence_after_sync();
    if (!bad) {
        float v[32];
        for (int c = 0; c < N; c += 32) {
            umma::tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + c, v);
            for (int j = 0; j < 32 && c + j < N; ++j) D[(size_t)tid * N + c + j] = v[j];
        }
    }
    if (tid == 0) {
        // the product still runs after a timed-out wait: it must finish before
        // the tensor memory is released (if it never does, the memory stays
        // allocated, status 2, and the context can no longer be trusted)
        drained = bad ? (umma::mbar_wait(&mbar, 0, umma::DRAIN_NS) ? 1 : 0) : 1;
        if (bad) *status = drained ? 1 : 2;
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (warp == 0 && drained) umma::tmem_dealloc(tmem, ncols);
}

// The self-test kernel's dynamic shared-memory limit: 200 KB, above the
// largest static-path problem (k = n = 256: 193 KB) and below the 227 KB a
// CTA may hold with the kernel's own static shared memory. Both entry points
// set this one value on every call, so no call can leave the limit below
// what another call's launch needs.
constexpr int SELFTEST_SMEM_MAX = 200 * 1024;

// ------------------------------------------------------------- fast kernels

constexpr int POOL = wc::NET_POOL, JW = wc::NET_JW, D = wc::NET_D;
constexpr uint32_t TILE_J = 128u * 128u * 2u;  // one [128][128] 16-bit operand tile
constexpr uint32_t ATOM = 128u * 128u;         // one 128-row x 64-column atom of 16-bit operands

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    return p + ((1024u - (umma::smem_u32(p) & 1023u)) & 1023u);
}

// Row statistics of a LayerNorm whose row is spread over the four column
// groups of a 16-warp CTA (warp w: rows 32 (w % 4) .., columns group w / 4).
__device__ __forceinline__ void row_stats4(const float* v, int n, float (*part)[4], int row, int cg, int width,
                                           float* mean, float* inv) {
    float s = 0.0f;
    for (int j = 0; j < n; ++j) s += v[j];
    part[row][cg] = s;
    __syncthreads();
    const float m = (part[row][0] + part[row][1] + part[row][2] + part[row][3]) / (float)width;
    __syncthreads();
    float q = 0.0f;
    for (int j = 0; j < n; ++j) q += (v[j] - m) * (v[j] - m);
    part[row][cg] = q;
    __syncthreads();
    *inv = rsqrtf((part[row][0] + part[row][1] + part[row][2] + part[row][3]) / (float)width + 1e-5f);
    *mean = m;
}

// A read-only 16-byte load the compiler keeps where it is written (a
// loop-invariant load hoisted out of a loop would hold its registers
// throughout).
__device__ __forceinline__ float4 ldg4_inplace(const float4* p) {
    float4 v;
    asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}

// One tile = up to 128 network rows of one job: first local row, count.
struct HeadTile {
    uint32_t job, first, count, pad;
};

// The join chain for traverser p (net.rs:801-832), one 128-row tile of one
// job at a time: z = jp + [pooled_p | pooled_o] Wb + b, three residual
// blocks z += W_i LNGELU(z) + b_i, and out = LNGELU(z), written as the head's
// A-operand image. One thread per row (TMEM lane), so a row's LayerNorm
// needs no exchange between threads. The residual stream z lives in TMEM:
// initialised with jp + b by tcgen05.st, each layer's MMA accumulates onto it,
// and the epilogue adds the running sum of the block biases. The four weight
// tiles stream through one 32 KB slot by bulk copy (the next layer's weight
// lands during this layer's epilogue) and the next tile's pooled images
// land during the last layer, so a CTA needs ~69 KB of shared memory and
// three run per SM, each one's MMAs and copies overlapping the others'
// epilogues. The epilogue takes the row's 128 values in two halves (read
// twice from TMEM: once for the statistics, once for LayerNorm and GELU).
template <bool H>
__global__ void __launch_bounds__(128, 3)
    k_join_fast(const JobDev* __restrict__ jobs, const HeadTile* __restrict__ tiles, uint32_t ntiles, FastNetDev fn,
                int p, const uint16_t* __restrict__ pool_img, const uint16_t* __restrict__ jp,
                uint16_t* __restrict__ zout_img, int* __restrict__ err) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t bar_in, bar_w, bar_mma;
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    if (umma::misaligned16(fn.join_tiles) || umma::misaligned16(pool_img) || umma::misaligned16(jp) ||
        umma::misaligned16(zout_img)) {  // entry self-check: a launch contract broken, nothing touched
        if (threadIdx.x == 0) atomicExch(err, 31);
        return;
    }
    uint8_t* smem = align1024(smem_raw);
    uint8_t* sWt = smem;               // the current layer's weight tile
    uint8_t* sA = smem + TILE_J;
    // [0] b with the seat folded in, [1..3] running sums of the block biases;
    // then per layer the LayerNorm's (gamma, beta) column pairs packed for
    // ln_gelu2
    float (*vec)[JW] = reinterpret_cast<float (*)[JW]>(sA + TILE_J);
    uint32_t (*gb2)[JW] = reinterpret_cast<uint32_t (*)[JW]>(sA + TILE_J + 4 * JW * 4);
    const int tid = threadIdx.x, warp = tid >> 5;
    for (int i = tid; i < 4 * (JW / 2); i += blockDim.x) {
        const int L = i / (JW / 2), c = 2 * (i % (JW / 2));
        umma::pack_gb2(fn.ln_g[L], fn.ln_b[L], c, &gb2[L][c]);
    }
    for (int i = tid; i < 4 * JW; i += blockDim.x) {
        const int v = i / JW, c = i % JW;
        float x = v == 0 ? fn.beff[p][c] : 0.0f;
        for (int u = 0; u < v; ++u) x += fn.bj[u][c];
        vec[v][c] = x;
    }
    if (tid == 0) {
        umma::mbar_init(&bar_in, 1);
        umma::mbar_init(&bar_w, 1);
        umma::mbar_init(&bar_mma, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        abort_flag = 0;
    }
    if (warp == 0) umma::tmem_alloc(&tmem_slot, 128);
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = tmem_slot;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const uint32_t my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const uint64_t uses = (uint64_t)my_tiles * 4;  // weight-slot uses: Wb, W1, W2, W3 per tile
    bool pend_in = false, pend_w = false;
    auto load_weight = [&](uint64_t k) {
        const uint8_t* src = fn.join_tiles + (size_t)(k & 3) * TILE_J;
        umma::expect_tx(&bar_w, TILE_J);
        for (uint32_t o = 0; o < TILE_J; o += ATOM) umma::bulk_g2s(sWt + o, src + o, ATOM, &bar_w);
        pend_w = true;
    };
    auto load_pooled = [&](uint32_t t) {
        const uint8_t* base = reinterpret_cast<const uint8_t*>(pool_img) + (size_t)t * (2 * ATOM);
        umma::expect_tx(&bar_in, 2 * ATOM);
        umma::bulk_g2s(sA, base + p * ATOM, ATOM, &bar_in);
        umma::bulk_g2s(sA + ATOM, base + (1 - p) * ATOM, ATOM, &bar_in);
        pend_in = true;
    };
    // the jp rows of tile t into L2 (they are read at the tile's start)
    auto prefetch_jp = [&](uint32_t t) {
        const HeadTile ht = tiles[t];
        umma::bulk_prefetch_l2(jp + ((size_t)jobs[ht.job].row_base + ht.first) * JW, (size_t)ht.count * JW * 2);
    };
    if (tid == 0 && my_tiles) {
        load_pooled(blockIdx.x);
        load_weight(0);
        if (blockIdx.x + gridDim.x < ntiles) prefetch_jp(blockIdx.x + gridDim.x);
    }
    // The parity each barrier completes next (the same in every thread);
    // pend_in / pend_w (thread 0, which issues the copies) and pend_mma (every
    // thread) mark work issued but not yet seen to complete. Every stop
    // decision is block-uniform (__syncthreads_or), and nothing is issued
    // after a failed wait.
    uint32_t ph_in = 0, ph_w = 0, ph_mma = 0;
    bool pend_mma = false, dead = false;
    const uint64_t wait_ns = fn.wait_ns;
    uint64_t k = 0;
    const uint32_t idesc = umma::idesc16(128, 128, umma::Op16<H>::fmt);
    for (uint32_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const HeadTile ht = tiles[t];
        const JobDev& J = jobs[ht.job];
        const bool valid = (uint32_t)tid < ht.count;
        const uint32_t g = J.row_base + ht.first + tid;
        if (tid == 32 && t + 2 * gridDim.x < ntiles) prefetch_jp(t + 2 * gridDim.x);
        {  // z = jp + b
            const uint4* jr = reinterpret_cast<const uint4*>(jp + (size_t)(valid ? g : 0) * JW);
#pragma unroll 1
            for (int c4 = 0; c4 < 4; ++c4) {
                float v[32];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint4 q = valid ? jr[4 * c4 + i] : make_uint4(0, 0, 0, 0);
                    const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        v[8 * i + 2 * e] = umma::Op16<true>::lo(w4[e]) + vec[0][32 * c4 + 8 * i + 2 * e];
                        v[8 * i + 2 * e + 1] = umma::Op16<true>::hi(w4[e]) + vec[0][32 * c4 + 8 * i + 2 * e + 1];
                    }
                }
                umma::tmem_st32(tmem + lane_off + 32 * c4, v);
            }
        }
        umma::fence_before_sync();
        __syncthreads();
        umma::fence_after_sync();
#pragma unroll 1
        for (int L = 0; L < 4; ++L, ++k) {
            // the layer's operands: the pooled images (first layer) and its
            // weight tile; the previous layer's A writes precede this barrier
            {
                bool ok = true;
                if (tid == 0) {
                    if (L == 0) ok = umma::mbar_wait(&bar_in, ph_in, wait_ns);
                    ok = ok && umma::mbar_wait(&bar_w, ph_w, wait_ns);
                }
                dead = __syncthreads_or(!ok) != 0;
                umma::fence_after_sync();
                if (dead) break;
                if (L == 0) {
                    ph_in ^= 1u;
                    pend_in = false;
                }
                ph_w ^= 1u;
                pend_w = false;
            }
            if (tid == 0) {
                const uint32_t a = umma::smem_u32(sA), b = umma::smem_u32(sWt);
#pragma unroll
                for (int k0 = 0; k0 < JW; k0 += 16)
                    umma::mma16(tmem, umma::desc_at(a, 128, k0), umma::desc_at(b, 128, k0), idesc, 1u);
                umma::commit(&bar_mma);
            }
            pend_mma = true;
            {
                const bool ok = umma::mbar_wait(&bar_mma, ph_mma, wait_ns);
                umma::fence_before_sync();
                dead = __syncthreads_or(!ok) != 0;
                umma::fence_after_sync();
                if (dead) break;
                ph_mma ^= 1u;
                pend_mma = false;
            }
            if (tid == 0) {  // the slot and (after the last layer) sA are free again
                if (k + 1 < uses) load_weight(k + 1);
                if (L == 3 && t + gridDim.x < ntiles) load_pooled(t + gridDim.x);
            }
            // epilogue: the row's statistics over two 64-column halves, then
            // LayerNorm and GELU over the halves read again; the fp32 steps
            // run on column pairs (add / fma .f32x2), partial sums kept by
            // column mod 4 as four scalar chains would be
            const unsigned long long* cb2 = reinterpret_cast<const unsigned long long*>(vec[L]);  // bias sum pairs
            unsigned long long s2[2] = {0ull, 0ull}, q2[2] = {0ull, 0ull};
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                uint32_t zr[64];
                umma::tmem_ld32_nowait(tmem + lane_off + 64 * hf, zr);
                umma::tmem_ld32_nowait(tmem + lane_off + 64 * hf + 32, zr + 32);
                umma::tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 64; ++c) asm volatile("" : "+r"(zr[c]));  // the values exist after the wait
#pragma unroll
                for (int c = 0; c < 64; c += 2) {
                    unsigned long long x = umma::f2(zr[c], zr[c + 1]);
                    if (L) x = umma::f2_add(x, cb2[(64 * hf + c) / 2]);
                    s2[(c >> 1) & 1] = umma::f2_add(s2[(c >> 1) & 1], x);
                    q2[(c >> 1) & 1] = umma::f2_fma(x, x, q2[(c >> 1) & 1]);
                }
            }
            const float s = (umma::f2_lo(s2[0]) + umma::f2_hi(s2[0])) + (umma::f2_lo(s2[1]) + umma::f2_hi(s2[1]));
            const float sq = (umma::f2_lo(q2[0]) + umma::f2_hi(q2[0])) + (umma::f2_lo(q2[1]) + umma::f2_hi(q2[1]));
            const float mean = s * (1.0f / JW);
            const float inv = rsqrtf(fmaxf(sq * (1.0f / JW) - mean * mean, 0.0f) + 1e-5f);
            const float nm = -mean * inv;
            const unsigned long long inv2 = umma::f2(inv, inv), nm2 = umma::f2(nm, nm);
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                uint32_t zr[64];
                umma::tmem_ld32_nowait(tmem + lane_off + 64 * hf, zr);
                umma::tmem_ld32_nowait(tmem + lane_off + 64 * hf + 32, zr + 32);
                umma::tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 64; ++c) asm volatile("" : "+r"(zr[c]));
#pragma unroll
                for (int c8 = 0; c8 < 8; ++c8) {
                    uint32_t w4[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int c = 8 * c8 + 2 * j, cc = 64 * hf + c;
                        unsigned long long x = umma::f2(zr[c], zr[c + 1]);
                        if (L) x = umma::f2_add(x, cb2[cc / 2]);
                        const unsigned long long n = umma::f2_fma(x, inv2, nm2);
                        w4[j] = umma::ln_gelu2<H>(umma::f2_lo(n), umma::f2_hi(n), cc, gb2[L]);
                    }
                    const uint4 o = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                    const uint32_t off = umma::sw128_offset(128, tid, 64 * hf + 8 * c8);
                    if (L < 3)
                        *reinterpret_cast<uint4*>(sA + off) = o;
                    else
                        *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(zout_img) + (size_t)t * TILE_J + off) = o;
                }
            }
            if (L < 3) {  // the next layer's operand wait is the barrier
                umma::fence_async_smem();
                umma::fence_before_sync();
            }
        }
        if (dead) break;
        __syncthreads();
    }
    // Copies and a product still in flight after an early exit complete on
    // their own and must land before the shared memory and the tensor memory
    // go away. A drain that does not finish leaves the tensor memory
    // allocated and reports code 11: the device context can no longer be
    // trusted.
    if (tid == 0) {
        bool drained = true;
        if (pend_mma) drained = umma::mbar_wait(&bar_mma, ph_mma, umma::DRAIN_NS) && drained;
        if (pend_in) drained = umma::mbar_wait(&bar_in, ph_in, umma::DRAIN_NS) && drained;
        if (pend_w) drained = umma::mbar_wait(&bar_w, ph_w, umma::DRAIN_NS) && drained;
        abort_flag = drained ? 0 : 1;
        if (dead || !drained) atomicExch(err, drained ? 1 : 11);
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (warp == 0 && !abort_flag) umma::tmem_dealloc(tmem, 128);
}

// Pooled belief embeddings (search.rs:1512-1547) of one 128-row tile on the
// tensor cores: pooled_q = beta_q G_q, where beta_q[row][c] is the row's
// normalised reach on config c (player q's configs, by index; about 20 of
// ~110 nonzero per row) and G_q[c] = g(c). One thread per row computes its
// reach mass (kept: it is the opponent mass of the other player's readout)
// and scatters its normalised weights into a zeroed 128 x 128 A tile in
// shared memory; the job's g table arrives as a 64 x 128 B image by bulk
// copy; one MMA per 128 configs accumulates D = beta G (64 columns of TMEM),
// which becomes the player's 64-column atom of the tile's pooled image.
template <bool H>
__global__ void __launch_bounds__(128, 4)
    k_pool_fast(const JobDev* __restrict__ jobs, const HeadTile* __restrict__ tiles, uint32_t ntiles, int mask,
                uint16_t* __restrict__ pool_img, float* __restrict__ mass, int* __restrict__ err, uint64_t wait_ns) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t bar_g, bar_mma;
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    if (umma::misaligned16(pool_img)) {  // entry self-check: a launch contract broken, nothing touched
        if (threadIdx.x == 0) atomicExch(err, 32);
        return;
    }
    uint8_t* smem = align1024(smem_raw);
    uint8_t* sBeta = smem;           // [128 rows][128 configs]: 32 KB
    uint8_t* sG = smem + TILE_J;     // [64 features][128 configs]: 16 KB
    const int tid = threadIdx.x, warp = tid >> 5;
    if (tid == 0) {
        umma::mbar_init(&bar_g, 1);
        umma::mbar_init(&bar_mma, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        abort_flag = 0;
    }
    if (warp == 0) umma::tmem_alloc(&tmem_slot, 64);
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = tmem_slot;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const uint32_t idesc = umma::idesc16(128, 64, umma::Op16<H>::fmt);
    // Parities and pending work as in the join: the same in every thread
    // (pend_g is thread 0's, which issues the copy), stop decisions
    // block-uniform, nothing issued after a failed wait.
    uint32_t ph_g = 0, ph_mma = 0;
    bool pend_g = false, pend_mma = false, dead = false;
    for (uint32_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const HeadTile ht = tiles[t];
        const JobDev& J = jobs[ht.job];
        const bool valid = (uint32_t)tid < ht.count;
        const uint32_t r = ht.first + tid;
        for (int q = 0; q < 2; ++q) {
            if (!(mask & (1 << q))) continue;
            const uint32_t ncq = J.ncfg_player[q], nchunk = (ncq + 127) / 128;
            const float* w = nullptr;
            const uint32_t* lc = nullptr;
            uint32_t n = 0;
            float scale = 0.0f, flat = 0.0f;
            // the row's first EC entries, all loads issued at once (a typical
            // row has ~20), kept in registers for the scatter
            constexpr int EC = 24;
            float wr[EC];
            uint32_t cr[EC];
#pragma unroll
            for (int k = 0; k < EC; ++k) {
                wr[k] = 0.0f;
                cr[k] = 0xffffffffu;
            }
            if (valid) {  // one thread per row: its reach mass and normaliser
                w = J.reach + J.lr_ridx[2 * r + q];
                n = J.lr_nc[2 * r + q];
                lc = J.leaf_col + J.leaf_coff[2 * r + q];
#pragma unroll
                for (int k = 0; k < EC; ++k)
                    if ((uint32_t)k < n) {
                        wr[k] = w[k];
                        cr[k] = lc[k];
                    }
                float tot = 0.0f;
#pragma unroll
                for (int k = 0; k < EC; ++k) tot += wr[k];
                for (uint32_t e = EC; e < n; ++e) tot += w[e];
                mass[(size_t)(J.row_base + r) * 2 + q] = tot;
                if (tot > 1e-30f) scale = 1.0f / tot;
                else flat = 1.0f / (float)(n > 0 ? n : 1);
            }
            const uint8_t* gsrc = reinterpret_cast<const uint8_t*>(J.g16) +
                                  (q == 1 ? (J.ncfg_player[0] + 127) / 128 : 0) * (size_t)ATOM;
            for (uint32_t c = 0; c < nchunk; ++c) {
                if (tid == 0) {
                    umma::expect_tx(&bar_g, ATOM);
                    umma::bulk_g2s(sG, gsrc + (size_t)c * ATOM, ATOM, &bar_g);
                    pend_g = true;
                }
#pragma unroll
                for (int k = 0; k < 128; k += 8)
                    *reinterpret_cast<uint4*>(sBeta + umma::sw128_offset(128, tid, k)) = make_uint4(0, 0, 0, 0);
#pragma unroll
                for (int k = 0; k < EC; ++k) {
                    const uint32_t col = cr[k] - 128 * c;
                    if (col < 128)
                        *reinterpret_cast<uint16_t*>(sBeta + umma::sw128_offset(128, tid, col)) =
                            umma::Op16<H>::one(wr[k] * scale + flat);
                }
                for (uint32_t e = EC; e < n; ++e) {
                    const uint32_t col = lc[e] - 128 * c;
                    if (col < 128)
                        *reinterpret_cast<uint16_t*>(sBeta + umma::sw128_offset(128, tid, col)) =
                            umma::Op16<H>::one(w[e] * scale + flat);
                }
                {  // the scatter is done and (thread 0) the g chunk has landed
                    bool ok = true;
                    if (tid == 0) ok = umma::mbar_wait(&bar_g, ph_g, wait_ns);
                    umma::fence_async_smem();
                    umma::fence_before_sync();
                    dead = __syncthreads_or(!ok) != 0;
                    umma::fence_after_sync();
                    if (dead) break;
                    ph_g ^= 1u;
                    pend_g = false;
                }
                if (tid == 0) {
                    const uint32_t a = umma::smem_u32(sBeta), b = umma::smem_u32(sG);
#pragma unroll
                    for (int k0 = 0; k0 < 128; k0 += 16)
                        umma::mma16(tmem, umma::desc_at(a, 128, k0), umma::desc_at(b, 64, k0), idesc,
                                    (c > 0 || k0 > 0) ? 1u : 0u);
                    umma::commit(&bar_mma);
                }
                pend_mma = true;
                {
                    const bool ok = umma::mbar_wait(&bar_mma, ph_mma, wait_ns);
                    umma::fence_before_sync();
                    dead = __syncthreads_or(!ok) != 0;
                    umma::fence_after_sync();
                    if (dead) break;
                    ph_mma ^= 1u;
                    pend_mma = false;
                }
            }
            if (dead) break;
            // the row of the player's pooled atom in the tile image
            uint8_t* img = reinterpret_cast<uint8_t*>(pool_img) + (size_t)t * (2 * ATOM) + q * ATOM + tid * 128;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float v[32];
                if (nchunk) umma::tmem_ld32(tmem + lane_off + 32 * h, v);
                else
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = 0.0f;
#pragma unroll
                for (int c8 = 0; c8 < 4; ++c8) {
                    const uint32_t chunk = 4 * h + c8;
                    *reinterpret_cast<uint4*>(img + ((chunk ^ (tid & 7)) << 4)) = umma::pack_chunk<H>(v + 8 * c8);
                }
            }
            umma::fence_before_sync();
            __syncthreads();  // TMEM and sBeta are reused by the next player or tile
            umma::fence_after_sync();
        }
        if (dead) break;
    }
    // Drain what an early exit left in flight; code 14 when a drain does not
    // finish (the tensor memory then stays allocated).
    if (tid == 0) {
        bool drained = true;
        if (pend_mma) drained = umma::mbar_wait(&bar_mma, ph_mma, umma::DRAIN_NS) && drained;
        if (pend_g) drained = umma::mbar_wait(&bar_g, ph_g, umma::DRAIN_NS) && drained;
        abort_flag = drained ? 0 : 1;
        if (dead || !drained) atomicExch(err, drained ? 4 : 14);
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (warp == 0 && !abort_flag) umma::tmem_dealloc(tmem, 64);
}

// The join output layer, the readout LayerNorm and the per-config readout for
// traverser p (net.rs:833-853, search.rs:1587-1636):
// y = P + out * Wout + bout, h = LN(y), v(c) = (<f(c), h> + bias) * opp_reach.
// Two tensor-core products per 128-row tile: Y = out * Wout (A = the join
// output image in shared memory) and the readout V = H * F_p^T against the
// job's player-p f table (128 configs per pass), with H = LN(y) written by
// the epilogue into tensor memory as that product's A operand (f16: the
// readout is the product most sensitive to operand rounding). The P rows
// (which already include bout) arrive per tile by bulk copy, stored by the
// trunk as 64 KB tile images: row r at r * 512 bytes, its 16-byte chunk k at
// chunk k ^ (r & 7), so the epilogue's row-per-lane reads are conflict-free.
//
// Warp roles. Warps 0..15 run the epilogue: warp w owns rows 32 (w % 4) ..
// and the column group w / 4 (64 of y's 256 columns, 32 of each pass's
// configs). Warp 16 issues every bulk copy and product (issuing a product
// holds the issuing thread for most of its duration, so no epilogue warp
// waits on it). Handoffs: the products and copies arrive on mbarriers the
// epilogue waits for; the epilogue warps arrive on `h_ready` (H written, Y
// and P read) and `s_done` (a pass's staging read and scattered). While the
// epilogue scatters tile t, the next tile's Y product runs and its P image
// lands; its join-output image landed during tile t's epilogue; the row
// tables of the tile after next are prefetched into L2.
// TMEM: Y in columns 0..255, V in 256..383, H in 384..511; during the
// epilogue, V's first columns carry the LayerNorm partials.
template <bool H>
__global__ void __launch_bounds__(544, 1)
    k_head_fast(const JobDev* __restrict__ jobs, const HeadTile* __restrict__ tiles, uint32_t ntiles, FastNetDev fn,
                int p, const uint16_t* __restrict__ zout, const uint16_t* __restrict__ pimg,
                const float* __restrict__ mass, int* __restrict__ err) {
    constexpr uint32_t TY = 0, TV = 256, TH = 384;
    constexpr uint32_t NWORK = 512;  // epilogue threads
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t bar_y, bar_v, bar_a, bar_f, bar_p, h_ready, s_done;
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag, stuck;
    // f16: the LayerNorm's (gamma, beta) per column pair, packed; read as
    // uint2, so the array needs 8-byte alignment (a uint32_t array alone is
    // only guaranteed 4)
    __shared__ __align__(16) uint32_t gb2[D];
    if (umma::misaligned16(fn.out_tile) || umma::misaligned16(zout) || umma::misaligned16(pimg)) {
        if (threadIdx.x == 0) atomicExch(err, 33);  // entry self-check: a launch contract broken
        return;
    }
    uint8_t* smem = align1024(smem_raw);
    uint8_t* sW = smem;                  // [256][128] Wout: 64 KB
    uint8_t* sF = sW + 2 * TILE_J;       // [128][256] f image of a pass, then its staging: 64 KB
    uint8_t* sP = sF + 2 * TILE_J;       // [128][256] P tile image: 64 KB
    uint8_t* sA = sP + 2 * TILE_J;       // [128][128] join-output image: 32 KB
    float* stage = reinterpret_cast<float*>(sF);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    {
        const uint4* src = reinterpret_cast<const uint4*>(fn.out_tile);
        uint4* dst = reinterpret_cast<uint4*>(sW);
        for (uint32_t i = tid; i < 2 * TILE_J / 16; i += blockDim.x) dst[i] = src[i];
        for (int c = 2 * tid; c < D; c += 2 * blockDim.x) umma::pack_gb2(fn.ln_g[4], fn.ln_b[4], c, &gb2[c]);
    }
    if (tid == 0) {
        umma::mbar_init(&bar_y, 1);
        umma::mbar_init(&bar_v, 1);
        umma::mbar_init(&bar_a, 1);
        umma::mbar_init(&bar_f, 1);
        umma::mbar_init(&bar_p, 1);
        umma::mbar_init(&h_ready, NWORK / 32);
        umma::mbar_init(&s_done, NWORK / 32);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        abort_flag = 0;
        stuck = 0;
    }
    if (warp == 16) umma::tmem_alloc(&tmem_slot, 512);
    umma::fence_async_smem();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = tmem_slot;
    volatile int* abort_v = &abort_flag;
    const uint64_t wait_ns = fn.wait_ns;
    // a bounded wait that also gives up as soon as another thread has
    // recorded an abort (so no role waits out its limit on a dead partner)
    auto wait = [&](uint64_t* bar, uint32_t parity) {
        const uint32_t addr = umma::smem_u32(bar);
        if (umma::mbar_test(addr, parity)) return true;
        const uint64_t t0 = umma::now_ns();
        for (uint32_t i = 1;; ++i) {
            if (umma::mbar_test(addr, parity)) return true;
            if ((i & 15u) == 0u) {
                if (*abort_v) return false;
                if (umma::now_ns() - t0 >= wait_ns) break;
            }
        }
        *abort_v = 1;
        return false;
    };

    if (warp == 16) {
        // ------------------------------------------------------ the issuer
        if (lane == 0) {
            uint32_t ph_y = 0, ph_a = 0, ph_f = 0, ph_h = 0, ph_s = 0;
            bool pend_a = false, pend_f = false, pend_p = false, pend_y = false, pend_v = false;
            uint32_t ph_v = 0, ph_p = 0;
            auto load_a = [&](uint32_t t) {
                const uint8_t* src = reinterpret_cast<const uint8_t*>(zout) + (size_t)t * TILE_J;
                umma::expect_tx(&bar_a, TILE_J);
                umma::bulk_g2s(sA, src, ATOM, &bar_a);
                umma::bulk_g2s(sA + ATOM, src + ATOM, ATOM, &bar_a);
                pend_a = true;
            };
            auto load_p = [&](uint32_t t) {
                const uint32_t bytes = tiles[t].count * 512u;
                const uint8_t* src = reinterpret_cast<const uint8_t*>(pimg) + (size_t)t * 2 * TILE_J;
                umma::expect_tx(&bar_p, bytes);
                for (uint32_t o = 0; o < bytes; o += ATOM)
                    umma::bulk_g2s(sP + o, src + o, bytes - o < ATOM ? bytes - o : ATOM, &bar_p);
                pend_p = true;
                ph_p ^= 1u;   // the epilogue waits for it; tracked here for the exit
            };
            auto load_f = [&](uint32_t job, uint32_t pass) {
                const JobDev& J = jobs[job];
                const uint8_t* src = reinterpret_cast<const uint8_t*>(J.f16) +
                                     ((p == 1 ? (J.ncfg_player[0] + 127) / 128 : 0) + pass) * (size_t)(2 * TILE_J);
                umma::expect_tx(&bar_f, 2 * TILE_J);
                for (uint32_t o = 0; o < 2 * TILE_J; o += ATOM) umma::bulk_g2s(sF + o, src + o, ATOM, &bar_f);
                pend_f = true;
            };
            auto prefetch_rows = [&](uint32_t t) {
                const HeadTile ht = tiles[t];
                const JobDev& J = jobs[ht.job];
                umma::bulk_prefetch_l2(mass + ((size_t)J.row_base + ht.first) * 2, (size_t)ht.count * 8);
                umma::bulk_prefetch_l2(J.lr_nc + 2 * (size_t)ht.first, (size_t)ht.count * 8);
                umma::bulk_prefetch_l2(J.leaf_coff + 2 * (size_t)ht.first, (size_t)ht.count * 8);
                umma::bulk_prefetch_l2(J.lr_vidx + 2 * (size_t)ht.first, (size_t)ht.count * 8);
            };
            auto issue_y = [&]() -> bool {
                if (!wait(&bar_a, ph_a)) return false;
                ph_a ^= 1u;
                pend_a = false;
                umma::fence_after_sync();
                const uint32_t wa = umma::smem_u32(sA), wb = umma::smem_u32(sW);
                const uint32_t idesc = umma::idesc16(128, 256, umma::Op16<H>::fmt);
#pragma unroll
                for (int k0 = 0; k0 < JW; k0 += 16)
                    umma::mma16(tmem + TY, umma::desc_at(wa, 128, k0), umma::desc_at(wb, 256, k0), idesc, k0 > 0);
                umma::commit(&bar_y);
                pend_y = true;
                return true;
            };
            auto issue_v = [&]() -> bool {
                if (!wait(&bar_f, ph_f)) return false;
                ph_f ^= 1u;
                pend_f = false;
                umma::fence_after_sync();
                const uint32_t fa = umma::smem_u32(sF);
                const uint32_t idesc = umma::idesc16(128, 128, umma::Op16<true>::fmt);  // H, f(c): f16
#pragma unroll
                for (int k0 = 0; k0 < D; k0 += 16)
                    umma::mma16_ts(tmem + TV, tmem + TH + k0 / 2, umma::desc_at(fa, 128, k0), idesc, k0 > 0);
                umma::commit(&bar_v);
                pend_v = true;
                ph_v ^= 1u;
                return true;
            };
            const uint32_t G = gridDim.x;
            uint32_t t = blockIdx.x;
            bool ok = true;
            if (t < ntiles) {
                load_a(t);
                load_p(t);
                const uint32_t j0 = tiles[t].job;
                if (jobs[j0].ncfg_player[p]) load_f(j0, 0);
                if (t + G < ntiles) prefetch_rows(t + G);
                ok = issue_y();
            }
            for (; ok && t < ntiles; t += G) {
                const uint32_t tn = t + G;
                const HeadTile ht = tiles[t];
                const uint32_t npass = (jobs[ht.job].ncfg_player[p] + 127) / 128;
                // Y(t) done: its join-output image has been read
                if (!(ok = wait(&bar_y, ph_y))) break;
                ph_y ^= 1u;
                pend_y = false;
                if (tn < ntiles) load_a(tn);
                if (tn + G < ntiles) prefetch_rows(tn + G);
                // the epilogue has read Y(t) and P(t) and written H(t)
                if (!(ok = wait(&h_ready, ph_h))) break;
                ph_h ^= 1u;
                pend_p = false;
                umma::fence_after_sync();
                if (tn < ntiles) load_p(tn);
                if (npass && !(ok = issue_v())) break;
                if (tn < ntiles && !(ok = issue_y())) break;
                for (uint32_t k = 0; k < npass; ++k) {
                    // pass k's staging has been read and V consumed: sF is free
                    if (!(ok = wait(&s_done, ph_s))) break;
                    ph_s ^= 1u;
                    pend_v = false;
                    umma::fence_after_sync();
                    if (k + 1 < npass) {
                        load_f(ht.job, k + 1);
                        if (!(ok = issue_v())) break;
                    }
                }
                if (!ok) break;
                if (tn < ntiles) {
                    const uint32_t jn = tiles[tn].job;
                    if (jobs[jn].ncfg_player[p]) load_f(jn, 0);
                }
            }
            // nothing may be in flight when the shared and tensor memory are
            // released: issued products and copies complete on their own.
            // A drain that does not finish leaves the tensor memory allocated
            // and reports code 12 (the device context can no longer be trusted).
            bool drained = true;
            if (pend_y) drained = umma::mbar_wait(&bar_y, ph_y, umma::DRAIN_NS) && drained;
            if (pend_v) drained = umma::mbar_wait(&bar_v, ph_v ^ 1u, umma::DRAIN_NS) && drained;
            if (pend_a) drained = umma::mbar_wait(&bar_a, ph_a, umma::DRAIN_NS) && drained;
            if (pend_f) drained = umma::mbar_wait(&bar_f, ph_f, umma::DRAIN_NS) && drained;
            if (pend_p) drained = umma::mbar_wait(&bar_p, ph_p ^ 1u, umma::DRAIN_NS) && drained;
            stuck = drained ? 0 : 1;
            if (!ok || !drained) atomicExch(err, drained ? 2 : 12);
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------- the epilogue
        const int quad = warp & 3, cg = warp >> 2;
        const int row = quad * 32 + lane;
        const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
        uint32_t ph_y = 0, ph_v = 0, ph_p = 0;
        bool bad = false;
        auto bar_or = [&](bool v) {   // named barrier over the epilogue threads, OR of v
            uint32_t r;
            asm volatile(
                "{\n\t.reg .pred p, q;\n\t"
                "setp.ne.u32 p, %1, 0;\n\t"
                "barrier.red.or.pred q, 1, 512, p;\n\t"
                "selp.u32 %0, 1, 0, q;\n\t}\n"
                : "=r"(r)
                : "r"((uint32_t)v)
                : "memory");
            return r != 0;
        };
        for (uint32_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
            const HeadTile ht = tiles[t];
            const JobDev& J = jobs[ht.job];
            const uint32_t npass = (J.ncfg_player[p] + 127) / 128;
            if (!wait(&bar_y, ph_y)) bad = true;
            ph_y ^= 1u;
            if (!wait(&bar_p, ph_p)) bad = true;
            ph_p ^= 1u;
            umma::fence_after_sync();
            // y = Y + P, in two 32-column halves: each half's mean and sum
            // of squared deviations, and y written back over Y (the fp32
            // steps on column pairs, add / fma .f32x2)
            float m2h[2], mh[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float v[32];
                umma::tmem_ld32(tmem + lane_off + TY + 64 * cg + 32 * h, v);
                unsigned long long s2[2] = {0ull, 0ull};
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint32_t k = (uint32_t)(8 * cg + 4 * h + c);
                    const uint4 q = *reinterpret_cast<const uint4*>(sP + row * 512 + 16 * (k ^ (uint32_t)(row & 7)));
                    const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const unsigned long long y = umma::f2_add(umma::f2(v[8 * c + 2 * i], v[8 * c + 2 * i + 1]),
                                                                  umma::f2(umma::Op16<true>::lo(w4[i]), umma::Op16<true>::hi(w4[i])));
                        v[8 * c + 2 * i] = umma::f2_lo(y);
                        v[8 * c + 2 * i + 1] = umma::f2_hi(y);
                        s2[i & 1] = umma::f2_add(s2[i & 1], y);
                    }
                }
                const float s = (umma::f2_lo(s2[0]) + umma::f2_hi(s2[0])) + (umma::f2_lo(s2[1]) + umma::f2_hi(s2[1]));
                const float m = s * (1.0f / 32);
                const unsigned long long nm2 = umma::f2(-m, -m);
                unsigned long long d2[2] = {0ull, 0ull};
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    const unsigned long long d = umma::f2_add(umma::f2(v[j], v[j + 1]), nm2);
                    d2[(j >> 1) & 1] = umma::f2_fma(d, d, d2[(j >> 1) & 1]);
                }
                mh[h] = m;
                m2h[h] = (umma::f2_lo(d2[0]) + umma::f2_hi(d2[0])) + (umma::f2_lo(d2[1]) + umma::f2_hi(d2[1]));
                umma::tmem_st32(tmem + lane_off + TY + 64 * cg + 32 * h, v);
            }
            // the row's four column groups meet through V's first columns
            {
                const float m = 0.5f * (mh[0] + mh[1]);
                const float m2 = m2h[0] + m2h[1] + 16.0f * (mh[0] - mh[1]) * (mh[0] - mh[1]);
                uint32_t w2[2] = {__float_as_uint(m), __float_as_uint(m2)};
                asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1, %2};" ::"r"(tmem + lane_off + TV + 2 * cg),
                             "r"(w2[0]), "r"(w2[1])
                             : "memory");
                umma::tmem_wait_st();
            }
            umma::fence_before_sync();
            if (bar_or(bad)) break;
            umma::fence_after_sync();
            float mean, inv;
            {
                uint32_t r8[8];
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                             : "=r"(r8[0]), "=r"(r8[1]), "=r"(r8[2]), "=r"(r8[3]), "=r"(r8[4]), "=r"(r8[5]),
                               "=r"(r8[6]), "=r"(r8[7])
                             : "r"(tmem + lane_off + TV));
                umma::tmem_wait_ld();
                float mc[4], m2 = 0.0f;
#pragma unroll
                for (int c = 0; c < 4; ++c) mc[c] = __uint_as_float(r8[2 * c]);
                mean = 0.25f * (mc[0] + mc[1] + mc[2] + mc[3]);
#pragma unroll
                for (int c = 0; c < 4; ++c) m2 += __uint_as_float(r8[2 * c + 1]) + 64.0f * (mc[c] - mean) * (mc[c] - mean);
                inv = rsqrtf(m2 * (1.0f / D) + 1e-5f);
            }
            // h = LN(y) as f16 pairs into H's TMEM columns (K = 64 cg ..)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float v[32];
                umma::tmem_ld32(tmem + lane_off + TY + 64 * cg + 32 * h, v);
                uint32_t hw[16];
                {
                    // the affine in f16x2 on the normalised pair (the result
                    // is an f16 operand either way)
                    const float nm = -mean * inv;
                    const unsigned long long inv2 = umma::f2(inv, inv), nmp = umma::f2(nm, nm);
#pragma unroll
                    for (int c = 0; c < 16; ++c) {
                        const uint2 gb = *reinterpret_cast<const uint2*>(&gb2[64 * cg + 32 * h + 2 * c]);
                        const unsigned long long y = umma::f2_fma(umma::f2(v[2 * c], v[2 * c + 1]), inv2, nmp);
                        const __half2 n = __floats2half2_rn(umma::f2_lo(y), umma::f2_hi(y));
                        const __half2 x = __hfma2(n, *reinterpret_cast<const __half2*>(&gb.x),
                                                  *reinterpret_cast<const __half2*>(&gb.y));
                        hw[c] = *reinterpret_cast<const uint32_t*>(&x);
                    }
                }
                asm volatile(
                    "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
                    "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(tmem + lane_off + TH + 32 * cg + 16 * h),
                    "r"(hw[0]), "r"(hw[1]), "r"(hw[2]), "r"(hw[3]), "r"(hw[4]), "r"(hw[5]), "r"(hw[6]), "r"(hw[7]),
                    "r"(hw[8]), "r"(hw[9]), "r"(hw[10]), "r"(hw[11]), "r"(hw[12]), "r"(hw[13]), "r"(hw[14]), "r"(hw[15])
                    : "memory");
            }
            umma::tmem_wait_st();
            umma::fence_async_smem();     // the P reads precede the next P image's bulk copy
            umma::fence_before_sync();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(umma::smem_u32(&h_ready)) : "memory");
            // the scatter: warp w writes the values of rows 8 w .. 8 w + 7, a
            // row's entries across the lanes (coalesced column reads and value
            // writes). Lane i < 8 holds row 8 w + i's opponent reach mass (kept
            // by the pooling kernel), entry count, readout columns and value
            // slots (prefetched into L2); colv[i] is entry `lane` of row
            // 8 w + i, all eight loaded at once, during the readout product.
            float s_mass = 0.0f;
            uint32_t s_nc = 0;
            unsigned long long s_lcol = 0, s_out = 0;
            if (lane < 8 && (uint32_t)(8 * warp + lane) < ht.count) {
                const uint32_t r = ht.first + 8 * warp + lane;      // job-local network row
                s_mass = mass[(size_t)(J.row_base + r) * 2 + 1 - p];
                s_nc = J.lr_nc[2 * r + p];
                s_lcol = reinterpret_cast<unsigned long long>(J.leaf_col + J.leaf_coff[2 * r + p]);
                s_out = reinterpret_cast<unsigned long long>(J.vals[p] + J.lr_vidx[2 * r + p]);
            }
            uint32_t colv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t nc = __shfl_sync(0xffffffffu, s_nc, i);
                const uint32_t* lc = reinterpret_cast<const uint32_t*>(__shfl_sync(0xffffffffu, s_lcol, i));
                colv[i] = (uint32_t)lane < nc ? lc[lane] : 0xffffffffu;
            }
            for (uint32_t k = 0; k < npass; ++k) {
                const uint32_t nb = 128 * k;
                if (!wait(&bar_v, ph_v)) bad = true;
                ph_v ^= 1u;
                umma::fence_after_sync();
                {
                    float v[32];
                    umma::tmem_ld32(tmem + lane_off + TV + 32 * cg, v);
                    float* st = stage + row * 128 + 32 * cg;
#pragma unroll
                    for (int j = 0; j < 32; ++j) st[j ^ lane] = v[j];
                }
                umma::fence_before_sync();
                if (bar_or(bad)) { bad = true; break; }
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    // staging row R was written with the XOR key R & 31
                    const int R = 8 * warp + i;
                    const float* st = stage + R * 128;
                    const uint32_t key = (uint32_t)(R & 31);
                    const float om = __shfl_sync(0xffffffffu, s_mass, i);
                    float* o = reinterpret_cast<float*>(__shfl_sync(0xffffffffu, s_out, i));
                    const uint32_t col = colv[i] - nb;
                    if (col < 128) o[lane] = (st[(col & ~31u) | ((col & 31u) ^ key)] + fn.vbias) * om;
                    const uint32_t nc = __shfl_sync(0xffffffffu, s_nc, i);
                    if (nc > 32) {  // the row's further entries
                        const uint32_t* lc = reinterpret_cast<const uint32_t*>(__shfl_sync(0xffffffffu, s_lcol, i));
                        for (uint32_t e = 32 + lane; e < nc; e += 32) {
                            const uint32_t c2 = lc[e] - nb;
                            if (c2 < 128) o[e] = (st[(c2 & ~31u) | ((c2 & 31u) ^ key)] + fn.vbias) * om;
                        }
                    }
                }
                umma::fence_async_smem();  // the staging reads precede the next bulk copy into sF
                __syncwarp();
                if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(umma::smem_u32(&s_done)) : "memory");
            }
            if (bad) break;
        }
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (warp == 16 && !stuck) umma::tmem_dealloc(tmem, 512);
}

// f(c) of every config as the readout's B-operand images: for each player,
// passes of 128 configs (by index among the player's configs) x 256, K-major
// and 128-byte swizzled; player 0's passes first, always f16 (the readout's
// operand type). Likewise g(c) as the pooling's B images (64 features x 128
// configs) in the chain's type H.
template <bool H>
__global__ void k_pack_f16(const JobDev* __restrict__ jobs, const uint32_t* __restrict__ cfg_job,
                           const uint32_t* __restrict__ cfg_local, uint32_t total_cfgs) {
    const uint32_t e = blockIdx.x;
    if (e >= total_cfgs) return;
    const JobDev& J = jobs[cfg_job[e]];
    const uint32_t c = cfg_local[e];
    const uint32_t col = J.cfg_col[c], i = col & 127;
    uint8_t* img = reinterpret_cast<uint8_t*>(J.f16) +
                   ((J.cplayer[c] == 1 ? (J.ncfg_player[0] + 127) / 128 : 0) + (col >> 7)) * (size_t)(2 * TILE_J);
    for (int j = threadIdx.x; j < D; j += blockDim.x)
        *reinterpret_cast<uint16_t*>(img + umma::sw128_offset(128, i, j)) = umma::Op16<true>::one(J.cf[(size_t)c * D + j]);
    // g(c) into the pooling B image: row = feature, K = config index
    uint8_t* gimg = reinterpret_cast<uint8_t*>(J.g16) +
                    ((J.cplayer[c] == 1 ? (J.ncfg_player[0] + 127) / 128 : 0) + (col >> 7)) * (size_t)ATOM;
    for (int j = threadIdx.x; j < POOL; j += blockDim.x)
        *reinterpret_cast<uint16_t*>(gimg + umma::sw128_offset(64, j, i)) = umma::Op16<H>::one(J.cg[(size_t)c * POOL + j]);
}

static int num_sms() {
    int dev = 0, n = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

void launch_pool_fast(const JobDev* jobs, const void* tiles, uint32_t ntiles, int mask, uint16_t* pool_img, float* mass,
                      bool half, int* err, uint64_t wait_ns, cudaStream_t s) {
    if (!ntiles || !mask) return;
    const size_t smem = TILE_J + ATOM + 1024;
    auto kern = half ? k_pool_fast<true> : k_pool_fast<false>;
    if (!raise_smem_limit((const void*)kern, smem)) return;
    const uint32_t grid = std::min<uint32_t>(ntiles, 4u * (uint32_t)num_sms());
    kern<<<grid, 128, smem, s>>>(jobs, reinterpret_cast<const HeadTile*>(tiles), ntiles, mask, pool_img, mass, err,
                                 wait_ns);
}

bool raise_smem_limit(const void* fn, size_t smem) {
    static std::mutex mu;
    static std::set<std::pair<int, const void*>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (done.count({dev, fn})) return true;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return false;
    done.insert({dev, fn});
    return true;
}

void launch_join_fast(const JobDev* jobs, const void* tiles, uint32_t ntiles, const FastNetDev& fn, int p,
                      const uint16_t* pool_img, const uint16_t* jp, uint16_t* zout_img, int* err, cudaStream_t s) {
    if (!ntiles) return;
    const size_t smem = 2 * TILE_J + 8 * JW * 4 + 1024;  // the weight slot, the A operand, the vectors
    auto kern = fn.half ? k_join_fast<true> : k_join_fast<false>;
    if (!raise_smem_limit((const void*)kern, smem)) return;
    uint32_t grid = std::min<uint32_t>(ntiles, 3u * (uint32_t)num_sms());
    kern<<<grid, 128, smem, s>>>(jobs, reinterpret_cast<const HeadTile*>(tiles), ntiles, fn, p, pool_img, jp, zout_img,
                                 err);
}

void launch_head_fast(const JobDev* jobs, const void* tiles, uint32_t ntiles, const FastNetDev& fn, int p,
                      const uint16_t* zout, const uint16_t* pb, const float* mass, int* err, cudaStream_t s) {
    if (!ntiles) return;
    const size_t smem = 7 * TILE_J + 1024;
    auto kern = fn.half ? k_head_fast<true> : k_head_fast<false>;
    if (!raise_smem_limit((const void*)kern, smem)) return;
    uint32_t grid = std::min<uint32_t>(ntiles, (uint32_t)num_sms());
    kern<<<grid, 544, smem, s>>>(jobs, reinterpret_cast<const HeadTile*>(tiles), ntiles, fn, p, zout, pb, mass, err);
}

void launch_pack_f16(const JobDev* jobs, const uint32_t* cfg_job, const uint32_t* cfg_local, uint32_t total_cfgs,
                     bool half, cudaStream_t s) {
    if (!total_cfgs) return;
    if (half) k_pack_f16<true><<<total_cfgs, 128, 0, s>>>(jobs, cfg_job, cfg_local, total_cfgs);
    else k_pack_f16<false><<<total_cfgs, 128, 0, s>>>(jobs, cfg_job, cfg_local, total_cfgs);
}

int umma_selftest(const uint16_t* A, const uint16_t* B, int K, int N, float* D) {
    if (K <= 0 || K % 64 || N % 16 || N < 16 || N > 256) return 1;
    const size_t a_bytes = 128ull * K * 2, b_bytes = (size_t)N * K * 2, d_bytes = 128ull * N * 4;
    const size_t smem = a_bytes + b_bytes + 1024;
    if (smem > (size_t)SELFTEST_SMEM_MAX) return 1;
    __nv_bfloat16 *dA = nullptr, *dB = nullptr;
    float* dD = nullptr;
    int* dS = nullptr;
    int status = 0, rc = 0;
    if (cudaMalloc(&dA, a_bytes) != cudaSuccess || cudaMalloc(&dB, b_bytes) != cudaSuccess ||
        cudaMalloc(&dD, d_bytes) != cudaSuccess || cudaMalloc(&dS, 4) != cudaSuccess ||
        cudaMemcpy(dA, A, a_bytes, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dB, B, b_bytes, cudaMemcpyHostToDevice) != cudaSuccess || cudaMemset(dS, 0, 4) != cudaSuccess ||
        cudaFuncSetAttribute(k_umma_selftest, cudaFuncAttributeMaxDynamicSharedMemorySize, SELFTEST_SMEM_MAX) !=
            cudaSuccess) {
        rc = 2;
    } else {
        k_umma_selftest<<<1, 128, smem>>>(dA, dB, K, N, dD, dS);
        if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
            cudaMemcpy(D, dD, d_bytes, cudaMemcpyDeviceToHost) != cudaSuccess ||
            cudaMemcpy(&status, dS, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
            rc = 2;
        else if (status)
            rc = 3;
    }
    cudaFree(dA);
    cudaFree(dB);
    cudaFree(dD);
    cudaFree(dS);
    return rc;
}

// ------------------------------------------ allocation-free GEMM self-test
// The same tcgen05 self-test as umma_selftest, for callers that must not
// allocate device memory: a host engine whose device memory belongs to another
// allocator (a caching allocator that owns the free memory, or a fixed arena
// sized at start-up), and callers on a latency-bound path, where cudaMalloc
// and cudaFree would synchronise the device and stall every other stream.
// Instead of four cudaMalloc'd buffers, the operands, the result and the
// status word live in one file-scope device array sized for the largest
// accepted problem (k = n = 256): 320.25 KB, held by every GPU that loads
// this library until the process exits.
constexpr size_t SCR_STATUS = 0, SCR_A = 256, SCR_B = SCR_A + 128 * 256 * 2, SCR_D = SCR_B + 256 * 256 * 2;
constexpr size_t STATIC_SCRATCH_BYTES = SCR_D + 128 * 256 * 4;  // 327,936 bytes
static __device__ __align__(256) uint8_t g_gemm_scratch[STATIC_SCRATCH_BYTES];

// Per-device set-up of the static path: the device address of
// g_gemm_scratch (host code cannot use the array's name as a device pointer:
// it names a host-side stand-in) and a private non-blocking stream, so the
// call synchronises with nothing but its own work. Done once per device, on
// that device's first call, with the device current.
struct StaticSetup {
    uint8_t* scratch = nullptr;
    cudaStream_t stream = nullptr;
};

static bool static_setup(StaticSetup* out) {
    static std::mutex mu;
    static std::map<int, StaticSetup> per_dev;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    std::lock_guard<std::mutex> lock(mu);
    auto it = per_dev.find(dev);
    if (it != per_dev.end()) {
        *out = it->second;
        return true;
    }
    StaticSetup st;
    if (cudaGetSymbolAddress((void**)&st.scratch, g_gemm_scratch) != cudaSuccess) return false;
    if (cudaStreamCreateWithFlags(&st.stream, cudaStreamNonBlocking) != cudaSuccess) return false;
    per_dev[dev] = st;
    *out = st;
    return true;
}

int umma_selftest_static(const uint16_t* A, const uint16_t* B, int K, int N, float* D) {
    if (K <= 0 || K % 64 || N % 16 || N < 16 || N > 256) return 1;
    if (K > 256) return 4;  // beyond the static scratch
    StaticSetup st;
    if (!static_setup(&st)) return 5;
    uint8_t* scr = st.scratch;
    cudaStream_t s = st.stream;
    const size_t a_bytes = 128ull * K * 2, b_bytes = (size_t)N * K * 2, d_bytes = 128ull * N * 4;
    auto* dA = reinterpret_cast<__nv_bfloat16*>(scr + SCR_A);
    auto* dB = reinterpret_cast<__nv_bfloat16*>(scr + SCR_B);
    auto* dD = reinterpret_cast<float*>(scr + SCR_D);
    auto* dS = reinterpret_cast<int*>(scr + SCR_STATUS);
    // The array keeps the previous call's contents: A and B are rewritten in
    // full, D in full by a successful kernel, and the status word must start
    // at zero.
    if (cudaMemcpyAsync(dA, A, a_bytes, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(dB, B, b_bytes, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemsetAsync(dS, 0, 4, s) != cudaSuccess)
        return 2;
    if (cudaFuncSetAttribute(k_umma_selftest, cudaFuncAttributeMaxDynamicSharedMemorySize, SELFTEST_SMEM_MAX) !=
        cudaSuccess)
        return 2;
    const size_t smem = a_bytes + b_bytes + 1024;
    k_umma_selftest<<<1, 128, smem, s>>>(dA, dB, K, N, dD, dS);
    if (cudaGetLastError() != cudaSuccess) return 2;  // not launched: D would be a previous call's
    int status = 0;
    if (cudaMemcpyAsync(D, dD, d_bytes, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyAsync(&status, dS, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return 2;
    return status ? 3 : 0;
}

}  // namespace wcdev
