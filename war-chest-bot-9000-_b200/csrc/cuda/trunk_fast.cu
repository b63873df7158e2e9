// The board trunk on the tensor cores (net.rs:558-731): tokens and stem,
// eight residual blocks, the final norm, the board readout P and the join
// projection jp, for three boards (111 hex rows, padded to M = 128) per tile.
//
// Each CTA keeps the residual stream x of its tile in registers: 12 warps,
// warp w owns TMEM lanes 32 (w % 4) .. + 31 (hex rows) and columns
// 32 (w / 4) .. + 31. Per block the two GEMMs run on tcgen05:
//   mix: [a | sum of the six neighbours' a] (K = 192) x W_mix (N = 96)
//   out: LNGELU(y) (K = 96) x W_out (N = 96)
// with the block's weight tiles streamed from global memory by bulk
// asynchronous copies into two shared-memory buffers (the next block's
// weights land while this block computes). The per-board pooling GEMM,
// the stem and the board readout are small and run on the CUDA cores with
// fp32 weights.
//
// The operands of both products, and the stored rows P and jp, are f16 in
// either tensor-core network mode: the trunk runs once per solve (its cost
// does not scale with the iterations), and its error reaches every leaf
// value through the near-orthogonal readout <f(c), h>, which amplifies it
// several times; bf16 operands here alone put the leaf values near 1e-2
// relative error, f16 (three more mantissa bits) keeps them near 1e-3.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "../host/netlayout.h"
#include "device.h"
#include "kernels.h"
#include "umma.cuh"

namespace wcdev {

using wc::NetLayout;

__constant__ NetLayout c_Lt;
__constant__ uint8_t c_nbt[37][6];
__constant__ uint8_t c_islt[37];

namespace {

constexpr int NH = 37, BOARDS = 3, ROWS = BOARDS * NH;  // 111 real rows per tile
constexpr int C = wc::NET_C, TYPE = wc::NET_TYPE, D = wc::NET_D, JW = wc::NET_JW;
constexpr int NTYPE = 10, NSLOT = 5, HEX_FACTS = 6, LOOSE = 15, PILE = 4;
constexpr uint32_t MIX_BYTES = 96 * 3 * 128;   // [96][192] swizzled: 3 atoms
constexpr uint32_t OUT_BYTES = 96 * 2 * 128;   // [96][96]: 2 atoms (second half used)
constexpr uint32_t BLOCK_BYTES = MIX_BYTES + OUT_BYTES;  // 61440
constexpr uint32_t A1_BYTES = 128 * 3 * 128;   // [128][192]
constexpr uint32_t A2_BYTES = 128 * 2 * 128;   // [128][96]
using F16 = umma::Op16<true>;

// One elected thread: fetch a block's weight tiles into `dst`.
__device__ __forceinline__ void fetch_block(uint8_t* dst, const uint8_t* tiles, int blk, uint64_t* bar) {
    umma::expect_tx(bar, BLOCK_BYTES);
    const uint8_t* src = tiles + (size_t)blk * BLOCK_BYTES;
    for (uint32_t o = 0; o < BLOCK_BYTES; o += 15360) umma::bulk_g2s(dst + o, src + o, 15360, bar);
}

// out[i][n] = bias[n] + sum_k in[i][k] * W[k][n] for the NB rows of a tile, on
// the CUDA cores: one thread per (column n, K slice), the NB rows in
// registers so every weight load feeds NB FMAs, and the loads unrolled so
// several are in flight (the weights come from L2). With KS > 1 the K slices
// meet in `part` (KS * NB * N floats). `in` has row stride ldi, `out` ldo.
// With RS > 1 (and KS == 1) the rows are split into RS groups as well, so
// N * RS threads share the work. U weight loads are unrolled, so about U are
// in flight per thread (each batch of U costs one L2 round trip).
template <int NB, int K, int N, int KS, int RS = 1, int U = 8>
__device__ __forceinline__ void rows_gemm(const float* in, int ldi, const float* __restrict__ W,
                                          const float* __restrict__ bias, float* out, int ldo, float* part) {
    static_assert(RS == 1 || KS == 1, "split rows or K, not both");
    constexpr int KC = (K + KS - 1) / KS;
    constexpr int NR = (NB + RS - 1) / RS;
    for (int it = threadIdx.x; it < N * KS * RS; it += blockDim.x) {
        const int n = it % N, ks = (it / N) % KS, rs = it / (N * KS);
        const int k0 = ks * KC, k1 = k0 + KC < K ? k0 + KC : K;
        const int r0 = rs * NR;
        float acc[NR];
#pragma unroll
        for (int i = 0; i < NR; ++i) acc[i] = 0.0f;
#pragma unroll U
        for (int k = k0; k < k1; ++k) {
            const float w = __ldg(W + (size_t)k * N + n);
#pragma unroll
            for (int i = 0; i < NR; ++i)
                if (r0 + i < NB) acc[i] += in[(r0 + i) * ldi + k] * w;
        }
        if (KS == 1) {
#pragma unroll
            for (int i = 0; i < NR; ++i)
                if (r0 + i < NB) out[(r0 + i) * ldo + n] = acc[i] + (bias ? bias[n] : 0.0f);
        } else {
#pragma unroll
            for (int i = 0; i < NB; ++i) part[(ks * NB + i) * N + n] = acc[i];
        }
    }
    if (KS > 1) {
        __syncthreads();
        for (int it = threadIdx.x; it < NB * N; it += blockDim.x) {
            const int i = it / N, n = it % N;
            float v = bias ? bias[n] : 0.0f;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) v += part[(ks * NB + i) * N + n];
            out[i * ldo + n] = v;
        }
    }
}

// Eight consecutive f16 operands of row r, columns [k, k + 8), as floats.
__device__ __forceinline__ void ld_chunk(const uint8_t* tile, uint32_t R, uint32_t r, uint32_t k, float* v) {
    const uint4 q = *reinterpret_cast<const uint4*>(tile + umma::sw128_offset(R, r, k));
    const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[2 * i] = F16::lo(w4[i]);
        v[2 * i + 1] = F16::hi(w4[i]);
    }
}

}  // namespace

struct TrunkSmem {  // the non-operand scratch
    float part_s[128][3];
    float part_q[128][3];
    float pooled[BOARDS][2 * C];
    float gb[BOARDS][C];
    float part[4 * BOARDS * C];  // K-slice partial sums of the pooling GEMM
    // per block and LayerNorm: (gamma, beta) column pairs for ln_gelu2, which
    // reads them as uint2 (8-byte alignment required)
    alignas(16) uint32_t gb2[wc::NET_BLOCKS][2][C];
    uint64_t wbar[2];
    uint64_t mbar;
    uint32_t tmem_slot;
    int abort_flag;
};

// Stem scratch, aliased onto the A operands before the first block.
struct StemSmem {
    float piles[BOARDS][NTYPE * PILE];
    float loose[BOARDS][LOOSE];
    float facts[ROWS][HEX_FACTS];
    int occ[ROWS];
    float proj[BOARDS][NTYPE * C];
    float glob[BOARDS][C];
    float tpool[BOARDS][C];
};

// Readout scratch, aliased onto the A operands after the last block.
struct HeadSmem {
    float x[ROWS][C];
    float input[BOARDS][2 * C + LOOSE];
    float P[BOARDS][D];
    float jp[BOARDS][JW];
    float part[3 * BOARDS * D];  // K-slice partial sums of the readout GEMMs
};

__global__ void __launch_bounds__(384, 1)
    k_trunk_fast(const JobDev* __restrict__ jobs, const uint32_t* __restrict__ row_job,
                 const uint32_t* __restrict__ row_local, uint32_t total_rows, const uint8_t* __restrict__ tiles,
                 const float* __restrict__ W, const float* __restrict__ B, const float* __restrict__ LN,
                 const FastNetDev fn, uint16_t* __restrict__ g_pb, uint16_t* __restrict__ g_jp, int* __restrict__ err) {
    extern __shared__ uint8_t smem_raw[];
    if (umma::misaligned16(tiles) || umma::misaligned16(fn.stem_pb) || umma::misaligned16(fn.stem_w) ||
        umma::misaligned16(fn.trunk_ob)) {  // entry self-check: a launch contract broken, nothing touched
        if (threadIdx.x == 0) atomicExch(err, 34);
        return;
    }
    uint8_t* smem = smem_raw + ((1024u - (umma::smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sW[2] = {smem, smem + BLOCK_BYTES};
    uint8_t* sA1 = smem + 2 * BLOCK_BYTES;
    uint8_t* sA2 = sA1 + A1_BYTES;
    TrunkSmem& S = *reinterpret_cast<TrunkSmem*>(sA2 + A2_BYTES);
    StemSmem& St = *reinterpret_cast<StemSmem*>(sA1);
    HeadSmem& Hd = *reinterpret_cast<HeadSmem*>(sA1);
    static_assert(sizeof(StemSmem) <= A1_BYTES + A2_BYTES, "stem scratch must fit the operand space");
    static_assert(sizeof(HeadSmem) <= A1_BYTES + A2_BYTES, "readout scratch must fit the operand space");

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quad = warp & 3, cg = warp >> 2;
    const int row = quad * 32 + lane;       // hex row of the tile (TMEM lane)
    const int board = row / NH, hex = row % NH;
    const bool real_row = row < ROWS;
    const int col0 = cg * 32;
    const uint32_t ntiles = (total_rows + BOARDS - 1) / BOARDS;
    const NetLayout& L = c_Lt;

    for (int i = tid; i < wc::NET_BLOCKS * 2 * (C / 2); i += blockDim.x) {
        const int blk = i / C, which = (i / (C / 2)) % 2, c = 2 * (i % (C / 2));
        const int ln = NetLayout::ln_block(blk, which);
        umma::pack_gb2(LN + L.norm_g[ln], LN + L.norm_b[ln], c, &S.gb2[blk][which][c]);
    }
    if (tid == 0) {
        umma::mbar_init(&S.wbar[0], 1);
        umma::mbar_init(&S.wbar[1], 1);
        umma::mbar_init(&S.mbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        S.abort_flag = 0;
    }
    if (warp == 0) umma::tmem_alloc(&S.tmem_slot, 256);
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = S.tmem_slot;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    // this thread's row is fixed: its six neighbour rows (-1: none), read
    // once from the constant table (a per-lane gather there serialises)
    int nbr[6];
#pragma unroll
    for (int d = 0; d < 6; ++d) {
        const uint8_t nbh = real_row ? c_nbt[hex][d] : (uint8_t)255;
        nbr[d] = nbh == 255 ? -1 : board * NH + nbh;
    }
    // Barrier bookkeeping, identical in every thread (each decision below is
    // block-uniform): the parity each barrier completes next, and whether an
    // issued copy or product has not yet been seen to complete on it.
    uint32_t wphase[2] = {0, 0}, mphase = 0;
    bool wpend[2] = {false, false}, mpend = false, dead = false;
    const uint64_t wait_ns = fn.wait_ns;
    if (blockIdx.x < ntiles) {
        if (tid == 0) fetch_block(sW[0], tiles, 0, &S.wbar[0]);
        wpend[0] = true;
    }

    for (uint32_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        // ---------------------------------------------------------- stem
        uint32_t gb_[BOARDS];
        int nb = 0;
        for (int i = 0; i < BOARDS; ++i) {
            uint32_t g = tile * BOARDS + i;
            gb_[i] = g;
            if (g < total_rows) nb = i + 1;
        }
        for (int q = tid; q < ROWS; q += blockDim.x) {
            int i = q / NH, h = q % NH;
            float* f = St.facts[q];
            for (int k = 0; k < HEX_FACTS; ++k) f[k] = 0.0f;
            St.occ[q] = -1;
            if (i >= nb) continue;
            const JobDev& J = jobs[row_job[gb_[i]]];
            const uint8_t* rw = J.gpu_rows + (size_t)J.row_gpu[row_local[gb_[i]]] * 201;
            uint8_t owner = rw[h], slot = rw[37 + h], marker = rw[111 + h];
            if (owner != 255) {
                f[owner] = 1.0f;
                f[2] = (float)rw[74 + h] / 5.0f;
                if (slot != 255) St.occ[q] = owner * NSLOT + slot;
            }
            if (marker != 255) f[3 + marker] = 1.0f;
            f[5] = c_islt[h] ? 1.0f : 0.0f;
        }
        for (int q = tid; q < BOARDS * (NTYPE * PILE + LOOSE); q += blockDim.x) {
            int i = q / (NTYPE * PILE + LOOSE), k = q % (NTYPE * PILE + LOOSE);
            if (i >= nb) {
                if (k < NTYPE * PILE) St.piles[i][k] = 0.0f;
                else St.loose[i][k - NTYPE * PILE] = 0.0f;
                continue;
            }
            const JobDev& J = jobs[row_job[gb_[i]]];
            const uint8_t* rw = J.gpu_rows + (size_t)J.row_gpu[row_local[gb_[i]]] * 201;
            if (k < NTYPE * PILE) {
                St.piles[i][k] = (float)rw[148 + k] / 5.0f;
            } else {
                int j = k - NTYPE * PILE;
                float v;
                if (j < 12) {
                    int p = j / 6, f = j % 6;
                    uint8_t mh = rw[188 + p];
                    v = f == 0 ? (float)mh / 6.0f
                      : f == 1 ? (float)(6 - mh) / 6.0f
                      : f == 2 ? (float)rw[190 + p] / 3.0f
                      : f == 3 ? (float)rw[192 + p] / 21.0f
                      : f == 4 ? (float)rw[194 + p] / 21.0f
                               : (rw[196] == p ? 1.0f : 0.0f);
                } else if (j == 12) {
                    v = (float)(uint16_t)(rw[199] | (rw[200] << 8)) / 256.0f;
                } else if (j == 13) {
                    v = rw[197] ? 1.0f : 0.0f;
                } else {
                    v = rw[198] == 0 ? 1.0f : 0.0f;
                }
                St.loose[i][j] = v;
            }
        }
        __syncthreads();
        // proj[i][t] = tokens[i][t] W_tok with tokens = piles W_pile + cards + seat,
        // by linearity piles (W_pile W_tok) + the job's (cards + seat) W_tok
        for (int q = tid; q < BOARDS * NTYPE * C; q += blockDim.x) {
            const int i = q / (NTYPE * C), t = (q / C) % NTYPE, c = q % C;
            float acc = 0.0f;
            if (i < nb) {
                const JobDev& J = jobs[row_job[gb_[i]]];
                acc = J.tokproj[t * C + c];
#pragma unroll
                for (int k = 0; k < PILE; ++k) acc += St.piles[i][t * PILE + k] * fn.pile_tok[k * C + c];
            }
            St.proj[i][t * C + c] = acc;
        }
        rows_gemm<BOARDS, LOOSE, C, 1>(&St.loose[0][0], LOOSE, W + L.glob_stem.w, nullptr, &St.glob[0][0], C, nullptr);
        __syncthreads();
        for (int q = tid; q < BOARDS * C; q += blockDim.x) {
            int i = q / C, c = q % C;
            float acc = 0.0f;
            for (int t = 0; t < NTYPE; ++t) acc += umma::gelu_fast(St.proj[i][t * C + c]) / (float)NTYPE;
            St.tpool[i][c] = acc;
        }
        __syncthreads();
        // x = facts W_hex + (pos[hex] + b_hex) + occupant's token projection + glob + tpool
        float x[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) x[j] = 0.0f;
        if (real_row && board < nb) {
            float f[HEX_FACTS];
#pragma unroll
            for (int k = 0; k < HEX_FACTS; ++k) f[k] = St.facts[row][k];
            const int occ = St.occ[row];
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
                const int c = col0 + 4 * j4;
                float4 v = __ldg(reinterpret_cast<const float4*>(fn.stem_pb + hex * C + c));
#pragma unroll
                for (int k = 0; k < HEX_FACTS; ++k) {
                    const float4 w = __ldg(reinterpret_cast<const float4*>(fn.stem_w + k * C + c));
                    v.x += f[k] * w.x;
                    v.y += f[k] * w.y;
                    v.z += f[k] * w.z;
                    v.w += f[k] * w.w;
                }
                const float* g = &St.glob[board][c];
                const float* tp = &St.tpool[board][c];
                x[4 * j4] = v.x + (occ >= 0 ? St.proj[board][occ * C + c] : 0.0f) + g[0] + tp[0];
                x[4 * j4 + 1] = v.y + (occ >= 0 ? St.proj[board][occ * C + c + 1] : 0.0f) + g[1] + tp[1];
                x[4 * j4 + 2] = v.z + (occ >= 0 ? St.proj[board][occ * C + c + 2] : 0.0f) + g[2] + tp[2];
                x[4 * j4 + 3] = v.w + (occ >= 0 ? St.proj[board][occ * C + c + 3] : 0.0f) + g[3] + tp[3];
            }
        }
        __syncthreads();  // stem scratch is dead from here

        // ------------------------------------------------- residual blocks
#pragma unroll 1
        for (int blk = 0; blk < wc::NET_BLOCKS; ++blk) {
            const int buf = blk & 1;
            // LNGELU(x) -> A1 columns 0..95
            {
                float s = 0.0f;
#pragma unroll
                for (int j = 0; j < 32; ++j) s += x[j];
                S.part_s[row][cg] = s;
                __syncthreads();
                const float mean = (S.part_s[row][0] + S.part_s[row][1] + S.part_s[row][2]) * (1.0f / C);
                float q = 0.0f;
#pragma unroll
                for (int j = 0; j < 32; ++j) q += (x[j] - mean) * (x[j] - mean);
                S.part_q[row][cg] = q;
                __syncthreads();
                const float inv = rsqrtf((S.part_q[row][0] + S.part_q[row][1] + S.part_q[row][2]) * (1.0f / C) + 1e-5f);
                const float nm = -mean * inv;
                const float* gam = LN + L.norm_g[NetLayout::ln_block(blk, 0)];
                const float* bet = LN + L.norm_b[NetLayout::ln_block(blk, 0)];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t w4[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int k = 8 * c + 2 * j;
                        w4[j] = real_row ? umma::ln_gelu2<true>(x[k] * inv + nm, x[k + 1] * inv + nm, col0 + k, S.gb2[blk][0])
                                         : 0u;
                    }
                    *reinterpret_cast<uint4*>(sA1 + umma::sw128_offset(128, row, col0 + 8 * c)) =
                        make_uint4(w4[0], w4[1], w4[2], w4[3]);
                }
            }
            __syncthreads();
            // neighbour sums -> columns 96..191; board pooling (mean | max) of a
            {
                {
                    // packed f16 adds (the sum is stored as an f16 operand anyway)
                    __half2 acc[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) acc[j] = __float2half2_rn(0.0f);
                    {
#pragma unroll
                        for (int d = 0; d < 6; ++d) {
                            const int nr = nbr[d];
                            if (nr < 0) continue;
#pragma unroll
                            for (int c = 0; c < 4; ++c) {
                                const uint4 q = *reinterpret_cast<const uint4*>(sA1 + umma::sw128_offset(128, nr, col0 + 8 * c));
                                const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                                for (int e = 0; e < 4; ++e)
                                    acc[4 * c + e] = __hadd2(acc[4 * c + e], *reinterpret_cast<const __half2*>(&w4[e]));
                            }
                        }
                    }
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        uint4 o;
                        o.x = *reinterpret_cast<const uint32_t*>(&acc[4 * c]);
                        o.y = *reinterpret_cast<const uint32_t*>(&acc[4 * c + 1]);
                        o.z = *reinterpret_cast<const uint32_t*>(&acc[4 * c + 2]);
                        o.w = *reinterpret_cast<const uint32_t*>(&acc[4 * c + 3]);
                        *reinterpret_cast<uint4*>(sA1 + umma::sw128_offset(128, row, C + col0 + 8 * c)) = o;
                    }
                }
            }
            // mean | max over each board's hexes: (board, 8-column chunk, hex group)
            // partials in the free A2 space, then one thread per (board, column)
            {
                constexpr int HG = 10;  // hex groups: hexes h = g, g + HG, ...
                float* psum = reinterpret_cast<float*>(sA2);                 // [BOARDS][C][HG]
                float* pmax = psum + BOARDS * C * HG;
                if (tid < BOARDS * (C / 8) * HG) {
                    const int gidx = tid % HG, c0 = ((tid / HG) % (C / 8)) * 8, i = tid / (HG * (C / 8));
                    float sum[8], mx[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) { sum[j] = 0.0f; mx[j] = -INFINITY; }
                    for (int h = gidx; h < NH; h += HG) {
                        float v[8];
                        ld_chunk(sA1, 128, i * NH + h, c0, v);
#pragma unroll
                        for (int j = 0; j < 8; ++j) { sum[j] += v[j]; mx[j] = fmaxf(mx[j], v[j]); }
                    }
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        psum[(i * C + c0 + j) * HG + gidx] = sum[j];
                        pmax[(i * C + c0 + j) * HG + gidx] = mx[j];
                    }
                }
                __syncthreads();
                if (tid < BOARDS * C) {
                    const int i = tid / C, c = tid % C;
                    float sm = 0.0f, m = -INFINITY;
#pragma unroll
                    for (int gg = 0; gg < HG; ++gg) {
                        sm += psum[(i * C + c) * HG + gg];
                        m = fmaxf(m, pmax[(i * C + c) * HG + gg]);
                    }
                    S.pooled[i][c] = sm * (1.0f / NH);
                    S.pooled[i][C + c] = m;
                }
            }
            __syncthreads();
            rows_gemm<BOARDS, 2 * C, C, 4, 1, 16>(&S.pooled[0][0], 2 * C, W + L.pool[blk].w, fn.trunk_pb + blk * C,
                                                  &S.gb[0][0], C, S.part);
            // mix product (weights of this block must have landed)
            {
                const bool ok = umma::mbar_wait(&S.wbar[buf], wphase[buf], wait_ns);
                umma::fence_async_smem();
                umma::fence_before_sync();
                dead = __syncthreads_or(!ok) != 0;
                umma::fence_after_sync();
                if (dead) break;  // the copy stays pending: drained at the exit
                wphase[buf] ^= 1u;
                wpend[buf] = false;
            }
            if (tid == 0) {
                const uint32_t aa = umma::smem_u32(sA1), wb = umma::smem_u32(sW[buf]);
                const uint32_t idesc = umma::idesc16(128, 96, F16::fmt);
#pragma unroll
                for (int k0 = 0; k0 < 2 * C; k0 += 16)
                    umma::mma16(tmem, umma::desc_at(aa, 128, k0), umma::desc_at(wb, 96, k0), idesc, k0 > 0);
                umma::commit(&S.mbar);
            }
            mpend = true;
            {
                const bool ok = umma::mbar_wait(&S.mbar, mphase, wait_ns);
                umma::fence_before_sync();
                dead = __syncthreads_or(!ok) != 0;
                umma::fence_after_sync();
                if (dead) break;
                mphase ^= 1u;
                mpend = false;
            }
            // y = mix + (b_mix + pooled W_pool + b_pool); LNGELU -> A2
            float y[32];
            {
                float v[32];
                umma::tmem_ld32(tmem + lane_off + col0, v);
                const float* gbr = &S.gb[real_row ? board : 0][col0];
#pragma unroll
                for (int j = 0; j < 32; ++j) y[j] = v[j] + gbr[j];
                float s = 0.0f;
#pragma unroll
                for (int j = 0; j < 32; ++j) s += y[j];
                S.part_s[row][cg] = s;
                __syncthreads();
                const float mean = (S.part_s[row][0] + S.part_s[row][1] + S.part_s[row][2]) * (1.0f / C);
                float q = 0.0f;
#pragma unroll
                for (int j = 0; j < 32; ++j) q += (y[j] - mean) * (y[j] - mean);
                S.part_q[row][cg] = q;
                __syncthreads();
                const float inv = rsqrtf((S.part_q[row][0] + S.part_q[row][1] + S.part_q[row][2]) * (1.0f / C) + 1e-5f);
                const float nm = -mean * inv;
                const float* gam = LN + L.norm_g[NetLayout::ln_block(blk, 1)];
                const float* bet = LN + L.norm_b[NetLayout::ln_block(blk, 1)];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t w4[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int k = 8 * c + 2 * j;
                        w4[j] = real_row ? umma::ln_gelu2<true>(y[k] * inv + nm, y[k + 1] * inv + nm, col0 + k, S.gb2[blk][1])
                                         : 0u;
                    }
                    *reinterpret_cast<uint4*>(sA2 + umma::sw128_offset(128, row, col0 + 8 * c)) =
                        make_uint4(w4[0], w4[1], w4[2], w4[3]);
                }
            }
            umma::fence_async_smem();
            umma::fence_before_sync();
            __syncthreads();
            umma::fence_after_sync();
            if (tid == 0) {
                const uint32_t aa = umma::smem_u32(sA2), wb = umma::smem_u32(sW[buf] + MIX_BYTES);
                const uint32_t idesc = umma::idesc16(128, 96, F16::fmt);
#pragma unroll
                for (int k0 = 0; k0 < C; k0 += 16)
                    umma::mma16(tmem + 128, umma::desc_at(aa, 128, k0), umma::desc_at(wb, 96, k0), idesc, k0 > 0);
                umma::commit(&S.mbar);
            }
            mpend = true;
            {
                const bool ok = umma::mbar_wait(&S.mbar, mphase, wait_ns);
                umma::fence_before_sync();
                dead = __syncthreads_or(!ok) != 0;
                umma::fence_after_sync();
                if (dead) break;
                mphase ^= 1u;
                mpend = false;
            }
            // the other buffer is free: fetch the next block (or the next tile's first)
            if (blk + 1 < wc::NET_BLOCKS || tile + gridDim.x < ntiles) {
                if (tid == 0) fetch_block(sW[buf ^ 1], tiles, (blk + 1) % wc::NET_BLOCKS, &S.wbar[buf ^ 1]);
                wpend[buf ^ 1] = true;
            }
            {
                float v[32];
                umma::tmem_ld32(tmem + lane_off + 128 + col0, v);
                const float4* ob = reinterpret_cast<const float4*>(fn.trunk_ob + blk * C + col0);
#pragma unroll
                for (int j4 = 0; j4 < 8; ++j4) {
                    const float4 b4 = __ldg(ob + j4);
                    x[4 * j4] += v[4 * j4] + b4.x;
                    x[4 * j4 + 1] += v[4 * j4 + 1] + b4.y;
                    x[4 * j4 + 2] += v[4 * j4 + 2] + b4.z;
                    x[4 * j4 + 3] += v[4 * j4 + 3] + b4.w;
                }
            }
        }
        if (dead) break;
        // -------------------------------------- final norm and the readout
        {
            float s = 0.0f;
#pragma unroll
            for (int j = 0; j < 32; ++j) s += x[j];
            S.part_s[row][cg] = s;
            __syncthreads();
            const float mean = (S.part_s[row][0] + S.part_s[row][1] + S.part_s[row][2]) * (1.0f / C);
            float q = 0.0f;
#pragma unroll
            for (int j = 0; j < 32; ++j) q += (x[j] - mean) * (x[j] - mean);
            S.part_q[row][cg] = q;
            __syncthreads();
            const float inv = rsqrtf((S.part_q[row][0] + S.part_q[row][1] + S.part_q[row][2]) * (1.0f / C) + 1e-5f);
            const float* gam = LN + L.norm_g[NetLayout::LN_TRUNK];
            const float* bet = LN + L.norm_b[NetLayout::LN_TRUNK];
            if (real_row) {
#pragma unroll
                for (int j = 0; j < 32; ++j) Hd.x[row][col0 + j] = umma::gelu_fast((x[j] - mean) * inv * gam[col0 + j] + bet[col0 + j]);
            }
        }
        __syncthreads();
        for (int q = tid; q < BOARDS * (2 * C + LOOSE); q += blockDim.x) {
            int i = q / (2 * C + LOOSE), k = q % (2 * C + LOOSE);
            float v = 0.0f;
            if (k < C) {
                for (int h = 0; h < NH; ++h) v += Hd.x[i * NH + h][k] / (float)NH;
            } else if (k < 2 * C) {
                v = -INFINITY;
                for (int h = 0; h < NH; ++h) v = fmaxf(v, Hd.x[i * NH + h][k - C]);
            } else {
                v = 0.0f;
            }
            Hd.input[i][k] = v;
        }
        __syncthreads();
        // loose scalars are re-read from the rows (the stem scratch is gone)
        for (int q = tid; q < BOARDS * LOOSE; q += blockDim.x) {
            int i = q / LOOSE, j = q % LOOSE;
            float v = 0.0f;
            if (i < nb) {
                const JobDev& J = jobs[row_job[gb_[i]]];
                const uint8_t* rw = J.gpu_rows + (size_t)J.row_gpu[row_local[gb_[i]]] * 201;
                if (j < 12) {
                    int p = j / 6, f = j % 6;
                    uint8_t mh = rw[188 + p];
                    v = f == 0 ? (float)mh / 6.0f
                      : f == 1 ? (float)(6 - mh) / 6.0f
                      : f == 2 ? (float)rw[190 + p] / 3.0f
                      : f == 3 ? (float)rw[192 + p] / 21.0f
                      : f == 4 ? (float)rw[194 + p] / 21.0f
                               : (rw[196] == p ? 1.0f : 0.0f);
                } else if (j == 12) {
                    v = (float)(uint16_t)(rw[199] | (rw[200] << 8)) / 256.0f;
                } else if (j == 13) {
                    v = rw[197] ? 1.0f : 0.0f;
                } else {
                    v = rw[198] == 0 ? 1.0f : 0.0f;
                }
            }
            Hd.input[i][2 * C + j] = v;
        }
        __syncthreads();
        rows_gemm<BOARDS, 2 * C + LOOSE, D, 3, 1, 23>(&Hd.input[0][0], 2 * C + LOOSE, W + L.board_out.w,
                                                      B + L.board_out.b, &Hd.P[0][0], D, Hd.part);
        __syncthreads();
        // P + bout (the join output bias, which the readout adds to every row)
        // and jp are stored as 16-bit operands minus their row mean: every
        // consumer of them (the join residual stream, the readout y) goes
        // through a LayerNorm, which ignores a per-row constant, so the shift
        // is exact and only shrinks the rounding.
        const float* bout = B + L.join_out.b;
        if (tid < BOARDS * 32) {
            const int i = tid / 32, l = tid % 32;
            float s = 0.0f;
            for (int c = l; c < D; c += 32) s += Hd.P[i][c] + bout[c];
#pragma unroll
            for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (l == 0) S.gb[i][0] = s / (float)D;
        }
        __syncthreads();
        // P goes to the readout's per-tile images: the row's 128-row tile of
        // its job (64 KB), row r at r * 512 bytes, its 16-byte chunk k at k ^ (r & 7)
        for (int q = tid; q < BOARDS * D; q += blockDim.x) {
            int i = q / D, c = q % D;
            if (i < nb) {
                const uint32_t lr = row_local[gb_[i]];
                const size_t slot = jobs[row_job[gb_[i]]].tile_base + lr / 128;
                const uint32_t rt = lr % 128;
                g_pb[slot * 32768 + rt * 256 + ((uint32_t)(c >> 3) ^ (rt & 7)) * 8 + (c & 7)] =
                    F16::one(Hd.P[i][c] + bout[c] - S.gb[i][0]);
            }
        }
        rows_gemm<BOARDS, D, JW, 3, 1, 22>(&Hd.P[0][0], D, W + L.join_p.w, nullptr, &Hd.jp[0][0], JW, Hd.part);
        __syncthreads();
        if (tid < BOARDS * 32) {
            const int i = tid / 32, l = tid % 32;
            float s = 0.0f;
            for (int c = l; c < JW; c += 32) s += Hd.jp[i][c];
#pragma unroll
            for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (l == 0) S.gb[i][1] = s / (float)JW;
        }
        __syncthreads();
        for (int q = tid; q < BOARDS * JW; q += blockDim.x) {
            int i = q / JW, c = q % JW;
            if (i < nb)
                g_jp[((size_t)jobs[row_job[gb_[i]]].row_base + row_local[gb_[i]]) * JW + c] =
                    F16::one(Hd.jp[i][c] - S.gb[i][1]);
        }
        __syncthreads();
    }
    // Every thread leaves the loops at the same point (`dead` comes from
    // __syncthreads_or). Nothing was issued after a failed wait, so what may
    // still be in flight is exactly what is marked pending: it completes on
    // its own and must land before the shared memory and the tensor memory
    // are released. A drain that does not finish leaves the tensor memory
    // allocated (a product may still write it) and reports code 13: the
    // device context can no longer be trusted.
    if (tid == 0) {
        bool drained = true;
        if (mpend) drained = umma::mbar_wait(&S.mbar, mphase, umma::DRAIN_NS) && drained;
        for (int b = 0; b < 2; ++b)
            if (wpend[b]) drained = umma::mbar_wait(&S.wbar[b], wphase[b], umma::DRAIN_NS) && drained;
        S.abort_flag = drained ? 0 : 1;
        if (dead || !drained) atomicExch(err, drained ? 3 : 13);
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (warp == 0 && !S.abort_flag) umma::tmem_dealloc(tmem, 256);
}

void trunk_set_constants(const NetLayout& L, const uint8_t* neighbors, const uint8_t* is_location) {
    cudaMemcpyToSymbol(c_Lt, &L, sizeof(NetLayout));
    cudaMemcpyToSymbol(c_nbt, neighbors, 37 * 6);
    cudaMemcpyToSymbol(c_islt, is_location, 37);
}

size_t trunk_tiles_bytes() { return (size_t)wc::NET_BLOCKS * BLOCK_BYTES; }

// The per-job part of the stem's token projection: (cards + seat) W_tok per
// card type (the trunk adds the pile counts times W_pile W_tok).
__global__ void k_tokproj(const JobDev* __restrict__ jobs, const float* __restrict__ W) {
    const JobDev& J = jobs[blockIdx.x];
    const NetLayout& L = c_Lt;
    for (int i = threadIdx.x; i < NTYPE * C; i += blockDim.x) {
        const int t = i / C, c = i % C;
        float acc = 0.0f;
        for (int j = 0; j < TYPE; ++j)
            acc += (J.cards[t * TYPE + j] + W[L.seat + (t / NSLOT) * TYPE + j]) * W[L.tok_stem.w + j * C + c];
        J.tokproj[i] = acc;
    }
}

void launch_tokproj(const JobDev* jobs, uint32_t njobs, const float* W, cudaStream_t s) {
    if (njobs) k_tokproj<<<njobs, 256, 0, s>>>(jobs, W);
}

// P and jp of every duplicate row from its representative (the first row of
// its job with the same public row bytes, which the trunk computed): one
// warp per row, 16-byte chunks; a P row's chunk k sits at k ^ (row & 7) of
// its 512-byte row in the tile image, so the chunk is read at the
// representative's position and written at the duplicate's.
__global__ void __launch_bounds__(256) k_board_dup(const JobDev* __restrict__ jobs, const uint32_t* __restrict__ dup,
                                                   uint32_t n, uint16_t* __restrict__ g_pb, uint16_t* __restrict__ g_jp) {
    const uint32_t w = blockIdx.x * 8 + threadIdx.x / 32, lane = threadIdx.x % 32;
    if (w >= n) return;
    const JobDev& J = jobs[dup[3 * w]];
    const uint32_t d = dup[3 * w + 1], r = dup[3 * w + 2];
    const size_t td = (size_t)J.tile_base + d / 128, tr = (size_t)J.tile_base + r / 128;
    const uint32_t rd = d % 128, rr = r % 128;
    const uint4* src = reinterpret_cast<const uint4*>(g_pb + tr * 32768 + rr * 256);
    uint4* dst = reinterpret_cast<uint4*>(g_pb + td * 32768 + rd * 256);
    dst[lane ^ (rd & 7)] = src[lane ^ (rr & 7)];
    if (lane < JW / 8)
        reinterpret_cast<uint4*>(g_jp + ((size_t)J.row_base + d) * JW)[lane] =
            reinterpret_cast<const uint4*>(g_jp + ((size_t)J.row_base + r) * JW)[lane];
}

void launch_board_dup(const JobDev* jobs, const uint32_t* dup, uint32_t n, uint16_t* g_pb, uint16_t* g_jp,
                      cudaStream_t s) {
    if (n) k_board_dup<<<(n + 7) / 8, 256, 0, s>>>(jobs, dup, n, g_pb, g_jp);
}

void launch_trunk_fast(const JobDev* jobs, const uint32_t* row_job, const uint32_t* row_local, uint32_t total_rows,
                       const uint8_t* tiles, const float* W, const float* B, const float* LN, const FastNetDev& fn,
                       uint16_t* g_pb, uint16_t* g_jp, int* err, cudaStream_t s) {
    if (!total_rows) return;
    const size_t smem = 2 * BLOCK_BYTES + A1_BYTES + A2_BYTES + sizeof(TrunkSmem) + 1024;
    auto kern = k_trunk_fast;
    if (!raise_smem_limit((const void*)kern, smem)) return;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    uint32_t ntiles = (total_rows + BOARDS - 1) / BOARDS;
    uint32_t grid = std::min<uint32_t>(ntiles, (uint32_t)sms);
    kern<<<grid, 384, smem, s>>>(jobs, row_job, row_local, total_rows, tiles, W, B, LN, fn, g_pb, g_jp, err);
}

}  // namespace wcdev
