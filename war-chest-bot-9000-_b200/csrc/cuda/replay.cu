// The training batch's device expansion: compact replay rows in, the value
// network's public input for both canonical seat views out
// (train/gpu_batch.py:22-117 _expand_rows and make_batch, train/train.py:
// 70-79 public_sizes and 249-270 make_batch, engine/src/rebel.rs:1144-1234
// write_public_features_raw and 1353-1393 expand_row, train/mirror.py:60-85
// mirror_rows).
//
// View 2r is replay row r; view 2r + 1 is its mirror (the board rotated by
// 180 degrees and the seats exchanged), applied while the row is read rather
// than materialised. The per-seat hand / face-down / bag sizes come from the
// first config of each (row, seat) span of the config arrays, exchanged for
// the mirrored view. Every feature is one IEEE division of a small integer
// (or a table entry), so the floats equal the CPU encoder's bit for bit.
//
// Byte work bound by HBM writes (PUBFEAT floats per view against 215 bytes
// read): one warp per view, the row staged in shared memory, the features
// written lane-strided (coalesced), each section's features computed with
// selects and table reads (no divergent branches, no divisions).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <set>

#include "../host/pbs.h"
#include "kernels.h"

namespace wcdev {

namespace {

using namespace wc;

__constant__ float c_card_feat[N_UNITS * CARD_FEATS];
__constant__ uint8_t c_is_loc[N_HEXES];
__constant__ uint8_t c_hex_mirror[N_HEXES];
// k / d for every byte k and the divisors the encoding uses, each the IEEE
// quotient (computed on the host): a table read equals the division the CPU
// encoder does, without the division's instruction sequence per feature
constexpr int Q5 = 0, Q3 = 1, Q21 = 2, Q6 = 3;
__constant__ float c_quot[4][256];

constexpr int VIEWS_PER_CTA = 8;
constexpr int ROW_STRIDE = (ROW_BYTES + 15) / 16 * 16;
static_assert(HEX_CH == 16 && PILE_COUNTS == 4, "the index arithmetic below");

__device__ __forceinline__ uint32_t flip_seat(uint32_t v) { return v == 0 ? 1u : (v == 1 ? 0u : v); }

// np.searchsorted(seg, key, 'left') by the whole warp: each round probes 32
// points that split the remaining range into 33 parts and keeps the part the
// ballot names (seg is sorted, so the probes below `key` are a prefix), about
// four dependent loads for a million configs; the last <= 32 candidates are
// counted directly.
__device__ __forceinline__ uint64_t span_start(const int64_t* __restrict__ seg, uint64_t m, int64_t key,
                                              uint32_t lane) {
    uint64_t lo = 0, hi = m;  // the answer lies in [lo, hi]
    while (hi - lo > 32) {
        const uint64_t len = hi - lo;
        const bool less = seg[lo + len * (lane + 1) / 33] < key;
        const uint32_t cnt = __popc(__ballot_sync(0xffffffffu, less));
        const uint64_t nlo = cnt ? lo + len * cnt / 33 + 1 : lo;
        const uint64_t nhi = cnt < 32 ? lo + len * (cnt + 1) / 33 : hi;
        lo = nlo;
        hi = nhi;
    }
    const bool less = lo + lane < hi && seg[lo + lane] < key;
    return lo + __popc(__ballot_sync(0xffffffffu, less));
}

// A grid of persistent CTAs: the tables are staged once per CTA, and each
// warp expands views v, v + 8 G, ... (G CTAs).
__global__ void __launch_bounds__(32 * VIEWS_PER_CTA)
    k_replay_expand(const uint8_t* __restrict__ rows, uint32_t nviews, const uint8_t* __restrict__ cc,
                    const int64_t* __restrict__ seg, uint64_t m, float* __restrict__ x) {
    __shared__ float s_quot[4][256];
    __shared__ float s_card[N_UNITS * CARD_FEATS];
    __shared__ uint8_t s_loc[N_HEXES], s_mir[N_HEXES];
    __shared__ uint8_t s_row[VIEWS_PER_CTA][ROW_STRIDE];
    __shared__ uint32_t s_size[VIEWS_PER_CTA][6];  // hand[2], fd[2], bag[2] of the view's seats
    __shared__ float s_hex[VIEWS_PER_CTA][HEX_BLOCK];  // a view's hex block as [channel][hex]
    const uint32_t tid = threadIdx.x, w = tid / 32, lane = tid % 32;
    for (uint32_t i = tid; i < 4 * 256; i += blockDim.x) s_quot[i / 256][i % 256] = c_quot[i / 256][i % 256];
    for (uint32_t i = tid; i < N_UNITS * CARD_FEATS; i += blockDim.x) s_card[i] = c_card_feat[i];
    if (tid < N_HEXES) {
        s_loc[tid] = c_is_loc[tid];
        s_mir[tid] = c_hex_mirror[tid];
    }
    __syncthreads();
    for (uint32_t v = blockIdx.x * VIEWS_PER_CTA + w; v < nviews; v += gridDim.x * VIEWS_PER_CTA) {
        __syncwarp();  // the previous view's reads of s_row, s_size and s_hex are done
        const uint32_t r = v >> 1;
        const bool mir = v & 1u;
        const uint8_t* row = rows + (size_t)r * ROW_BYTES;
        for (uint32_t k = lane; k < ROW_BYTES; k += 32) s_row[w][k] = row[k];
        {
            // public_sizes: each seat's first config (the mirrored view reads
            // the other seat's span); lane 2 z + q sums zone z of seat q
            uint64_t st[2];
#pragma unroll
            for (int q = 0; q < 2; ++q) st[q] = span_start(seg, m, 2 * (int64_t)r + (mir ? 1 - q : q), lane);
            if (lane < 6) {
                const uint32_t q = lane & 1u, z = lane >> 1;
                const uint64_t at = q ? st[1] : st[0];
                uint32_t sum = 0;
                if (at < m)
                    for (int k = 0; k < NSLOT; ++k) sum += cc[at * CCOUNTS + z * NSLOT + k];
                s_size[w][2 * z + q] = sum & 0xffu;  // the sums are cast to u8 (.astype(np.uint8))
            }
        }
        __syncwarp();
        const uint8_t* R = s_row[w];
        float* out = x + (size_t)v * PUBFEAT;
        // per hex (one lane each, in two rounds): owner one-hot, height / 5,
        // marker one-hot, location, the owner's slot one-hot, decoded once
        // into the warp's staging as [channel][hex]; each seat's markers on
        // the board counted by ballot
        float* sv = s_hex[w];
        uint32_t on_board[2] = {0, 0};
#pragma unroll
        for (int base = 0; base < N_HEXES; base += 32) {
            const int h = base + (int)lane;
            const bool live = h < N_HEXES;
            const int hh = live ? h : 0;
            const int src = mir ? s_mir[hh] : hh;
            uint32_t owner = R[ROW_HEX_OWNER + src], marker = R[ROW_HEX_MARKER + src];
            if (mir) {
                owner = flip_seat(owner);
                marker = flip_seat(marker);
            }
            const uint32_t slot = R[ROW_HEX_SLOT + src];
            on_board[0] += __popc(__ballot_sync(0xffffffffu, live && marker == 0));
            on_board[1] += __popc(__ballot_sync(0xffffffffu, live && marker == 1));
            if (live) {
                const uint32_t hot = owner < 2 && slot < NSLOT ? owner * NSLOT + slot : 0xffu;
                sv[0 * N_HEXES + h] = owner == 0 ? 1.0f : 0.0f;
                sv[1 * N_HEXES + h] = owner == 1 ? 1.0f : 0.0f;
                sv[2 * N_HEXES + h] = owner != NONE ? s_quot[Q5][R[ROW_HEX_HEIGHT + src]] : 0.0f;
                sv[3 * N_HEXES + h] = marker == 0 ? 1.0f : 0.0f;
                sv[4 * N_HEXES + h] = marker == 1 ? 1.0f : 0.0f;
                sv[5 * N_HEXES + h] = s_loc[h] ? 1.0f : 0.0f;
#pragma unroll
                for (int k = 0; k < NTYPE; ++k) sv[(HEX_FACTS + k) * N_HEXES + h] = hot == (uint32_t)k ? 1.0f : 0.0f;
            }
        }
        __syncwarp();
        for (int j = lane; j < HEX_BLOCK; j += 32) out[j] = sv[(j & 15) * N_HEXES + (j >> 4)];
        // the piles of each coin type / 5 (the mirror exchanges the seats' halves)
        for (int q = lane; q < NTYPE * PILE_COUNTS; q += 32) {
            const int t = q >> 2, st = mir ? (t + NSLOT) % NTYPE : t;
            out[OFF_PILES + q] = s_quot[Q5][R[ROW_PILES + st * PILE_COUNTS + (q & 3)]];
        }
        // the printed card facts of each coin type's unit
        for (int q = lane; q < NTYPE * CARD_FEATS; q += 32) {
            const int t = q / CARD_FEATS, f = q - t * CARD_FEATS, st = mir ? (t + NSLOT) % NTYPE : t;
            const uint32_t id = R[ROW_IDS + st];
            out[OFF_CARDS + q] = id < (uint32_t)N_UNITS ? s_card[id * CARD_FEATS + f] : 0.0f;
        }
        // per seat: markers in hand and on the board / 6, hand / 3, face-down and
        // bag / 21, initiative; then plies remaining / 256, initiative moved, to act
        if (lane < LOOSE) {
            const uint32_t seat = lane < 2 * PLAYER_SCALARS ? lane / PLAYER_SCALARS : 0;
            const uint32_t seat_board = seat ? on_board[1] : on_board[0];
            uint32_t init = mir ? flip_seat(R[ROW_INITIATIVE]) : R[ROW_INITIATIVE];
            if (init > 1) init = 0;  // expand_row's guard (rebel.rs:1377)
            const uint32_t to_act = mir ? flip_seat(R[ROW_TO_ACT]) : R[ROW_TO_ACT];
            const uint32_t plies = R[ROW_PLIES] | ((uint32_t)R[ROW_PLIES + 1] << 8);
            const uint32_t in_hand = ((uint32_t)MARKERS_TOTAL - seat_board) & 0xffu;  // u8 arithmetic, as the encoder's
            float val;
            if (lane < 2 * PLAYER_SCALARS) {
                const uint32_t f = lane % PLAYER_SCALARS;
                val = f == 0   ? s_quot[Q6][in_hand]
                      : f == 1 ? s_quot[Q6][((uint32_t)MARKERS_TOTAL - in_hand) & 0xffu]
                      : f == 2 ? s_quot[Q3][s_size[w][seat]]
                      : f == 3 ? s_quot[Q21][s_size[w][2 + seat]]
                      : f == 4 ? s_quot[Q21][s_size[w][4 + seat]]
                               : (init == seat ? 1.0f : 0.0f);
            } else {
                const uint32_t g = lane - 2 * PLAYER_SCALARS;
                // MAX_MAIN_PLAYS is 2^8: the quotient is exact, a product by 2^-8
                val = g == 0 ? (float)plies * (1.0f / (float)MAX_MAIN_PLAYS)
                      : g == 1 ? (R[ROW_INIT_MOVED] != 0 ? 1.0f : 0.0f)
                               : (to_act == 0 ? 1.0f : 0.0f);
            }
            out[OFF_LOOSE + lane] = val;
        }
    }
}

// phi = config counts / CNORM (train/train.py:267)
__global__ void k_replay_phi(const uint8_t* __restrict__ cc, uint64_t total, float* __restrict__ phi) {
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x)
        phi[i] = (float)cc[i] / CNORM;
}

std::mutex g_tables_mu;
std::set<int> g_tables_ready;

}  // namespace

bool replay_tables_ready() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    std::lock_guard<std::mutex> lk(g_tables_mu);
    if (g_tables_ready.count(dev)) return true;
    float card[N_UNITS * CARD_FEATS];
    for (int u = 0; u < N_UNITS; ++u) write_card_features((uint8_t)u, card + u * CARD_FEATS);
    float quot[4][256];
    const float div[4] = {5.0f, 3.0f, MAX_COINS, 6.0f};
    for (int d = 0; d < 4; ++d)
        for (int k = 0; k < 256; ++k) quot[d][k] = (float)k / div[d];
    uint8_t loc[N_HEXES], mirror[N_HEXES];
    for (int h = 0; h < N_HEXES; ++h) {
        loc[h] = board().is_location[h] ? 1 : 0;
        mirror[h] = (uint8_t)mirror_hex(h);
    }
    if (cudaMemcpyToSymbol(c_card_feat, card, sizeof card) != cudaSuccess ||
        cudaMemcpyToSymbol(c_is_loc, loc, sizeof loc) != cudaSuccess ||
        cudaMemcpyToSymbol(c_hex_mirror, mirror, sizeof mirror) != cudaSuccess ||
        cudaMemcpyToSymbol(c_quot, quot, sizeof quot) != cudaSuccess)
        return false;
    g_tables_ready.insert(dev);
    return true;
}

void launch_replay_expand(const uint8_t* rows, uint32_t nrows, const uint8_t* cc, const int64_t* seg, uint64_t m,
                          float* x, float* phi, cudaStream_t s) {
    const uint32_t nviews = 2 * nrows;
    if (nviews) {
        int dev = 0, sms = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const uint32_t want = (nviews + VIEWS_PER_CTA - 1) / VIEWS_PER_CTA;
        k_replay_expand<<<std::min<uint32_t>(want, (uint32_t)sms * 8), 32 * VIEWS_PER_CTA, 0, s>>>(rows, nviews, cc, seg, m, x);
    }
    const uint64_t total = m * (uint64_t)CCOUNTS;
    if (total) k_replay_phi<<<(unsigned)std::min<uint64_t>((total + 255) / 256, 148ull * 16), 256, 0, s>>>(cc, total, phi);
}

}  // namespace wcdev
