// The v5 value network in fp32 on CUDA cores, in the reference CPU's exact
// operation order (engine/src/net.rs:544-853): every matrix product is a
// sequential-k accumulation starting from 0 (or from the residual the
// reference adds into), the bias is added after the full sum, LayerNorm takes
// sequential sums with eps 1e-5, GELU is the tanh form with the shared
// deterministic tanh (host/detmath.h). Compiled with
// -fmad=false. This is the "precise" network path used for parity against the
// CPU oracle; the tensor-core path is net_fast.cu.
#include <cuda_runtime.h>

#include <cstdint>

#include "../host/detmath.h"
#include "device.h"
#include "kernels.h"

namespace wcdev {

using wc::NetLayout;

__constant__ NetLayout c_L;
__constant__ uint8_t c_neighbors[37][6];
__constant__ uint8_t c_is_location[37];

constexpr int N_HEXES = 37, NSLOT = 5, NTYPE = 10, CARD_FEATS = 25, HEX_FACTS = 6, LOOSE = 15, PILE = 4;
constexpr int TYPE = wc::NET_TYPE, C = wc::NET_C, D = wc::NET_D, POOL = wc::NET_POOL, CFGH = wc::NET_CFGH,
              JW = wc::NET_JW;
constexpr int ROW_HEX_OWNER = 0, ROW_HEX_SLOT = 37, ROW_HEX_HEIGHT = 74, ROW_HEX_MARKER = 111, ROW_PILES = 148,
              ROW_MARKERS = 188, ROW_HAND = 190, ROW_FD = 192, ROW_BAG = 194, ROW_INITIATIVE = 196,
              ROW_INIT_MOVED = 197, ROW_TO_ACT = 198, ROW_PLIES = 199, ROW_BYTES = 201;

__device__ __forceinline__ float gelu(float x) { return wc::det_gelu(x); }

// out[j] for j in [0, o): sum_k in[k] * W[k * o + j], sequential in k.
__device__ __forceinline__ float dot_col(const float* in, const float* W, int i, int o, int j, float acc) {
    for (int k = 0; k < i; ++k) acc += in[k] * W[(size_t)k * o + j];
    return acc;
}

// LayerNorm (+GELU) of `rows` rows of `width`, each row's statistics taken
// sequentially by one thread (net.rs:380-405).
__device__ void ln_rows(float* x, int rows, int width, int norm, bool act, float* stat, const float* LN) {
    __syncthreads();
    for (int r = threadIdx.x; r < rows; r += blockDim.x) {
        const float* row = x + r * width;
        float s = 0.0f;
        for (int j = 0; j < width; ++j) s += row[j];
        float mean = s / (float)width;
        float v = 0.0f;
        for (int j = 0; j < width; ++j) v += (row[j] - mean) * (row[j] - mean);
        float var = v / (float)width;
        stat[2 * r] = mean;
        stat[2 * r + 1] = 1.0f / sqrtf(var + 1e-5f);
    }
    __syncthreads();
    const float* g = LN + c_L.norm_g[norm];
    const float* b = LN + c_L.norm_b[norm];
    for (int q = threadIdx.x; q < rows * width; q += blockDim.x) {
        int r = q / width, j = q % width;
        float y = (x[q] - stat[2 * r]) * stat[2 * r + 1] * g[j] + b[j];
        x[q] = act ? gelu(y) : y;
    }
    __syncthreads();
}

// Card tokens for both seat views (net.rs:544-555) and cfg_m over them (net.rs:777-779).
__global__ void k_cards(const JobDev* __restrict__ jobs, const float* __restrict__ W, const float* __restrict__ B) {
    const JobDev& J = jobs[blockIdx.x];
    __shared__ float hid[2 * NTYPE][TYPE];
    __shared__ float tok[2 * NTYPE][TYPE];
    const wc::NetSpan c1 = c_L.card[0], c2 = c_L.card[1], m = c_L.cfg_m;
    for (int q = threadIdx.x; q < 2 * NTYPE * TYPE; q += blockDim.x) {
        int t = q / TYPE, j = q % TYPE;
        float acc = dot_col(J.card_feat + t * CARD_FEATS, W + c1.w, CARD_FEATS, TYPE, j, 0.0f);
        hid[t][j] = gelu(acc + B[c1.b + j]);
    }
    __syncthreads();
    for (int q = threadIdx.x; q < 2 * NTYPE * TYPE; q += blockDim.x) {
        int t = q / TYPE, j = q % TYPE;
        float acc = dot_col(&hid[t][0], W + c2.w, TYPE, TYPE, j, 0.0f);
        tok[t][j] = acc + B[c2.b + j];
        J.cards[q] = tok[t][j];
    }
    __syncthreads();
    for (int q = threadIdx.x; q < 2 * NTYPE * 3 * POOL; q += blockDim.x) {
        int t = q / (3 * POOL), j = q % (3 * POOL);
        J.cardm[q] = dot_col(&tok[t][0], W + m.w, TYPE, 3 * POOL, j, 0.0f);
    }
}

struct TrunkSmem {
    float x[N_HEXES * C];
    float a[N_HEXES * C];
    float mixed[N_HEXES * 2 * C];
    float y[N_HEXES * C];
    float tokens[NTYPE * TYPE];
    float proj[NTYPE * C];
    float pool[C];
    float glob[C];
    float pooled[2 * C];
    float gb[C];
    float facts[N_HEXES * HEX_FACTS];
    float piles[NTYPE * PILE];
    float loose[LOOSE];
    float input[2 * C + LOOSE];
    float P[D];
    float stat[2 * N_HEXES];
    int occ[N_HEXES];
};

// One network row through tokens, stem, the 8-block trunk, the board readout
// and the join projection (net.rs:558-731).
__global__ void k_trunk(const JobDev* __restrict__ jobs, const uint32_t* __restrict__ row_job,
                        const uint32_t* __restrict__ row_local, const float* __restrict__ W,
                        const float* __restrict__ B, const float* __restrict__ LN) {
    extern __shared__ float smem_raw[];
    TrunkSmem& S = *reinterpret_cast<TrunkSmem*>(smem_raw);
    const JobDev& J = jobs[row_job[blockIdx.x]];
    const uint32_t r = row_local[blockIdx.x];
    const uint8_t* row = J.gpu_rows + (size_t)J.row_gpu[r] * ROW_BYTES;
    const int tid = threadIdx.x, nt = blockDim.x;

    // expand the compact public row (rebel.rs:1144-1233)
    for (int h = tid; h < N_HEXES; h += nt) {
        uint8_t owner = row[ROW_HEX_OWNER + h], slot = row[ROW_HEX_SLOT + h], marker = row[ROW_HEX_MARKER + h];
        float* f = S.facts + h * HEX_FACTS;
        for (int k = 0; k < HEX_FACTS; ++k) f[k] = 0.0f;
        S.occ[h] = -1;
        if (owner != 255) {
            f[owner] = 1.0f;
            f[2] = (float)row[ROW_HEX_HEIGHT + h] / 5.0f;
            if (slot != 255) S.occ[h] = owner * NSLOT + slot;
        }
        if (marker != 255) f[3 + marker] = 1.0f;
        f[5] = c_is_location[h] ? 1.0f : 0.0f;
    }
    for (int q = tid; q < NTYPE * PILE; q += nt) S.piles[q] = (float)row[ROW_PILES + q] / 5.0f;
    if (tid == 0) {
        for (int p = 0; p < 2; ++p) {
            float* o = S.loose + 6 * p;
            uint8_t mh = row[ROW_MARKERS + p];
            o[0] = (float)mh / 6.0f;
            o[1] = (float)(6 - mh) / 6.0f;
            o[2] = (float)row[ROW_HAND + p] / 3.0f;
            o[3] = (float)row[ROW_FD + p] / 21.0f;
            o[4] = (float)row[ROW_BAG + p] / 21.0f;
            o[5] = row[ROW_INITIATIVE] == p ? 1.0f : 0.0f;
        }
        uint16_t plies = (uint16_t)(row[ROW_PLIES] | (row[ROW_PLIES + 1] << 8));
        S.loose[12] = (float)plies / 256.0f;
        S.loose[13] = row[ROW_INIT_MOVED] ? 1.0f : 0.0f;
        S.loose[14] = row[ROW_TO_ACT] == 0 ? 1.0f : 0.0f;
    }
    __syncthreads();
    // tokens: pile counts, then card token + seat embedding (view 0)
    const float* seat = W + c_L.seat;
    for (int q = tid; q < NTYPE * TYPE; q += nt) {
        int t = q / TYPE, j = q % TYPE;
        float acc = dot_col(S.piles + t * PILE, W + c_L.pile.w, PILE, TYPE, j, 0.0f);
        S.tokens[q] = acc + (J.cards[t * TYPE + j] + seat[(t / NSLOT) * TYPE + j]);
    }
    __syncthreads();
    for (int q = tid; q < NTYPE * C; q += nt) {
        int t = q / C, j = q % C;
        S.proj[q] = dot_col(S.tokens + t * TYPE, W + c_L.tok_stem.w, TYPE, C, j, 0.0f);
    }
    for (int j = tid; j < C; j += nt) S.glob[j] = dot_col(S.loose, W + c_L.glob_stem.w, LOOSE, C, j, 0.0f);
    __syncthreads();
    for (int j = tid; j < C; j += nt) {
        float acc = 0.0f;
        for (int t = 0; t < NTYPE; ++t) acc += gelu(S.proj[t * C + j]) / (float)NTYPE;
        S.pool[j] = acc;
    }
    __syncthreads();
    const float* pos = W + c_L.pos;
    for (int q = tid; q < N_HEXES * C; q += nt) {
        int h = q / C, j = q % C;
        float acc = dot_col(S.facts + h * HEX_FACTS, W + c_L.hex_stem.w, HEX_FACTS, C, j, 0.0f) + B[c_L.hex_stem.b + j];
        float occ = S.occ[h] >= 0 ? S.proj[S.occ[h] * C + j] : 0.0f;
        S.x[q] = acc + (occ + pos[h * C + j] + S.glob[j] + S.pool[j]);
    }
    // residual blocks
    for (int i = 0; i < wc::NET_BLOCKS; ++i) {
        __syncthreads();
        for (int q = tid; q < N_HEXES * C; q += nt) S.a[q] = S.x[q];
        ln_rows(S.a, N_HEXES, C, NetLayout::ln_block(i, 0), true, S.stat, LN);
        for (int q = tid; q < N_HEXES * C; q += nt) {
            int h = q / C, j = q % C;
            S.mixed[h * 2 * C + j] = S.a[q];
            float acc = 0.0f;
            for (int d = 0; d < 6; ++d) {
                uint8_t nb = c_neighbors[h][d];
                if (nb == 255) continue;
                acc += S.a[nb * C + j];
            }
            S.mixed[h * 2 * C + C + j] = acc;
        }
        for (int j = tid; j < C; j += nt) {
            float mean = 0.0f, mx = -INFINITY;
            for (int h = 0; h < N_HEXES; ++h) {
                float v = S.a[h * C + j];
                mean += v / (float)N_HEXES;
                mx = fmaxf(mx, v);
            }
            S.pooled[j] = mean;
            S.pooled[C + j] = mx;
        }
        __syncthreads();
        const wc::NetSpan mx = c_L.mix[i], pl = c_L.pool[i], ou = c_L.out[i];
        for (int j = tid; j < C; j += nt) S.gb[j] = dot_col(S.pooled, W + pl.w, 2 * C, C, j, 0.0f) + B[pl.b + j];
        __syncthreads();
        for (int q = tid; q < N_HEXES * C; q += nt) {
            int h = q / C, j = q % C;
            float acc = dot_col(S.mixed + h * 2 * C, W + mx.w, 2 * C, C, j, 0.0f) + B[mx.b + j];
            S.y[q] = acc + S.gb[j];
        }
        ln_rows(S.y, N_HEXES, C, NetLayout::ln_block(i, 1), true, S.stat, LN);
        for (int q = tid; q < N_HEXES * C; q += nt) {
            int h = q / C, j = q % C;
            float z = dot_col(S.y + h * C, W + ou.w, C, C, j, 0.0f) + B[ou.b + j];
            S.x[q] += z;
        }
    }
    ln_rows(S.x, N_HEXES, C, NetLayout::LN_TRUNK, true, S.stat, LN);
    for (int j = tid; j < C; j += nt) {
        float mean = 0.0f, mx = -INFINITY;
        for (int h = 0; h < N_HEXES; ++h) {
            float v = S.x[h * C + j];
            mean += v / (float)N_HEXES;
            mx = fmaxf(mx, v);
        }
        S.input[j] = mean;
        S.input[C + j] = mx;
    }
    for (int j = tid; j < LOOSE; j += nt) S.input[2 * C + j] = S.loose[j];
    __syncthreads();
    const wc::NetSpan bo = c_L.board_out;
    for (int j = tid; j < D; j += nt) {
        float v = dot_col(S.input, W + bo.w, 2 * C + LOOSE, D, j, 0.0f) + B[bo.b + j];
        S.P[j] = v;
        J.pb[(size_t)r * D + j] = v;
    }
    __syncthreads();
    for (int j = tid; j < JW; j += nt) J.jp[(size_t)r * JW + j] = dot_col(S.P, W + c_L.join_p.w, D, JW, j, 0.0f);
}

// f(c) and g(c) for one interned config (net.rs:735-797).
__global__ void k_configs(const JobDev* __restrict__ jobs, const uint32_t* __restrict__ cfg_job,
                          const uint32_t* __restrict__ cfg_local, const float* __restrict__ W,
                          const float* __restrict__ B, const float* __restrict__ LN) {
    const JobDev& J = jobs[cfg_job[blockIdx.x]];
    const uint32_t c = cfg_local[blockIdx.x];
    __shared__ float slots[NSLOT][3 + TYPE];
    __shared__ float hid[NSLOT][CFGH];
    __shared__ float u[CFGH];
    __shared__ float stat[2];
    const int tid = threadIdx.x, nt = blockDim.x;
    const float* phi = J.cphi + (size_t)c * 15;
    const int q = J.cplayer[c];
    for (int x = tid; x < NSLOT * (3 + TYPE); x += nt) {
        int k = x / (3 + TYPE), i = x % (3 + TYPE);
        float v;
        if (i < 3) v = phi[i * NSLOT + k];
        else v = J.cards[(q * NTYPE + k) * TYPE + (i - 3)];
        slots[k][i] = v;
    }
    __syncthreads();
    const wc::NetSpan c1 = c_L.cfg1;
    for (int x = tid; x < NSLOT * CFGH; x += nt) {
        int k = x / CFGH, j = x % CFGH;
        hid[k][j] = gelu(dot_col(&slots[k][0], W + c1.w, 3 + TYPE, CFGH, j, 0.0f) + B[c1.b + j]);
    }
    __syncthreads();
    for (int j = tid; j < CFGH; j += nt) {
        float acc = 0.0f;
        for (int k = 0; k < NSLOT; ++k) acc += hid[k][j];
        u[j] = acc;
    }
    ln_rows(u, 1, CFGH, NetLayout::LN_CFG, true, stat, LN);
    const wc::NetSpan cf = c_L.cfg_f, cg = c_L.cfg_g;
    for (int j = tid; j < D; j += nt) J.cf[(size_t)c * D + j] = dot_col(u, W + cf.w, CFGH, D, j, 0.0f) + B[cf.b + j];
    for (int j = tid; j < POOL; j += nt) {
        float g = dot_col(u, W + cg.w, CFGH, POOL, j, 0.0f) + B[cg.b + j];
        for (int k = 0; k < NSLOT; ++k) {
            const float* v = J.cardm + (size_t)(q * NTYPE + k) * 3 * POOL;
            for (int zone = 0; zone < 3; ++zone) {
                float count = phi[zone * NSLOT + k];
                if (count == 0.0f) continue;
                g += count * v[zone * POOL + j];
            }
        }
        J.cg[(size_t)c * POOL + j] = g;
    }
}

// Pooled belief embeddings of one network row (search.rs:1512-1547): per
// player, normalised reach over the leaf's configs weighting g(c).
__global__ void k_pool(const JobDev* __restrict__ jobs, const uint32_t* __restrict__ row_job,
                       const uint32_t* __restrict__ row_local, int mask) {
    const JobDev& J = jobs[row_job[blockIdx.x]];
    const uint32_t r = row_local[blockIdx.x];
    const int q = threadIdx.x / POOL, j = threadIdx.x % POOL;
    if (!(mask & (1 << q))) return;
    const float* w = J.reach + J.lr_ridx[2 * r + q];
    const uint32_t n = J.lr_nc[2 * r + q];
    const uint32_t* idx = J.leaf_cidx + J.leaf_coff[2 * r + q];
    float tot = 0.0f;
    for (uint32_t c = 0; c < n; ++c) tot += w[c];
    float scale, flat;
    if (tot > 1e-30f) { scale = 1.0f / tot; flat = 0.0f; }
    else { scale = 0.0f; flat = 1.0f / (float)(n > 0 ? n : 1); }
    float acc = 0.0f;
    for (uint32_t c = 0; c < n; ++c) acc += (w[c] * scale + flat) * J.cg[(size_t)idx[c] * POOL + j];
    J.pooled[((size_t)r * 2 + q) * POOL + j] = acc;
}

// The join for traverser p and the readout of p's configs (net.rs:801-853,
// search.rs:1587-1636).
__global__ void k_join_readout(const JobDev* __restrict__ jobs, const uint32_t* __restrict__ row_job,
                               const uint32_t* __restrict__ row_local, int p, const float* __restrict__ W,
                               const float* __restrict__ B, const float* __restrict__ LN) {
    const JobDev& J = jobs[row_job[blockIdx.x]];
    const uint32_t r = row_local[blockIdx.x];
    __shared__ float in[wc::NET_JOIN_IN];
    __shared__ float z[JW];
    __shared__ float t[JW];
    __shared__ float h[D];
    __shared__ float stat[2];
    __shared__ float opp_mass;
    const int tid = threadIdx.x, nt = blockDim.x;
    for (int j = tid; j < POOL; j += nt) {
        in[j] = J.pooled[((size_t)r * 2 + p) * POOL + j];
        in[POOL + j] = J.pooled[((size_t)r * 2 + 1 - p) * POOL + j];
    }
    if (tid == 0) in[2 * POOL] = p == 0 ? -1.0f : 1.0f;
    __syncthreads();
    const wc::NetSpan jb = c_L.join_b;
    for (int j = tid; j < JW; j += nt)
        z[j] = dot_col(in, W + jb.w, wc::NET_JOIN_IN, JW, j, J.jp[(size_t)r * JW + j]) + B[jb.b + j];
    for (int i = 0; i < wc::NET_JBLOCKS; ++i) {
        __syncthreads();
        for (int j = tid; j < JW; j += nt) t[j] = z[j];
        ln_rows(t, 1, JW, NetLayout::LN_JOIN + i, true, stat, LN);
        const wc::NetSpan jw = c_L.join_w[i];
        float d[JW / 32 > 0 ? JW / 32 : 1];
        int n = 0;
        for (int j = tid; j < JW; j += nt) d[n++] = dot_col(t, W + jw.w, JW, JW, j, 0.0f) + B[jw.b + j];
        __syncthreads();
        n = 0;
        for (int j = tid; j < JW; j += nt) z[j] += d[n++];
    }
    ln_rows(z, 1, JW, NetLayout::LN_JOUT, true, stat, LN);
    const wc::NetSpan jo = c_L.join_out;
    for (int j = tid; j < D; j += nt)
        h[j] = dot_col(z, W + jo.w, JW, D, j, J.pb[(size_t)r * D + j]) + B[jo.b + j];
    ln_rows(h, 1, D, NetLayout::LN_H, false, stat, LN);
    if (tid == 0) {
        const float* ro = J.reach + J.lr_ridx[2 * r + 1 - p];
        uint32_t no = J.lr_nc[2 * r + 1 - p];
        float s = 0.0f;
        for (uint32_t c = 0; c < no; ++c) s += ro[c];
        opp_mass = s;
    }
    __syncthreads();
    const uint32_t n = J.lr_nc[2 * r + p];
    const uint32_t* idx = J.leaf_cidx + J.leaf_coff[2 * r + p];
    float* out = J.vals[p] + J.lr_vidx[2 * r + p];
    const float vb = B[c_L.value_bias];
    for (uint32_t c = tid; c < n; c += nt) {
        const float* f = J.cf + (size_t)idx[c] * D;
        float v = vb;
        for (int j = 0; j < D; ++j) v += f[j] * h[j];
        out[c] = v * opp_mass;
    }
}

// ------------------------------------------------------------- launchers

void net_set_constants(const NetLayout& L, const uint8_t* neighbors, const uint8_t* is_location) {
    cudaMemcpyToSymbol(c_L, &L, sizeof(NetLayout));
    cudaMemcpyToSymbol(c_neighbors, neighbors, 37 * 6);
    cudaMemcpyToSymbol(c_is_location, is_location, 37);
}

void launch_cards(const JobDev* jobs, uint32_t njobs, const float* W, const float* B, cudaStream_t s) {
    if (njobs) k_cards<<<njobs, 256, 0, s>>>(jobs, W, B);
}

void launch_trunk(const JobDev* jobs, const uint32_t* row_job, const uint32_t* row_local, uint32_t nrows,
                  const float* W, const float* B, const float* LN, cudaStream_t s) {
    if (!nrows) return;
    size_t smem = sizeof(TrunkSmem);
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(k_trunk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        configured = true;
    }
    k_trunk<<<nrows, 384, smem, s>>>(jobs, row_job, row_local, W, B, LN);
}

void launch_configs(const JobDev* jobs, const uint32_t* cfg_job, const uint32_t* cfg_local, uint32_t ncfg,
                    const float* W, const float* B, const float* LN, cudaStream_t s) {
    if (ncfg) k_configs<<<ncfg, 128, 0, s>>>(jobs, cfg_job, cfg_local, W, B, LN);
}

void launch_pool(const JobDev* jobs, const uint32_t* row_job, const uint32_t* row_local, uint32_t nrows, int mask,
                 cudaStream_t s) {
    if (nrows) k_pool<<<nrows, 2 * POOL, 0, s>>>(jobs, row_job, row_local, mask);
}

void launch_join_readout(const JobDev* jobs, const uint32_t* row_job, const uint32_t* row_local, uint32_t nrows,
                         int p, const float* W, const float* B, const float* LN, cudaStream_t s) {
    if (nrows) k_join_readout<<<nrows, 128, 0, s>>>(jobs, row_job, row_local, p, W, B, LN);
}

}  // namespace wcdev
