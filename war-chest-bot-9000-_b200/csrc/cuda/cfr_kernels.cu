// CFR kernels: level-synchronous sweeps over a batch of independent subgames.
//
// Compiled with -fmad=false: every a*b+c below is a rounded product followed
// by a rounded add, and every per-output accumulation runs sequentially in
// the order the host flattener emitted, which is the reference CPU solver's
// order (engine/src/search.rs:1273-1351 reach, 1654-1803 backprop,
// 1818-1835 average, 899-938 snapshot). With a zero or empty value network a
// batch solve therefore reproduces the CPU oracle bit for bit.
//
// Memory layout: see host/job.h. One CTA per work item, one thread per task.
#include <cuda_fp16.h>

#include <algorithm>
#include <cfloat>
#include <cstdint>

#include "device.h"
#include "kernels.h"

namespace wcdev {

// Weight of a gather entry: a strategy cell, a draw probability, or 1.
__device__ __forceinline__ float entry_weight(const JobDev& J, const float* strat, uint32_t w) {
    return w < J.ncells ? strat[w] : J.drawp[w - J.ncells];
}

__device__ __forceinline__ const float* pick_strat(const JobDev& J, int strat_sel) {
    return strat_sel == STRAT_CUR ? J.cur : J.snap;
}

// Uniform initial strategy, zero regrets and sums (search.rs:820-836).
// The readout column of every leaf-config entry (leaf_col[e] =
// cfg_col[leaf_cidx[e]]), derived on the device after a job's tables land:
// one grid row of blocks per job, grid-stride over its entries.
__global__ void k_leaf_col(const JobDev* __restrict__ jobs, uint32_t first) {
    const JobDev& J = jobs[first + blockIdx.y];
    const uint32_t n = J.leaf_coff[2 * J.nrows_net];
    for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < n; e += gridDim.x * blockDim.x)
        J.leaf_col[e] = J.cfg_col[J.leaf_cidx[e]];
}

__global__ void k_init_rows(const JobDev* __restrict__ jobs, const WorkItem* __restrict__ items) {
    const WorkItem wi = items[blockIdx.x];
    if (threadIdx.x >= wi.count) return;
    const JobDev& J = jobs[wi.job];
    uint32_t row = wi.first + threadIdx.x;
    uint32_t lo = J.row_off[row], hi = J.row_off[row + 1];
    float k = (float)(hi - lo);
    for (uint32_t c = lo; c < hi; ++c) {
        J.cur[c] = 1.0f / k;
        J.regret[c] = 0.0f;
        J.sum[c] = 0.0f;
    }
}

// Traverser decision rows: node value under the strategy, then (regret mode)
// the fused regret update and regret matching with the 1e-6 floor.
// In regret mode an item's cells (at most ROW_CELL_CAP) are staged in shared
// memory: child values (gathered), strategy and regrets come in, and the new
// regrets and strategy go out, by coalesced cell-parallel loops; each row's
// arithmetic is the same sequence as below, on the staged copies.
__global__ void k_rows(const JobDev* __restrict__ jobs, const WorkItem* __restrict__ items, int p, int mode,
                       int strat_sel, float da, float db, float predict) {
    __shared__ float s_val[ROW_CELL_CAP], s_str[ROW_CELL_CAP], s_reg[ROW_CELL_CAP];
    const WorkItem wi = items[blockIdx.x];
    const JobDev& J = jobs[wi.job];
    if (mode == BACK_REGRET) {
        const uint32_t c0 = J.row_off[wi.first], nc = J.row_off[wi.first + wi.count] - c0;
        if (nc <= (uint32_t)ROW_CELL_CAP) {
            float* vals = J.vals[p];
            const float* strat = pick_strat(J, strat_sel);
            for (uint32_t i = threadIdx.x; i < nc; i += blockDim.x) {
                s_val[i] = vals[J.cell_vidx[c0 + i]];
                s_str[i] = strat[c0 + i];
                s_reg[i] = J.regret[c0 + i];
            }
            __syncthreads();
            if (threadIdx.x < wi.count) {
                const uint32_t row = wi.first + threadIdx.x;
                const uint32_t lo = J.row_off[row] - c0, hi = J.row_off[row + 1] - c0;
                float base = 0.0f;
                for (uint32_t c = lo; c < hi; ++c) base += s_val[c] * s_str[c];
                const float EPS = 1e-6f;
                float s = 0.0f;
                for (uint32_t c = lo; c < hi; ++c) {
                    float delta = 0.0f;
                    delta += s_val[c];
                    delta -= base;
                    float old = s_reg[c];
                    float r = old * (old > 0.0f ? da : db) + delta;
                    s_reg[c] = r;
                    float v = fmaxf(r + predict * delta, EPS);
                    s_str[c] = v;
                    s += v;
                }
                if (s > 0.0f) {
                    float inv = 1.0f / s;
                    for (uint32_t c = lo; c < hi; ++c) s_str[c] *= inv;
                }
                vals[wi.out_first + threadIdx.x] = base;
            }
            __syncthreads();
            for (uint32_t i = threadIdx.x; i < nc; i += blockDim.x) {
                J.regret[c0 + i] = s_reg[i];
                J.cur[c0 + i] = s_str[i];
            }
            return;
        }
    }
    if (threadIdx.x >= wi.count) return;
    uint32_t row = wi.first + threadIdx.x;
    uint32_t lo = J.row_off[row], hi = J.row_off[row + 1];
    float* vals = J.vals[p];
    const uint32_t* vidx = J.cell_vidx;
    float base;
    if (mode == BACK_BEST) {
        base = -INFINITY;
        for (uint32_t c = lo; c < hi; ++c) base = fmaxf(base, vals[vidx[c]]);
        if (base == -INFINITY) base = 0.0f;
    } else {
        const float* strat = pick_strat(J, strat_sel);
        base = 0.0f;
        for (uint32_t c = lo; c < hi; ++c) base += vals[vidx[c]] * strat[c];
    }
    if (mode == BACK_REGRET) {
        const float EPS = 1e-6f;
        float s = 0.0f;
        for (uint32_t c = lo; c < hi; ++c) {
            float delta = 0.0f;
            delta += vals[vidx[c]];
            delta -= base;
            float old = J.regret[c];
            float r = old * (old > 0.0f ? da : db) + delta;
            J.regret[c] = r;
            float v = fmaxf(r + predict * delta, EPS);
            J.cur[c] = v;
            s += v;
        }
        if (s > 0.0f) {
            float inv = 1.0f / s;
            for (uint32_t c = lo; c < hi; ++c) J.cur[c] *= inv;
        }
    }
    vals[wi.out_first + threadIdx.x] = base;
}

// Opponent decision nodes (sum over children) and chance nodes (draw-weighted
// average, or pass-through) for traverser p.
__global__ void k_vgather(const JobDev* __restrict__ jobs, const WorkItem* __restrict__ items, int p) {
    const WorkItem wi = items[blockIdx.x];
    if (threadIdx.x >= wi.count) return;
    const JobDev& J = jobs[wi.job];
    uint32_t task = wi.first + threadIdx.x;
    uint32_t lo = J.vg_start[task], hi = J.vg_start[task + 1];
    float* vals = J.vals[p];
    float v = 0.0f;
    for (uint32_t e = lo; e < hi; ++e) v += J.drawp[J.vge_w[e] - J.ncells] * vals[J.vge_idx[e]];
    vals[wi.out_first + threadIdx.x] = v;
}

// Reach into one child config: sum over (parent config, weight) entries.
// With sum_update, every decision entry also folds the fresh reach-weighted
// strategy into the running sum: sum = sum * dg + reach * cur.
__global__ void k_rgather(const JobDev* __restrict__ jobs, const WorkItem* __restrict__ items, int strat_sel,
                          int which_reach, int sum_update, float dg) {
    const WorkItem wi = items[blockIdx.x];
    if (threadIdx.x >= wi.count) return;
    const JobDev& J = jobs[wi.job];
    uint32_t task = wi.first + threadIdx.x;
    uint32_t lo = J.rg_start[task], hi = J.rg_start[task + 1];
    float* reach = which_reach ? J.reach2 : J.reach;
    const float* strat = pick_strat(J, strat_sel);
    float acc = 0.0f;
    for (uint32_t e = lo; e < hi; ++e) {
        uint32_t w = J.rge_w[e];
        float prod;
        if (w < J.ncells) {
            prod = reach[J.rge_src[e]] * strat[w];
            if (sum_update) J.sum[w] = J.sum[w] * dg + prod;
        } else {
            prod = reach[J.rge_src[e]] * J.drawp[w - J.ncells];
        }
        acc += prod;
    }
    reach[wi.out_first + threadIdx.x] = acc;
}

// Terminal leaves: utility times the opponent's reach mass (search.rs:1591-1604).
__global__ void k_terminal(const JobDev* __restrict__ jobs, const WorkItem* __restrict__ items, int p) {
    const WorkItem wi = items[blockIdx.x];
    if (threadIdx.x >= wi.count) return;
    const JobDev& J = jobs[wi.job];
    uint32_t leaf = wi.first + threadIdx.x;
    int opp = 1 - p;
    const float* ro = J.reach + J.tl_ridx[2 * leaf + opp];
    uint32_t no = J.tl_nc[2 * leaf + opp];
    float s = 0.0f;
    for (uint32_t c = 0; c < no; ++c) s += ro[c];
    float u = p == 0 ? J.tl_util0[leaf] : -J.tl_util0[leaf];
    float v = u * s;
    float* out = J.vals[p] + J.tl_vidx[2 * leaf + p];
    uint32_t n = J.tl_nc[2 * leaf + p];
    for (uint32_t c = 0; c < n; ++c) out[c] = v;
}

// Network rows with no value network: every config is worth 0.
__global__ void k_netrows_zero(const JobDev* __restrict__ jobs, const WorkItem* __restrict__ items, int p) {
    const WorkItem wi = items[blockIdx.x];
    if (threadIdx.x >= wi.count) return;
    const JobDev& J = jobs[wi.job];
    uint32_t r = wi.first + threadIdx.x;
    float* out = J.vals[p] + J.lr_vidx[2 * r + p];
    uint32_t n = J.lr_nc[2 * r + p];
    for (uint32_t c = 0; c < n; ++c) out[c] = 0.0f;
}

// Seed both root reach blocks from the root belief or a carried root.
__global__ void k_seed_root(const JobDev* __restrict__ jobs, int which_reach, int carried_index) {
    const JobDev& J = jobs[blockIdx.x];
    float* reach = which_reach ? J.reach2 : J.reach;
    uint32_t n0 = J.root_nc[0], n1 = J.root_nc[1];
    const float* src;
    if (carried_index < 0) {
        src = J.root_belief;
    } else {
        if ((uint32_t)carried_index >= J.ncarried) return;
        src = J.carried + (size_t)carried_index * (n0 + n1);
    }
    for (uint32_t i = threadIdx.x; i < n0; i += blockDim.x) reach[J.root_rblk[0] + i] = src[i];
    for (uint32_t i = threadIdx.x; i < n1; i += blockDim.x) reach[J.root_rblk[1] + i] = src[n0 + i];
}

// Materialise the average strategy of every row (search.rs:913-937); a player
// whose sum was never updated keeps the literal current strategy.
__global__ void k_snapshot(const JobDev* __restrict__ jobs, const WorkItem* __restrict__ items, int touched0,
                           int touched1) {
    const WorkItem wi = items[blockIdx.x];
    if (threadIdx.x >= wi.count) return;
    const JobDev& J = jobs[wi.job];
    uint32_t row = wi.first + threadIdx.x;
    uint32_t lo = J.row_off[row], hi = J.row_off[row + 1];
    int touched = J.row_player[row] == 0 ? touched0 : touched1;
    if (!touched) {
        for (uint32_t c = lo; c < hi; ++c) J.snap[c] = J.cur[c];
        return;
    }
    float s = 0.0f;
    for (uint32_t c = lo; c < hi; ++c) s += J.sum[c];
    uint32_t len = hi - lo;
    float k = (float)(len > 0 ? len : 1);
    for (uint32_t c = lo; c < hi; ++c) J.snap[c] = s > 0.0f ? J.sum[c] / s : 1.0f / k;
}

// snapshot 0 is the literal initial strategy (search.rs:882-888)
__global__ void k_copy_cur_to_snap(const JobDev* __restrict__ jobs, const WorkItem* __restrict__ items) {
    const WorkItem wi = items[blockIdx.x];
    if (threadIdx.x >= wi.count) return;
    const JobDev& J = jobs[wi.job];
    uint32_t row = wi.first + threadIdx.x;
    for (uint32_t c = J.row_off[row]; c < J.row_off[row + 1]; ++c) J.snap[c] = J.cur[c];
}

// Final strategy back into the reference cell order.
__global__ void k_unsort(const JobDev* __restrict__ jobs, const WorkItem* __restrict__ items) {
    const WorkItem wi = items[blockIdx.x];
    if (threadIdx.x >= wi.count) return;
    const JobDev& J = jobs[wi.job];
    uint32_t c = wi.first + threadIdx.x;
    J.out_strategy[J.cell_ref[c]] = J.snap[c];
}

// Root values of one Phase-2 root for traverser p.
__global__ void k_collect_root(const JobDev* __restrict__ jobs, int root_index, int p) {
    const JobDev& J = jobs[blockIdx.x];
    if ((uint32_t)root_index >= J.ncarried) return;
    uint32_t n0 = J.root_nc[0], n = J.root_nc[p];
    float* out = J.out_roots + (size_t)root_index * (n0 + J.root_nc[1]) + (p == 1 ? n0 : 0);
    const float* v = J.vals[p] + J.root_vblk[p];
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) out[i] = v[i];
}

// NashConv passes (search.rs:1884-1907): the root block of traverser p's
// value arena into slot 0 (value under the average) or 1 (best response)
// of the job's conv output, [slot][player 0 configs | player 1 configs].
__global__ void k_collect_conv(const JobDev* __restrict__ jobs, int slot, int p) {
    const JobDev& J = jobs[blockIdx.x];
    const uint32_t n0 = J.root_nc[0], n = J.root_nc[p];
    float* out = J.out_conv + (size_t)slot * (n0 + J.root_nc[1]) + (p == 1 ? n0 : 0);
    const float* v = J.vals[p] + J.root_vblk[p];
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) out[i] = v[i];
}

// Normalised exit-leaf beliefs under one snapshot (search.rs:1937-1956),
// stored as f16 like the reference's carry store.
__global__ void k_carry(const JobDev* __restrict__ jobs, const WorkItem* __restrict__ items, int snap_index) {
    const WorkItem wi = items[blockIdx.x];
    if (threadIdx.x >= wi.count) return;
    const JobDev& J = jobs[wi.job];
    uint32_t e = wi.first + threadIdx.x;
    const uint32_t* ridx;
    const uint32_t* ncs;
    uint32_t k;
    if (e < J.nrows_net) { ridx = J.lr_ridx; ncs = J.lr_nc; k = e; }
    else { ridx = J.tl_ridx; ncs = J.tl_nc; k = e - J.nrows_net; }
    uint16_t* out = J.out_carry + (size_t)snap_index * J.carry_width + J.carry_off[e];
    for (int q = 0; q < 2; ++q) {
        const float* w = J.reach2 + ridx[2 * k + q];
        uint32_t n = ncs[2 * k + q];
        float tot = 0.0f;
        for (uint32_t c = 0; c < n; ++c) tot += w[c];
        float scale, flat;
        if (tot > 1e-30f) { scale = 1.0f / tot; flat = 0.0f; }
        else { scale = 0.0f; flat = 1.0f / (float)(n > 0 ? n : 1); }
        for (uint32_t c = 0; c < n; ++c) out[c] = __half_as_ushort(__float2half_rn(w[c] * scale + flat));
        out += n;
    }
}

// ------------------------------------------------------------- launchers

void launch_leaf_col(const JobDev* jobs, uint32_t njobs, cudaStream_t s) {
    for (uint32_t first = 0; first < njobs; first += 65535u)
        k_leaf_col<<<dim3(16, std::min(65535u, njobs - first)), 256, 0, s>>>(jobs, first);
}

void launch_init_rows(const JobDev* jobs, const WorkItem* items, uint32_t n, cudaStream_t s) {
    if (n) k_init_rows<<<n, WI_TASKS, 0, s>>>(jobs, items);
}
void launch_rows(const JobDev* jobs, const WorkItem* items, uint32_t n, int p, int mode, int strat_sel, float da,
                 float db, float predict, cudaStream_t s) {
    if (n) k_rows<<<n, WI_TASKS, 0, s>>>(jobs, items, p, mode, strat_sel, da, db, predict);
}
void launch_vgather(const JobDev* jobs, const WorkItem* items, uint32_t n, int p, cudaStream_t s) {
    if (n) k_vgather<<<n, WI_TASKS, 0, s>>>(jobs, items, p);
}
void launch_rgather(const JobDev* jobs, const WorkItem* items, uint32_t n, int strat_sel, int which_reach,
                    int sum_update, float dg, cudaStream_t s) {
    if (n) k_rgather<<<n, WI_TASKS, 0, s>>>(jobs, items, strat_sel, which_reach, sum_update, dg);
}
void launch_terminal(const JobDev* jobs, const WorkItem* items, uint32_t n, int p, cudaStream_t s) {
    if (n) k_terminal<<<n, WI_TASKS, 0, s>>>(jobs, items, p);
}
void launch_netrows_zero(const JobDev* jobs, const WorkItem* items, uint32_t n, int p, cudaStream_t s) {
    if (n) k_netrows_zero<<<n, WI_TASKS, 0, s>>>(jobs, items, p);
}
void launch_seed_root(const JobDev* jobs, uint32_t njobs, int which_reach, int carried_index, cudaStream_t s) {
    if (njobs) k_seed_root<<<njobs, 128, 0, s>>>(jobs, which_reach, carried_index);
}
void launch_snapshot(const JobDev* jobs, const WorkItem* items, uint32_t n, int t0, int t1, cudaStream_t s) {
    if (n) k_snapshot<<<n, WI_TASKS, 0, s>>>(jobs, items, t0, t1);
}
void launch_copy_cur_to_snap(const JobDev* jobs, const WorkItem* items, uint32_t n, cudaStream_t s) {
    if (n) k_copy_cur_to_snap<<<n, WI_TASKS, 0, s>>>(jobs, items);
}
void launch_unsort(const JobDev* jobs, const WorkItem* items, uint32_t n, cudaStream_t s) {
    if (n) k_unsort<<<n, WI_TASKS, 0, s>>>(jobs, items);
}
void launch_collect_root(const JobDev* jobs, uint32_t njobs, int root_index, int p, cudaStream_t s) {
    if (njobs) k_collect_root<<<njobs, 128, 0, s>>>(jobs, root_index, p);
}
void launch_collect_conv(const JobDev* jobs, uint32_t njobs, int slot, int p, cudaStream_t s) {
    if (njobs) k_collect_conv<<<njobs, 128, 0, s>>>(jobs, slot, p);
}
void launch_carry(const JobDev* jobs, const WorkItem* items, uint32_t n, int snap_index, cudaStream_t s) {
    if (n) k_carry<<<n, WI_TASKS, 0, s>>>(jobs, items, snap_index);
}

}  // namespace wcdev
