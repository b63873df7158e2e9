// Descriptors shared by the host runtime and the kernels.
//
// A batch holds many independent subgame solves ("jobs"). Every job keeps its
// own job-local index space (see host/job.h); a JobDev carries the device
// pointers of that job's tables and state. Per-level kernels run over work
// items, each a bounded slice of one job's task list, so a CTA resolves its
// job once and then streams contiguous tasks.
#pragma once
#include <cstdint>

namespace wcdev {

constexpr int WI_TASKS = 256;  // tasks per work item == threads per CTA

struct JobDev {
    // ---- immutable tables
    const uint32_t* cell_vidx;
    const uint32_t* row_off;
    const uint8_t* row_player;
    const uint32_t* vg_start;
    const uint32_t* vge_idx;
    const uint32_t* vge_w;
    const uint32_t* rg_start;
    const uint32_t* rge_src;
    const uint32_t* rge_w;
    const float* drawp;
    const uint32_t* cell_ref;
    const uint32_t* lr_ridx;
    const uint32_t* lr_nc;
    const uint32_t* lr_vidx;
    const uint32_t* leaf_coff;
    const uint32_t* leaf_cidx;
    const uint32_t* tl_ridx;
    const uint32_t* tl_nc;
    const uint32_t* tl_vidx;
    const float* tl_util0;
    const uint8_t* gpu_rows;
    const float* cphi;
    const uint8_t* cplayer;
    const float* card_feat;
    const float* root_belief;
    const float* carried;
    const uint32_t* carry_off;  // nexit + 1
    const float* weights_w;     // network blob (device), shared by all jobs
    const float* weights_b;
    const float* weights_ln;
    float* cardm;      // [2][NTYPE][3 * POOL]: cfg_m applied to the card tokens
    // ---- mutable solve state
    float* cur;
    float* regret;
    float* sum;
    float* snap;       // latest materialised average (sorted cells)
    float* reach;
    float* reach2;     // scratch reach arena for carried beliefs
    float* vals[2];    // per-traverser value arenas
    // ---- network state (per solve)
    float* cards;      // [2][NTYPE][TYPE]
    float* pb;         // [rows][D]
    float* jp;         // [rows][JW]
    float* cf;         // [ncfg][D]
    float* cg;         // [ncfg][POOL]
    float* pooled;     // [rows][2][POOL]
    float* h;          // [rows][D]
    // ---- outputs
    float* out_strategy;   // ncells, reference order
    float* out_roots;      // ncarried * (root_nc0 + root_nc1)
    uint16_t* out_carry;   // (nsnaps - 1) * carry_width, f16
    // ---- sizes
    uint32_t ncells, ndraw, nrows_net, nterm, ncfg, ncarried, reach_len, nexit;
    uint32_t root_nc[2], root_rblk[2], root_vblk[2];
    uint32_t carry_width;  // sum over exit nodes of nc0 + nc1
};

struct WorkItem {
    uint32_t job, first, count, out_first;
};

}  // namespace wcdev
