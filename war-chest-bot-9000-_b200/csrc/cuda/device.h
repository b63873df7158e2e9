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
constexpr int ROW_CELL_CAP = 2048;  // cells of a regret-matching work item staged in shared memory

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
    const uint8_t* gpu_rows;   // the distinct public rows (201 bytes each)
    const uint32_t* row_gpu;   // per network row: its public row's index in gpu_rows
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
    const uint32_t* cfg_col;  // config -> index among its player's configs
    uint32_t* leaf_col;       // per leaf_cidx entry: its config's cfg_col (the readout column), derived on
                              // the device at upload (k_leaf_col), so host tables do not carry it
    uint16_t* f16;     // fast path: f(c) as readout operand images, 128 configs x D each (64 KB),
                       // player 0's ceil(n0 / 128) passes then player 1's
    uint16_t* g16;     // fast path: g(c) as pooling operand images, 64 x 128 configs each (16 KB), same order
    uint32_t ncfg_player[2];
    uint32_t row_base; // first global network row of this job
    uint32_t tile_base; // first 128-row leaf tile of this job (tensor-core path)
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
    float* tokproj;    // fast path: [NTYPE][C] = (cards + seat) W_tok, the per-job part of the token projection
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
    float* out_conv;       // 2 * (root_nc0 + root_nc1): root values under the average, then best responses
    // ---- sizes
    uint32_t ncells, ndraw, nrows_net, nterm, ncfg, ncarried, reach_len, nexit;
    uint32_t root_nc[2], root_rblk[2], root_vblk[2];
    uint32_t carry_width;  // sum over exit nodes of nc0 + nc1
};

// Device pointers of the bf16 tensor-core network (one per device): weight
// matrices as swizzled K-major B tiles ([out][in], see umma.cuh), fp32 bias
// and LayerNorm vectors.
struct FastNetDev {
    const uint8_t* join_tiles;  // join_b (inputs 0..127), join_w[0..2]: 4 x [128][128]
    const uint8_t* out_tile;    // join_out: [256][128]
    const uint8_t* trunk_tiles; // per trunk block: mix [96][192], out [96][96]
    const float* beff[2];       // join_b bias with the seat input (-1 / +1) folded in
    const float* bj[3];
    const float* bout;
    const float* ln_g[5];       // LN_JOIN + 0..2, LN_JOUT, LN_H
    const float* ln_b[5];
    float vbias;
    const float* pile_tok;      // [4][96] = W_pile W_tok: pile counts straight to the token projection
    const float* trunk_pb;      // per trunk block [96]: the pooling bias plus the mix bias (both add to y)
    const float* trunk_ob;      // per trunk block [96]: the out bias
    const float* stem_w;        // [6][96] the hex stem weights (16-byte aligned copy)
    const float* stem_pb;       // [37][96] the hex's position embedding plus the hex stem bias
    int half;                   // the per-iteration chain's operands (pooling, join, join output): 1 = f16,
                                // 0 = bf16; the trunk, P / jp and the readout are f16 in both
    uint64_t wait_ns;           // limit of each mbarrier wait, ns of %globaltimer (umma::WAIT_NS)
};

struct WorkItem {
    uint32_t job, first, count, out_first;
};

}  // namespace wcdev
