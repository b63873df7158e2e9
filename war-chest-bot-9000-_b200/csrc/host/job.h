// The flattened device image of one subgame solve ("job").
//
// The reference ships a built tree to its GPU service as a PackedJob
// (engine/src/serialize.rs:143-150, docs/TREE.md); this is the B200 layout
// of the same contract, built from the same tree:
//
//   * nodes are grouped by public-tree level (root = 0);
//   * legal cells are sorted by (level, acting player, node, config row), so
//     every (level, player) set of regret-matching rows is one contiguous
//     CSR range of the cell arenas (regret, current, running sum);
//   * reach blocks are allocated per (level, moving player); the idle
//     player's reach at a child is the parent's block (aliased, never
//     copied), and every (level, mover) output range is contiguous;
//   * each traverser has its own value arena, allocated per level as
//     [own decision rows | other non-leaf nodes | leaves];
//   * every gather list (reach into a child config, value into a node) keeps
//     the reference CPU solver's accumulation order (search.rs:1322-1348,
//     1692-1700, 1720-1740, 1794-1800), so a sequential per-output sum is
//     bit-identical to the oracle.
// All indices are job-local; a batch gives each job its own device arenas.
#pragma once
#include <cstdint>
#include <memory>
#include <vector>

#include "roots.h"

namespace wc {

// Work kinds of a per-level task list.
enum TaskKind : uint32_t { TK_ROWS = 0, TK_VGATHER = 1, TK_RGATHER = 2 };

struct LevelRange {
    uint32_t first = 0, count = 0, out_first = 0;
};

struct JobImage {
    SolveCfg cfg;
    uint32_t nodes = 0, ncells = 0, ndraw = 0, nlevels = 0;
    uint32_t nrows_net = 0, nterm = 0, ncfg = 0, ndec_rows = 0;
    uint32_t root_nc[2] = {0, 0};
    uint32_t reach_len = 0, val_len[2] = {0, 0};
    // cells, sorted
    std::vector<uint32_t> cell_ref;   // sorted cell -> reference cell
    std::vector<uint32_t> cell_vidx;  // successor value index in the acting player's value arena
    std::vector<uint32_t> row_off;    // ndec_rows + 1, over sorted cells
    std::vector<uint8_t> row_player;  // acting player of each row
    // per (level, player): ranges in row / vgather / rgather task spaces
    std::vector<LevelRange> rows_rng, vg_rng, rg_rng;  // index: level * 2 + player
    std::vector<uint32_t> vg_start, vge_idx, vge_w;
    std::vector<uint32_t> rg_start, rge_src, rge_w;
    std::vector<float> drawp;         // ndraw + 1, last entry 1.0
    uint32_t root_rblk[2] = {0, 0};   // root reach blocks
    uint32_t root_vblk[2] = {0, 0};   // root value blocks (per traverser arena)
    // network rows (reference leaf_rows order) and terminal leaves
    std::vector<uint32_t> lr_ridx, lr_nc, lr_vidx;  // [2 * nrows_net] player-major per row: [r*2+q]
    std::vector<uint32_t> leaf_coff, leaf_cidx;
    std::vector<uint32_t> tl_ridx, tl_nc, tl_vidx;  // [2 * nterm]
    std::vector<float> tl_util0;                    // utility for player 0
    std::vector<uint8_t> gpu_rows;                  // the distinct public rows, GPU_ROW_BYTES each
    std::vector<uint32_t> row_rep;                  // per network row: the first row with the same public row bytes
    std::vector<uint32_t> row_gpu;                  // per network row: its public row's index in gpu_rows
    std::vector<float> cphi;                        // ncfg * CFEAT
    std::vector<uint8_t> cplayer;
    std::vector<uint32_t> cfg_col;                  // index of each config among its player's configs
    uint32_t ncfg_player[2] = {0, 0};
    std::vector<float> card_feat;                   // 2 views * NTYPE * CARD_FEATS
    // root beliefs and the carried roots Phase 2 values
    std::vector<float> root_belief;                 // root_nc[0] + root_nc[1]
    std::vector<float> carried;                     // ncarried * (root_nc[0] + root_nc[1])
    uint32_t ncarried = 0;
    // bookkeeping for the reference layout
    std::vector<uint32_t> exit_nodes;               // network rows then terminal leaves (reference ids)
    std::vector<uint32_t> snap_iters;
    size_t table_bytes() const;
};

// Flatten a built tree. `carried` holds ncarried root pairs (p0 then p1); when
// empty the live root belief is the single Phase-2 root, as the reference's
// first level (selfplay.rs:716-733).
std::unique_ptr<JobImage> flatten(const Tree& t, const std::vector<float>& carried, uint32_t ncarried);

}  // namespace wc
