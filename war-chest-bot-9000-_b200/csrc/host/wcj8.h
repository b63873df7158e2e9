// The reference's job byte format, WCJ8 (engine/src/serialize.rs:33-150
// PackedMeta / PackedTables / PackedJob, 689-955 PackedTables::from_solver,
// 1051-1262 to_bytes / from_bytes; docs/TREE.md): little-endian, a u32 count
// before every array, f32 floats. The writer flattens a built tree into the
// reference's tables exactly as its from_solver does, so the bytes are the
// ones the reference engine would send its GPU service for the same subgame;
// the reader parses such bytes (with the reference's count checks) back into a
// tree this library's flattener turns into a device job.
#pragma once
#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "tree.h"

namespace wc {

constexpr uint32_t WCJ8_MAGIC = 0x57434A38u;  // "WCJ8"
constexpr uint32_t WCJ8_VERSION = 8;

struct Wcj8Job {
    // meta (serialize.rs:38-51)
    uint32_t depth = 0, iters = 0;
    bool snapshots = false;
    float alpha = 0, beta = 0, gamma = 0, predict = 0;
    std::vector<uint32_t> snap_iters, net_dims;
    // tables (serialize.rs:55-136)
    uint32_t nodes = 0, ncfg = 0, rows = 0, ncells = 0;
    std::vector<uint8_t> node_kind, node_player;
    std::vector<uint32_t> node_child_start, node_child, obs_off, obs_start, obs_act, obs_child;
    std::vector<uint32_t> legal_row_of, legal_off, legal_action, legal_child, legal_trans, cell_row;
    std::vector<uint32_t> draw_off, draw_to;
    std::vector<float> draw_p;
    std::vector<uint32_t> draw_row_off, draw_row_start, cfg_off, reach_off, soff;
    std::vector<uint32_t> node_parent, rev_row_of, rev_start, rev_src, rev_cell;
    std::vector<uint32_t> rvd_row_of, rvd_start, rvd_src;
    std::vector<float> rvd_p;
    std::vector<uint32_t> leaf_rows, term_leaves;
    std::vector<float> terminal_utility;
    std::vector<uint32_t> leaf_coff, leaf_cidx, snap_coff;
    std::vector<uint8_t> leaf_raw;
    std::vector<float> card_feat, cphi;
    std::vector<uint8_t> cplayer;
    std::vector<uint32_t> bfs_order, level_start;
    // beliefs (serialize.rs:143-150): the live root, then the carried roots
    std::vector<float> root[2];
    std::vector<std::vector<float>> carried[2];
};

// PackedJob::from_solver (serialize.rs:340-357, 689-955) of a built, uncapped
// tree; `carried` holds ncarried root pairs [p0 | p1].
Wcj8Job wcj8_from_tree(const Tree& t, const std::vector<float>& carried, uint32_t ncarried,
                       const std::vector<uint32_t>& net_dims);
// to_bytes (serialize.rs:1051-1125).
std::vector<uint8_t> wcj8_write(const Wcj8Job& j);
// from_bytes (serialize.rs:1127-1240): false with a message on malformed
// input (bad magic or version, truncated or trailing bytes, a count that
// disagrees with the header).
bool wcj8_read(const uint8_t* data, size_t n, Wcj8Job* out, std::string* err);
// A tree the flattener can solve, rebuilt from the tables (structure, config
// support sizes, legal cells, draws, leaves, configs, public rows, card ids
// recovered from the card facts), and the carried roots as flatten takes
// them. Support entries are placeholders: a solve reads only their counts.
std::unique_ptr<Tree> wcj8_tree(const Wcj8Job& j, std::vector<float>* carried, uint32_t* ncarried,
                                std::string* err);

}  // namespace wc
