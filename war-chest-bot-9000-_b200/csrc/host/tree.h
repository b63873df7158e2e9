// Depth-limited public subgame trees, built exactly as the reference solver
// builds them (engine/src/search.rs:942-1255, node_actions :280-364,
// push_row/intern_config :1386-1462), but written straight into flat
// tree-wide CSR arrays instead of per-node vectors.
//
// Node ids are the reference's (DFS preorder: a parent before its children,
// public children in first-appearance order of their observation key), so a
// node's legal cells occupy soff[i]..soff[i+1] exactly as in the reference
// `Solver::soff`, and strategies are comparable cell for cell.
#pragma once
#include <cstdint>
#include <memory>
#include <unordered_map>
#include <vector>

#include "pbs.h"

namespace wc {

// CFR rule (search.rs:133-185).
struct CfrRule {
    float alpha, beta, gamma, predict;
    static CfrRule linear() { return {1.0f, 1.0f, 1.0f, 0.0f}; }
    static CfrRule plus();
    static CfrRule dcfr() { return {1.5f, 0.0f, 2.0f, 0.0f}; }
    static CfrRule pcfr();
    static CfrRule sapcfr();
    static bool named(const char* name, CfrRule* out);
};
// t^p / (t^p + 1) with the infinities evaluated (search.rs:187-193).
float cfr_factor(float t, float p);

// search.rs:50-95.
struct SolveCfg {
    int depth = 1;
    int iters = 64;
    bool snapshots = true;
    CfrRule cfr = CfrRule::linear();
    size_t node_cap = 0;
    bool keep_states = false;  // keep each node's State in Tree::states (search.rs:80, tests only)
};

std::vector<int> snapshot_iters(int iters);  // search.rs:102-110

constexpr uint32_t NO_TRANS = 0xFFFFFFFFu;
enum NodeKind : uint8_t { NK_DECISION = 0, NK_CHANCE = 1, NK_LEAF = 2 };

struct NodeRec {
    float util;          // terminal leaves: utility for `player`
    uint8_t player;
    uint8_t kind;
    uint8_t draw_steps;
    uint8_t terminal;    // leaf that is a terminal state
    uint32_t sup[2];     // support ids into Tree::supports
    uint32_t act_off;    // first action in acts/aslot/fdown/obs_child
    uint32_t na;
    uint32_t child_off;  // first public child in child[]
    uint32_t nch;
    uint32_t obs_off;    // obs_start segment (nch + 1 entries, node-local values)
    uint32_t row_off;    // legal_off segment (nc(player) + 1 entries, node-local values)
    uint32_t aoff_off;   // action_off segment (na + 1 entries, node-local values)
    uint32_t draw_off;   // chance: draw_start segment (rows + 1 entries, global values)
    uint32_t depth;      // public-tree level (root = 0)
};

struct Tree {
    Ctx ctx;
    SolveCfg cfg;
    Belief root_belief[2];
    bool capped = false;
    std::vector<NodeRec> nodes;
    std::vector<State> states;  // parallel to nodes when cfg.keep_states
    std::vector<std::vector<Config>> supports;
    // actions, per node contiguous
    std::vector<Action> acts;
    std::vector<int8_t> aslot;
    std::vector<uint8_t> fdown;
    std::vector<uint32_t> obs_child;  // action -> public-child index (node-local)
    // public children
    std::vector<uint32_t> child;
    std::vector<uint32_t> obs_start, obs_act;  // obs_act values node-local action ids; per node at act_off
    // legal cells (per node contiguous at soff[i])
    std::vector<uint32_t> soff;       // nodes + 1
    std::vector<uint32_t> legal_off;  // node-local row boundaries
    std::vector<uint32_t> legal_action, legal_child, legal_trans, cell_row;
    std::vector<uint32_t> action_off;   // node-local
    std::vector<uint32_t> action_cell;  // node-local cell ids, per node at soff[i]
    // draw maps (chance nodes)
    std::vector<uint32_t> draw_start;  // global offsets into draw_to/draw_p
    std::vector<uint32_t> draw_to;
    std::vector<float> draw_p;
    // leaf batch (search.rs:646-677)
    std::vector<uint32_t> leaf_rows, term_leaves;
    std::vector<uint32_t> leaf_coff, leaf_cidx;  // leaf_coff: 2 * rows + 1 entries
    std::vector<float> cphi;                     // ncfg * CFEAT
    std::vector<uint8_t> cplayer;
    std::vector<uint8_t> gpu_rows;               // rows * GPU_ROW_BYTES
    size_t ncfg = 0;
    uint8_t ids[2][NTYPE];                       // per seat view: unit index of each coin type

    size_t nc(uint32_t node, int p) const { return supports[nodes[node].sup[p]].size(); }
    size_t ncells() const { return soff.empty() ? 0 : soff.back(); }
    int max_depth() const;
};

// Build the subgame tree at `root` from both players' beliefs.
std::unique_ptr<Tree> build_tree(const State& root, const Ctx& ctx, const SolveCfg& cfg, const Belief bel[2]);

// The private actions at a node (search.rs:280-364).
void node_actions(const State& s, uint8_t player, const Ctx& ctx, const std::vector<Config>& cfgs,
                  std::vector<Action>& acts, std::vector<int8_t>& aslot, std::vector<uint8_t>& fdown);
uint8_t action_coin(const Action& a, const State& s);  // search.rs:249-270

}  // namespace wc
