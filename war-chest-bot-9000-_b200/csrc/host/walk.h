// Continual re-solving: a game that solves a depth-limited subgame at a
// decision, then walks the solved tree with the real game (acting on the CFR
// average, Bayes-filtering both beliefs on the public observations), and
// re-solves where the walk leaves the tree, carrying the beliefs the
// solve's per-iterate average strategies give at that exit into the next
// subgame's Phase 2. Restates engine/src/selfplay.rs:466-905 (finish_walk,
// Game::advance / resume) for two ReBeL seats, engine/src/serialize.rs:
// 209-330 (WalkTree: the part of the solved tree the walk reads) and
// engine/src/gpu/client.rs:20-92 (CarryStore::select and its f16 decode).
#pragma once
#include <cstdint>
#include <functional>
#include <memory>
#include <vector>

#include "roots.h"

namespace wc {

// The solved subgame's public tree as the walk reads it.
struct WalkTree {
    std::vector<uint8_t> kind, player, draw_steps;  // per node
    std::vector<uint32_t> soff;                     // nodes + 1: first strategy cell (reference order)
    std::vector<uint32_t> row_off, legal_off;       // node's config rows (node-local cell bounds)
    std::vector<uint32_t> act_off, na, obs_child;   // action -> public child index
    std::vector<uint32_t> child_off, nch, child;
    std::vector<uint32_t> sup;                      // per node: support ids of player 0, player 1
    std::vector<std::vector<Config>> supports;
    static std::shared_ptr<const WalkTree> from(const Tree& t);
    const std::vector<Config>& support(uint32_t node, int p) const { return supports[sup[2 * node + p]]; }
    uint32_t child_for_action(uint32_t node, uint32_t a) const { return child[child_off[node] + obs_child[act_off[node] + a]]; }
};

// The result of one solve as the walk consumes it: the average strategy in
// reference cell order, and the carry store (f16 exit beliefs per kept
// snapshot but the last, rows of [player 0 configs | player 1 configs] per
// exit node at carry_off[e]).
struct WalkResult {
    std::vector<float> strategy;
    std::vector<uint16_t> carries;
    uint32_t carry_snapshots = 0, carry_width = 0;
    std::vector<uint32_t> carry_off;   // nexit + 1
    std::vector<uint32_t> exit_nodes;  // reference node ids
    // A CPU solve's walk reads the exit beliefs off the solver instead
    // (Solver::carried_beliefs, search.rs:1937; selfplay.rs:480): per kept
    // snapshot but the last, [player 0 | player 1] in f32. Used when set.
    std::function<std::vector<std::vector<float>>(uint32_t node)> cpu_carried;
};

class Game {
public:
    enum Step { NEED_SOLVE = 1, ENDED = 2 };
    // A game from a seeded draft (make_game) or from a given root (state and
    // both beliefs); cfg is the subgame solve (depth, iterations, rule, node
    // cap); snapshots are always kept, since the walk carries them.
    Game(uint64_t seed, bool random_draft, const SolveCfg& cfg);
    Game(const Root& root, uint64_t seed, const SolveCfg& cfg);

    // Play until the next subgame must be solved (pending_tree() then holds
    // it, pending_roots() the roots Phase 2 values) or the game ends.
    Step advance();
    // Start the walk of the pending subgame with its solve's result.
    void resume(const WalkResult& r);
    // max_solves > 0: stop (ENDED) once that many subgames have been solved
    // and the walk of the last has left its tree.
    void set_max_solves(uint32_t n) { max_solves_ = n; }

    const Tree* pending_tree() const { return pending_.get(); }
    std::unique_ptr<Tree> take_pending_tree() { return std::move(pending_); }
    const std::vector<float>& pending_roots() const { return pending_roots_; }
    uint32_t pending_nroots() const { return pending_nroots_; }

    const State& state() const { return s_; }
    const Belief& belief(int p) const { return bel_[p]; }
    const Ctx& ctx() const { return ctx_; }
    // decisions, solves, capped solves (uniform fallback), walk decisions,
    // walk draws, ended, winner (-1 none), walking
    void counters(int64_t* out8) const;

private:
    void end_walk();
    Rng rng_;
    State s_;
    Ctx ctx_;
    Belief bel_[2];
    SolveCfg cfg_;
    std::vector<float> carried_;  // ncarried root pairs [p0 | p1]
    uint32_t ncarried_ = 0;
    // the walk
    std::shared_ptr<const WalkTree> tree_;
    std::shared_ptr<const WalkTree> pending_walk_;
    WalkResult res_;
    bool walking_ = false;
    uint32_t node_ = 0, drawn_ = 0;
    // the pending solve
    std::unique_ptr<Tree> pending_;
    std::vector<float> pending_roots_;
    uint32_t pending_nroots_ = 0;
    uint32_t max_solves_ = 0;
    int64_t decisions_ = 0, solves_ = 0, capped_ = 0, walk_decisions_ = 0, walk_draws_ = 0;
    bool stopped_ = false;
};

}  // namespace wc
