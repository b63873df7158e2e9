// Seeded subgame roots: a game from a seeded draft, played forward by uniform
// random play with the exact Bayes belief filter, stopped at a MainPlay solve
// site. Restates engine/src/selfplay.rs:59-81 (make_game), :588-905 (the
// game loop's chance and decision handling), :1124-1156 (resolve_chance),
// and engine/src/policy.rs:41-139 (NodePolicy frame/sample/posterior,
// uniform).
#pragma once
#include <cstdint>
#include <vector>

#include "tree.h"

namespace wc {

struct Root {
    State s;
    Ctx ctx;
    Belief bel[2];
};

State make_game(Rng& rng, bool random_draft);

// A decision node's per-config policy over its private actions.
struct NodePolicy {
    std::vector<Action> acts;
    std::vector<int8_t> aslot;
    std::vector<uint8_t> fdown;
    std::vector<uint32_t> legal_off, legal_action;
    std::vector<float> probs;
    static NodePolicy frame(const State& s, const Ctx& ctx, uint8_t player, const std::vector<Config>& cfgs);
    static NodePolicy uniform(const State& s, const Ctx& ctx, uint8_t player, const std::vector<Config>& cfgs);
    size_t sample(Rng& rng, size_t c) const;
    Belief posterior(const Belief& prior, uint32_t obs) const;
};

void resolve_chance(State& s, uint8_t player, Rng& rng);

// Play `plies` uniform decisions from a seeded game, then on to the next
// MainPlay decision. Returns false if the game ended first.
bool make_root(uint64_t seed, int plies, bool random_draft, Root* out);

// A uniform belief over every config consistent with the public counts
// (tests/rebel_solver.rs:50-64).
Belief uniform_belief(const State& s, const Ctx& ctx, uint8_t p);

// A belief-heavy root: make_root's position, then each player's belief
// replaced by up to `ncfg` configs drawn (seeded, without replacement) from
// every config consistent with the public counts (enumerate_configs,
// rebel.rs:270), the true config always among them, with Dirichlet(1)
// weights (normalised unit exponentials). Returns false if the game ended
// before the root.
bool make_wide_root(uint64_t seed, int plies, bool random_draft, uint32_t ncfg, Root* out);

// Serialized root: the State bytes, then per player u32 n, n configs
// (hand[5], fd[5], inflight i8), n f32 weights.
std::vector<uint8_t> root_to_bytes(const Root& r);
bool root_from_bytes(const uint8_t* data, size_t n, Root* out);

}  // namespace wc
