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

// Serialized root in the reference's format v3 (engine/src/roots.rs:247-313):
// the State field by field, little-endian (write_state), then per player
// u32 n, n configs (hand[5], fd[5], inflight or 0xff), n f32 weights.
// root_from_bytes fails on malformed or truncated input; with `used` it
// accepts trailing bytes and reports how many the root took, without it the
// root must fill the buffer exactly.
std::vector<uint8_t> root_to_bytes(const Root& r);
bool root_from_bytes(const uint8_t* data, size_t n, Root* out, size_t* used = nullptr);
void write_state(std::vector<uint8_t>& out, const State& s);
// read_state refuses a state whose fields would index out of range.
bool state_in_range(const State& s);
// The action names in-range fields and units on its source hexes, so apply
// indexes nothing out of range (legality aside).
bool action_well_formed(const State& s, const Action& a);
bool read_state(const uint8_t* data, size_t n, size_t* at, State* out);

// A roots file (write_roots, roots.rs:323-333): magic, version 3, count, then
// the roots back to back. Fills (offset, length) per root; false on a bad
// magic or version, or a malformed root.
constexpr uint32_t ROOTS_MAGIC = 0x57107207u, ROOTS_VERSION = 3;
bool roots_file_split(const uint8_t* data, size_t n, std::vector<std::pair<size_t, size_t>>* spans);

}  // namespace wc
