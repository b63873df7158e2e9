// TEST INFRASTRUCTURE (CPU only, never linked into the product library).
//
// The reference's public-belief-state tests, engine/tests/rebel_pbs.rs,
// restated over the host sources (rules, PBS, tree builder) and, where a test
// solves, the oracle's CPU solver. One function per reference test; each
// returns 0, or writes a message and returns nonzero. The file:line of the
// reference test is beside each.
#include <algorithm>
#include <array>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <utility>
#include <vector>

#include "../war-chest-bot-9000-_b200/csrc/host/roots.h"
#include "cfr_cpu.h"

using namespace wc;

namespace {

int failf(char* msg, size_t cap, const std::string& s) {
    if (msg && cap) std::snprintf(msg, cap, "%s", s.c_str());
    return 1;
}

std::string cfg_str(const Config& c) {
    char b[96];
    std::snprintf(b, sizeof b, "hand=[%d,%d,%d,%d,%d] fd=[%d,%d,%d,%d,%d] inflight=%d", c.hand[0], c.hand[1],
                  c.hand[2], c.hand[3], c.hand[4], c.fd[0], c.fd[1], c.fd[2], c.fd[3], c.fd[4], c.inflight);
    return b;
}

std::vector<Config> all_configs(const State& s, uint8_t p, const Ctx& ctx) {
    uint8_t res[NSLOT];
    reserve(s, p, ctx, res);
    const Config truth = true_config(s, p, ctx);
    return enumerate_configs(res, truth.hand_size(), truth.fd_size(), truth.inflight >= 0);
}

void random_apply(State& s, Rng& rng) {
    std::vector<Action> acts = s.legal_actions();
    s.apply_inplace(acts[rng.below(acts.size())]);
}

// rebel_pbs.rs:41-57: LayerNorms at the identity, everything else uniform in
// [-0.1, 0.1) from Rng(seed) (weights, then biases).
oracle::Net random_net(uint64_t seed) {
    oracle::Net n;
    Rng r(seed);
    n.w.resize(n.L.w_len);
    n.b.resize(n.L.b_len);
    for (float& x : n.w) x = ((float)r.unit_f64() - 0.5f) * 0.2f;
    for (float& x : n.b) x = ((float)r.unit_f64() - 0.5f) * 0.2f;
    n.ln.assign(n.L.ln_len, 0.0f);
    for (size_t i = 0; i < n.L.norm_g.size(); ++i)
        for (size_t k = n.L.norm_g[i]; k < n.L.norm_b[i]; ++k) n.ln[k] = 1.0f;
    n.empty = false;
    return n;
}

// rebel_pbs.rs:80-94: the private actions of config c with a uniform policy
// over its legal ones.
struct Row {
    std::vector<Action> acts;
    std::vector<int8_t> aslot;
    std::vector<uint8_t> fdown;
    std::vector<double> probs;
};
Row uniform_row(const State& s, const Ctx& ctx, uint8_t p, const Config& c) {
    Row r;
    node_actions(s, p, ctx, std::vector<Config>{c}, r.acts, r.aslot, r.fdown);
    size_t n = 0;
    for (int8_t k : r.aslot) n += action_legal(c, k) ? 1 : 0;
    for (int8_t k : r.aslot) r.probs.push_back(action_legal(c, k) && n > 0 ? 1.0 / (double)n : 0.0);
    return r;
}

// rebel_pbs.rs:99-115: the engine's own chance distribution.
std::vector<double> draw_weights(const State& s, uint8_t p, const std::vector<Action>& acts) {
    int bag_total = 0;
    for (int u = 0; u < N_UNITS; ++u) bag_total += s.zones[p][Z_BAG][u];
    std::vector<double> w;
    for (const Action& a : acts) {
        if (a.kind != K_DRAW || a.a == NONE) {
            w.push_back(0.0);
            continue;
        }
        const int u = a.a;
        w.push_back(bag_total > 0 ? (double)s.zones[p][Z_BAG][u]
                                  : (double)(s.zones[p][Z_FACEUP][u] + s.zones[p][Z_FACEDOWN][u]));
    }
    return w;
}

State world(const State& pubs, const Ctx& ctx, const Config& c0, const Config& c1) {
    State w = pubs;
    set_config(w, 0, ctx, c0);
    set_config(w, 1, ctx, c1);
    return w;
}

bool same_state(const State& a, const State& b) {
    if (std::memcmp(a.hex_type, b.hex_type, sizeof a.hex_type) || std::memcmp(a.hex_owner, b.hex_owner, sizeof a.hex_owner) ||
        std::memcmp(a.hex_height, b.hex_height, sizeof a.hex_height) ||
        std::memcmp(a.loc_marker, b.loc_marker, sizeof a.loc_marker) || std::memcmp(a.zones, b.zones, sizeof a.zones) ||
        std::memcmp(a.markers_hand, b.markers_hand, 2) || std::memcmp(a.turns_taken, b.turns_taken, 2))
        return false;
    if (a.initiative != b.initiative || a.initiative_moved != b.initiative_moved || a.round != b.round ||
        a.first_player != b.first_player || a.active != b.active || a.main_plays != b.main_plays ||
        a.winner != b.winner || a.adjudicated_draw != b.adjudicated_draw || !(a.pending == b.pending) ||
        a.conts.n != b.conts.n || a.wp_v2_triggered != b.wp_v2_triggered || a.interrupt != b.interrupt)
        return false;
    for (int i = 0; i < a.conts.n; ++i)
        if (!(a.conts.v[i] == b.conts.v[i])) return false;
    return true;
}

// Run body(seed) for every seed in [lo, hi) on the host's threads (the
// seeds are independent positions); the results are combined by the caller
// in seed order, so the outcome does not depend on the schedule.
template <class F>
void parallel_seeds(uint64_t lo, uint64_t hi, F&& body) {
    std::atomic<uint64_t> next{lo};
    const unsigned n = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    std::vector<std::thread> th;
    for (unsigned i = 0; i < n; ++i)
        th.emplace_back([&] {
            for (uint64_t s; (s = next.fetch_add(1)) < hi;) body(s);
        });
    for (auto& t : th) t.join();
}

const uint16_t DRAFT_POOL[19] = {1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 16, 17, 18, 19, 52, 53, 54};

// rebel_pbs.rs:118-163.
int leak_check(bool random_draft, int* checked, int* pending_seen, char* msg, size_t cap) {
    Rng rng(99);
    *checked = 0;
    *pending_seen = 0;
    std::vector<float> a(PUBFEAT), b(PUBFEAT);
    for (uint64_t g = 0; g < 12; ++g) {
        Rng gr(g + 1);
        State s = make_game(gr, random_draft);
        const Ctx ctx = Ctx::make(s);
        for (int step = 0; step < 150; ++step) {
            if (s.is_terminal()) break;
            for (uint8_t p = 0; p < 2; ++p) {
                std::vector<Config> all = all_configs(s, p, ctx);
                if (all.size() < 2) continue;
                State sa = s, sb = s;
                set_config(sa, p, ctx, all.front());
                write_public_features(sa, ctx, a.data());
                set_config(sb, p, ctx, all.back());
                write_public_features(sb, ctx, b.data());
                if (std::memcmp(a.data(), b.data(), 4 * a.size()) != 0)
                    return failf(msg, cap, "features changed when only player " + std::to_string(p) +
                                               "'s hidden config changed (game " + std::to_string(g) + ")");
                for (int h = 0; h < N_HEXES; ++h)
                    if (a[h * HEX_CH + 6] != 0.0f) {
                        ++*pending_seen;
                        break;
                    }
                ++*checked;
            }
            std::vector<Action> acts = s.legal_actions();
            if (acts.empty()) break;
            s.apply_inplace(acts[rng.below(acts.size())]);
        }
    }
    return 0;
}

using World = std::pair<uint64_t, uint64_t>;  // (config key of player 0, of player 1)

Config from_key(uint64_t k) {
    Config c;
    const uint64_t pend = k & 7u;
    c.inflight = pend == 0 ? (int8_t)-1 : (int8_t)(pend - 1);
    k >>= 3;
    for (int i = NSLOT - 1; i >= 0; --i) {
        c.fd[i] = (uint8_t)(k & 31u);
        k >>= 5;
    }
    for (int i = NSLOT - 1; i >= 0; --i) {
        c.hand[i] = (uint8_t)(k & 3u);
        k >>= 2;
    }
    return c;
}

// rebel_pbs.rs:362-416.
int compare(const std::map<World, double>& worlds, const Belief* bel, uint64_t seed, int step, const char* what,
            char* msg, size_t cap) {
    for (int p = 0; p < 2; ++p) {
        std::map<uint64_t, double> exact;
        double tot = 0.0;
        for (const auto& kv : worlds) {
            exact[p == 0 ? kv.first.first : kv.first.second] += kv.second;
            tot += kv.second;
        }
        for (auto& kv : exact) kv.second /= tot;
        const Belief& b = bel[p];
        for (const auto& kv : exact) {
            if (kv.second < 1e-9) continue;
            const int i = b.index_of(from_key(kv.first));
            const double got = i >= 0 ? (double)b.p[i] : 0.0;
            if (std::fabs(got - kv.second) >= 1e-5) {
                char m[256];
                std::snprintf(m, sizeof m, "seed %llu step %d (%s) player %d: config %s exact %.9f tracker %.9f",
                              (unsigned long long)seed, step, what, p, cfg_str(from_key(kv.first)).c_str(), kv.second,
                              got);
                return failf(msg, cap, m);
            }
        }
        for (size_t i = 0; i < b.cfg.size(); ++i) {
            if (b.p[i] < 1e-9f) continue;
            auto it = exact.find(b.cfg[i].key());
            const double w = it == exact.end() ? 0.0 : it->second;
            if (std::fabs((double)b.p[i] - w) >= 1e-5)
                return failf(msg, cap, "seed " + std::to_string(seed) + " step " + std::to_string(step) +
                                           ": tracker has a phantom config " + cfg_str(b.cfg[i]));
        }
    }
    return 0;
}

// rebel_pbs.rs:222-360.
int run_one_draft(uint64_t seed, const uint16_t* white, const uint16_t* black, int* steps_out, char* msg, size_t cap) {
    Rng rng(seed + 1);
    State s = State::from_draft(white, black, WHITE);
    const Ctx ctx = Ctx::make(s);
    Belief bel[2] = {Belief::point(Config()), Belief::point(Config())};
    std::map<World, double> worlds;
    worlds[{Config().key(), Config().key()}] = 1.0;
    int steps = 0;
    while (!s.is_terminal() && steps < 60 && worlds.size() < 20000) {
        const uint8_t p = s.to_act();
        if (s.is_chance()) {
            std::map<World, double> next;
            for (const auto& kv : worlds) {
                const Config c0 = from_key(kv.first.first), c1 = from_key(kv.first.second);
                State ws = world(s, ctx, c0, c1);
                std::vector<Action> acts = ws.legal_actions();
                std::vector<double> wts = draw_weights(ws, p, acts);
                double tot = 0.0;
                for (double x : wts) tot += x;
                if (!(tot > 0.0)) return failf(msg, cap, "a world had nothing to draw");
                for (size_t i = 0; i < acts.size(); ++i) {
                    if (wts[i] <= 0.0) continue;
                    State nx = ws;
                    nx.apply_inplace(acts[i]);
                    const uint64_t nk = true_config(nx, p, ctx).key();
                    World nc = p == 0 ? World{nk, kv.first.second} : World{kv.first.first, nk};
                    next[nc] += kv.second * wts[i] / tot;
                }
            }
            worlds.swap(next);
            uint8_t res[NSLOT], fu[NSLOT];
            reserve(s, p, ctx, res);
            faceup_counts(s, p, ctx, fu);
            const bool wp = s.pending.kind == C_WPDRAW;
            bel[p] = belief_after_draw(bel[p], res, fu, wp);
            std::vector<Action> acts = s.legal_actions();
            std::vector<double> wts = draw_weights(s, p, acts);
            s.apply_inplace(acts[rng.weighted_index(wts.data(), wts.size())]);
            if (compare(worlds, bel, seed, steps, "draw", msg, cap)) return 1;
            ++steps;
            continue;
        }
        // decision node: sample the real action from the announced policy
        const Config truth = true_config(s, p, ctx);
        Row row = uniform_row(s, ctx, p, truth);
        const size_t chosen = rng.weighted_index(row.probs.data(), row.probs.size());
        const uint32_t obs = obs_key(row.acts[chosen]);
        // brute force over the worlds
        std::map<World, double> next;
        for (const auto& kv : worlds) {
            const Config c0 = from_key(kv.first.first), c1 = from_key(kv.first.second);
            State ws = world(s, ctx, c0, c1);
            Row wr = uniform_row(ws, ctx, p, p == 0 ? c0 : c1);
            for (size_t i = 0; i < wr.acts.size(); ++i) {
                if (wr.probs[i] <= 0.0 || obs_key(wr.acts[i]) != obs) continue;
                State nx = ws;
                nx.apply_inplace(wr.acts[i]);
                const uint64_t nk = true_config(nx, p, ctx).key();
                World nc = p == 0 ? World{nk, kv.first.second} : World{kv.first.first, nk};
                next[nc] += kv.second * wr.probs[i];
            }
        }
        double tot = 0.0;
        for (const auto& kv : next) tot += kv.second;
        if (!(tot > 0.0)) return failf(msg, cap, "brute force lost every world at step " + std::to_string(steps));
        for (auto& kv : next) kv.second /= tot;
        worlds.swap(next);
        // the tracker: the same update, incrementally over configs
        const std::vector<Config> cfgs = bel[p].cfg;
        std::vector<std::pair<Config, float>> pairs;
        for (size_t ci = 0; ci < cfgs.size(); ++ci) {
            Row cr = uniform_row(s, ctx, p, cfgs[ci]);
            for (size_t i = 0; i < cr.acts.size(); ++i) {
                if (cr.probs[i] <= 0.0 || obs_key(cr.acts[i]) != obs) continue;
                Config n;
                if (advance_config(cfgs[ci], cr.aslot[i], cr.fdown[i] != 0, &n))
                    pairs.emplace_back(n, bel[p].p[ci] * (float)cr.probs[i]);
            }
        }
        bel[p] = Belief::from_pairs(std::move(pairs));
        s.apply_inplace(row.acts[chosen]);
        if (compare(worlds, bel, seed, steps, "decision", msg, cap)) return 1;
        ++steps;
    }
    *steps_out = steps;
    if (steps <= 8)
        return failf(msg, cap, "seed " + std::to_string(seed) + " produced too short a trace (" +
                                   std::to_string(steps) + " steps)");
    return 0;
}

// rebel_pbs.rs:712-764.
bool position_with_ambiguous_facedown(uint64_t seed, State* out, Ctx* ctx_out, Belief* bel) {
    Rng rng(seed);
    Rng gr(seed);
    State s = make_game(gr, false);
    const size_t n = 40 + rng.below(60);
    for (size_t i = 0; i < n; ++i) {
        if (s.is_terminal()) return false;
        std::vector<Action> acts = s.legal_actions();
        if (acts.empty()) return false;
        s.apply_inplace(acts[rng.below(acts.size())]);
    }
    while (!s.is_terminal() && s.is_chance()) random_apply(s, rng);
    if (s.is_terminal() || s.is_chance() || s.pending.kind != C_MAINPLAY) return false;
    const Ctx ctx = Ctx::make(s);
    for (uint8_t p = 0; p < 2; ++p) {
        bel[p] = uniform_belief(s, ctx, p);
        if (bel[p].cfg.empty()) return false;
    }
    const uint8_t me = s.to_act();
    std::map<uint64_t, int> hands;
    bool shared = false;
    for (const Config& c : bel[me].cfg) {
        uint64_t k = 0;
        for (int i = 0; i < NSLOT; ++i) k = (k << 8) | c.hand[i];
        shared = shared || ++hands[k] > 1;
    }
    if (!shared) return false;
    *out = s;
    *ctx_out = ctx;
    return true;
}

// The root row of config c in the latest average (Solver::average_strategy(0, c)).
std::vector<float> root_row(const oracle::Solver& sv, const Tree& t, size_t c) {
    const NodeRec& n0 = t.nodes[0];
    const uint32_t lo = t.soff[0] + t.legal_off[n0.row_off + c], hi = t.soff[0] + t.legal_off[n0.row_off + c + 1];
    const std::vector<float>& avg = sv.average();
    return std::vector<float>(avg.begin() + lo, avg.begin() + hi);
}

}  // namespace

extern "C" {

// rebel_pbs.rs:165-169 and 171-182 (random draft: the pending mask must fire).
int oracle_check_features_do_not_leak(int random_draft, int* stats2, char* msg, size_t cap) {
    int checked = 0, pending = 0;
    if (leak_check(random_draft != 0, &checked, &pending, msg, cap)) return 1;
    stats2[0] = checked;
    stats2[1] = pending;
    if (checked <= 500) return failf(msg, cap, "not enough positions exercised: " + std::to_string(checked));
    if (random_draft && pending == 0) return failf(msg, cap, "the pending-maneuver mask never fired");
    return 0;
}

// rebel_pbs.rs:198-220: the starter matchup, seeds 0..6; with_priests: the
// Warrior Priest draft, seeds 100..104.
int oracle_check_belief_tracker(int with_priests, int* steps_total, char* msg, size_t cap) {
    const uint16_t w0[4] = {17, 12, 4, 9}, b0[4] = {1, 3, 8, 16};
    const uint16_t w1[4] = {18, 17, 12, 4}, b1[4] = {54, 1, 3, 8};
    *steps_total = 0;
    const int n = with_priests ? 4 : 6;
    for (int i = 0; i < n; ++i) {
        int steps = 0;
        const uint64_t seed = with_priests ? 100 + (uint64_t)i : (uint64_t)i;
        if (run_one_draft(seed, with_priests ? w1 : w0, with_priests ? b1 : b0, &steps, msg, cap)) return 1;
        *steps_total += steps;
    }
    return 0;
}

// rebel_pbs.rs:418-459 (IDX_BITS = 24, rebel.rs:543).
int oracle_check_config_key_headroom(char* msg, size_t cap) {
    const int IDX_BITS = 24;
    for (uint64_t seed = 0; seed < 200; ++seed) {
        Rng r((seed * 0x9E3779B9ull) | 1);
        Config c;
        for (int k = 0; k < NSLOT; ++k) {
            c.hand[k] = (uint8_t)r.below(4);
            c.fd[k] = (uint8_t)r.below(6);
        }
        c.inflight = (r.next_u64() & 1) == 0 ? (int8_t)-1 : (int8_t)r.below(NSLOT);
        if (c.key() >= (1ull << (64 - IDX_BITS))) return failf(msg, cap, "config key leaves no room for the index");
        Config d = c;
        if (c.key() != d.key()) return failf(msg, cap, "equal configs, different keys");
        d.inflight = c.inflight < 0 ? 0 : (c.inflight + 1 < NSLOT ? (int8_t)(c.inflight + 1) : (int8_t)-1);
        if (c.inflight != d.inflight && c.key() == d.key()) return failf(msg, cap, "pending not in the key");
    }
    Config c;
    for (int k = 0; k < NSLOT; ++k) {
        c.hand[k] = 3;
        c.fd[k] = 5;
    }
    c.inflight = NSLOT - 1;
    if (c.key() >= (1ull << (64 - IDX_BITS))) return failf(msg, cap, "the extreme config overflows");
    return 0;
}

// rebel_pbs.rs:464-497: reported, not asserted (median, mean x 10, p99, positions).
int oracle_check_config_census(uint64_t* out4) {
    std::vector<size_t> sizes;
    Rng rng(0xC0FFEE);
    for (int g = 0; g < 200; ++g) {
        State s = make_game(rng, true);
        const Ctx ctx = Ctx::make(s);
        for (int step = 0; step < 300; ++step) {
            if (s.is_terminal()) break;
            for (uint8_t p = 0; p < 2; ++p) sizes.push_back(all_configs(s, p, ctx).size());
            random_apply(s, rng);
        }
    }
    std::sort(sizes.begin(), sizes.end());
    const size_t n = sizes.size();
    double mean = 0.0;
    for (size_t x : sizes) mean += (double)x;
    out4[0] = sizes[n / 2];
    out4[1] = (uint64_t)(10.0 * mean / (double)n);
    out4[2] = sizes[(size_t)((double)n * 0.99)];
    out4[3] = n;
    return 0;
}

// rebel_pbs.rs:501-545: write_root / read_root round trip of state, beliefs
// and every continuation, at every MainPlay along 30 random games.
int oracle_check_roots_round_trip(int* checked, char* msg, size_t cap) {
    *checked = 0;
    for (uint64_t seed = 0; seed < 30; ++seed) {
        Rng rng((seed * 0x9E3779B9ull) | 1);
        Root r;
        r.s = make_game(rng, true);
        r.ctx = Ctx::make(r.s);
        r.bel[0] = Belief::point(Config());
        r.bel[1] = Belief::point(Config());
        for (int step = 0; step < 40; ++step) {
            if (r.s.is_terminal()) break;
            if (r.s.pending.kind == C_MAINPLAY) {
                std::vector<uint8_t> bytes = root_to_bytes(r);
                Root back;
                if (!root_from_bytes(bytes.data(), bytes.size(), &back))
                    return failf(msg, cap, "seed " + std::to_string(seed) + ": the root did not parse back");
                if (!same_state(r.s, back.s)) return failf(msg, cap, "seed " + std::to_string(seed) + ": state did not round trip");
                for (int p = 0; p < 2; ++p)
                    if (r.bel[p].cfg.size() != back.bel[p].cfg.size() ||
                        !std::equal(r.bel[p].cfg.begin(), r.bel[p].cfg.end(), back.bel[p].cfg.begin()) ||
                        r.bel[p].p != back.bel[p].p)
                        return failf(msg, cap, "seed " + std::to_string(seed) + ": belief did not round trip");
                ++*checked;
            }
            random_apply(r.s, rng);
            const uint8_t p = r.s.to_act();
            if (r.s.is_chance()) {
                uint8_t res[NSLOT], fu[NSLOT];
                reserve(r.s, p, r.ctx, res);
                faceup_counts(r.s, p, r.ctx, fu);
                r.bel[p] = belief_after_draw(r.bel[p], res, fu, r.s.pending.kind == C_WPDRAW);
            } else {
                r.bel[p] = Belief::point(true_config(r.s, p, r.ctx));
            }
        }
    }
    return 0;
}

// rebel_pbs.rs:551-578, for the row format this build packs (the compact
// GPU row, rebel.rs:1274-1346): the packed row, expanded with the seat-0
// coin-type ids, gives the features of the live state at every MainPlay.
int oracle_check_packed_row_expands(int* checked, char* msg, size_t cap) {
    *checked = 0;
    std::vector<float> direct(PUBFEAT), expanded(PUBFEAT);
    for (uint64_t seed = 0; seed < 40; ++seed) {
        Rng rng((seed * 0x9E3779B9ull) | 1);
        State s = make_game(rng, true);
        const Ctx ctx = Ctx::make(s);
        int here = 0;
        for (int step = 0; step < 120; ++step) {
            if (s.is_terminal()) break;
            if (s.pending.kind == C_MAINPLAY) {
                uint8_t row[GPU_ROW_BYTES], ids[NTYPE];
                pack_gpu_row(s, ctx, row);
                for (int ty = 0; ty < NTYPE; ++ty) ids[ty] = ctx.slots[ty / NSLOT][ty % NSLOT];
                write_public_features(s, ctx, direct.data());
                expand_gpu_row(row, ids, expanded.data());
                if (std::memcmp(direct.data(), expanded.data(), 4 * PUBFEAT) != 0)
                    return failf(msg, cap, "seed " + std::to_string(seed) + ": packed row and live state encode differently");
                ++here;
            }
            random_apply(s, rng);
        }
        if (here <= 20) return failf(msg, cap, "seed " + std::to_string(seed) + " exercised too few MainPlay states");
        *checked += here;
    }
    return 0;
}

// rebel_pbs.rs:586-614 (write_config_feats, rebel.rs:194-201: counts / CNORM).
int oracle_check_config_features_separate(int* checked, char* msg, size_t cap) {
    *checked = 0;
    std::map<std::vector<uint32_t>, uint64_t> seen;
    for (uint64_t seed = 0; seed < 300; ++seed) {
        Rng r((seed * 0x9E3779B9ull) | 1);
        uint8_t res[NSLOT];
        for (int k = 0; k < NSLOT; ++k) res[k] = (uint8_t)r.below(6);
        for (uint8_t hs = 0; hs <= HAND_CAP; ++hs)
            for (uint8_t fs = 0; fs < 4; ++fs) {
                std::vector<Config> cfgs = enumerate_configs(res, hs, fs, false);
                seen.clear();
                for (const Config& c : cfgs)
                    for (int p = 0; p < 2; ++p) {
                        uint8_t cnt[CCOUNTS];
                        config_counts(c, res, cnt);
                        std::vector<uint32_t> key(CFEAT);
                        for (int k = 0; k < CFEAT; ++k) {
                            const float x = (float)cnt[k] / CNORM;
                            std::memcpy(&key[k], &x, 4);
                        }
                        auto ins = seen.emplace(key, c.key());
                        if (!ins.second && ins.first->second != c.key())
                            return failf(msg, cap, "two configs share a feature vector");
                        ++*checked;
                    }
            }
    }
    if (*checked <= 10000) return failf(msg, cap, "only " + std::to_string(*checked) + " config vectors exercised");
    return 0;
}

// rebel_pbs.rs:640-686.
int oracle_check_terminal_leaf_subgame(int* checked, char* msg, size_t cap) {
    const oracle::Net net = random_net(5);
    *checked = 0;
    for (uint64_t seed = 0; seed < 600; ++seed) {
        Rng rng((seed * 0x9E3779B9ull) | 1);
        State s = make_game(rng, false);
        for (uint64_t i = 0; i < 60 + seed % 100; ++i) {
            if (s.is_terminal()) break;
            random_apply(s, rng);
        }
        if (s.is_terminal() || s.is_chance()) continue;
        s.main_plays = MAX_MAIN_PLAYS - 1;  // one coin play from the horizon
        const Ctx ctx = Ctx::make(s);
        const Belief bel[2] = {uniform_belief(s, ctx, 0), uniform_belief(s, ctx, 1)};
        SolveCfg cfg;
        cfg.depth = 2;
        cfg.iters = 8;
        cfg.snapshots = true;
        auto t = build_tree(s, ctx, cfg, bel);
        for (const NodeRec& n : t->nodes)
            if (n.kind == NK_LEAF && !n.terminal) return failf(msg, cap, "expected every leaf terminal");
        oracle::Solver sv(*t, &net);
        sv.multistep(cfg.iters);
        std::vector<float> root(bel[0].p);
        root.insert(root.end(), bel[1].p.begin(), bel[1].p.end());
        auto v = sv.value_under({root});
        for (float x : v[0])
            if (!std::isfinite(x)) return failf(msg, cap, "a root value is not finite");
        if (++*checked >= 3) break;
    }
    if (*checked < 3) return failf(msg, cap, "only " + std::to_string(*checked) + " positions exercised");
    return 0;
}

// rebel_pbs.rs:697-727 (DRAFT_POOL, selfplay.rs; the Royal Coin with it).
int oracle_check_card_features_separate(char* msg, size_t cap) {
    std::map<std::vector<uint32_t>, int> seen;
    std::vector<int> units;
    for (uint16_t id : DRAFT_POOL) units.push_back(index_of_id(id));
    units.push_back(ROYAL_COIN);
    for (int u : units)
        if (u < 0) return failf(msg, cap, "the draft pool did not resolve to unit indices");
    if (units.size() != 20) return failf(msg, cap, "expected 20 units");
    for (int u : units) {
        float f[CARD_FEATS];
        write_card_features((uint8_t)u, f);
        std::vector<uint32_t> key(CARD_FEATS);
        std::memcpy(key.data(), f, sizeof f);
        auto ins = seen.emplace(key, u);
        if (!ins.second && ins.first->second != u)
            return failf(msg, cap, "units " + std::to_string(ins.first->second) + " and " + std::to_string(u) +
                                       " share a card vector");
    }
    return 0;
}

// rebel_pbs.rs:732-751.
int oracle_check_config_counts(char* msg, size_t cap) {
    const uint8_t res[NSLOT] = {4, 3, 5, 2, 1};
    Config c;
    const uint8_t hand[NSLOT] = {1, 0, 2, 0, 0}, fd[NSLOT] = {2, 1, 0, 0, 1}, bag[NSLOT] = {1, 2, 3, 2, 0};
    std::memcpy(c.hand, hand, NSLOT);
    std::memcpy(c.fd, fd, NSLOT);
    uint8_t cnt[CCOUNTS];
    config_counts(c, res, cnt);
    if (std::memcmp(cnt, hand, NSLOT)) return failf(msg, cap, "hand block");
    if (std::memcmp(cnt + NSLOT, fd, NSLOT)) return failf(msg, cap, "face-down block");
    if (std::memcmp(cnt + 2 * NSLOT, bag, NSLOT)) return failf(msg, cap, "bag block");
    return 0;
}

// rebel_pbs.rs:771-821: the same public position in two worlds (each
// player's first or last config set as the truth) solves bit-identically.
int oracle_check_solve_reads_only_beliefs(int* checked, char* msg, size_t cap) {
    const oracle::Net net = random_net(0xA11CE);
    SolveCfg cfg;
    cfg.depth = 2;
    cfg.iters = 8;
    cfg.snapshots = true;
    // per seed: -1 no ambiguous position, 0 agreed, 1 values moved, 2 strategy moved
    std::vector<int> outcome(80, -1);
    parallel_seeds(1, 80, [&](uint64_t seed) {
        State s;
        Ctx ctx;
        Belief bel[2];
        if (!position_with_ambiguous_facedown(seed, &s, &ctx, bel)) return;
        std::vector<std::vector<float>> runs[2];
        for (int pick = 0; pick < 2; ++pick) {
            State w = s;
            for (int p = 0; p < 2; ++p) set_config(w, (uint8_t)p, ctx, pick == 0 ? bel[p].cfg.front() : bel[p].cfg.back());
            auto t = build_tree(w, ctx, cfg, bel);
            oracle::Solver sv(*t, &net);
            sv.multistep(cfg.iters);
            std::vector<float> root(bel[0].p);
            root.insert(root.end(), bel[1].p.begin(), bel[1].p.end());
            auto v = sv.value_under({root});
            std::vector<float> strat;
            for (size_t c = 0; c < bel[w.to_act()].cfg.size(); ++c) {
                std::vector<float> r = root_row(sv, *t, c);
                strat.insert(strat.end(), r.begin(), r.end());
            }
            runs[pick] = {v[0], strat};
        }
        outcome[seed] = runs[0][0] != runs[1][0] ? 1 : runs[0][1] != runs[1][1] ? 2 : 0;
    });
    *checked = 0;
    for (uint64_t seed = 1; seed < 80; ++seed) {
        if (outcome[seed] == 1) return failf(msg, cap, "root values moved with the true world (seed " + std::to_string(seed) + ")");
        if (outcome[seed] == 2) return failf(msg, cap, "the root strategy moved with the true world (seed " + std::to_string(seed) + ")");
        if (outcome[seed] == 0) ++*checked;
    }
    if (*checked <= 20) return failf(msg, cap, "only " + std::to_string(*checked) + " positions exercised");
    return 0;
}

// The two worlds of rebel_pbs.rs:791-797 for one seed, as root bytes (the
// same beliefs, different true configs), so a test can build the product's
// jobs from both: 0 if the seed gives an ambiguous position.
int oracle_ambiguous_worlds(uint64_t seed, uint8_t* buf0, uint8_t* buf1, size_t cap, size_t* len0, size_t* len1) {
    State s;
    Ctx ctx;
    Belief bel[2];
    if (!position_with_ambiguous_facedown(seed, &s, &ctx, bel)) return 1;
    for (int pick = 0; pick < 2; ++pick) {
        Root r;
        r.s = s;
        for (int p = 0; p < 2; ++p) set_config(r.s, (uint8_t)p, ctx, pick == 0 ? bel[p].cfg.front() : bel[p].cfg.back());
        r.ctx = ctx;
        r.bel[0] = bel[0];
        r.bel[1] = bel[1];
        std::vector<uint8_t> b = root_to_bytes(r);
        if (b.size() > cap) return 2;
        std::memcpy(pick == 0 ? buf0 : buf1, b.data(), b.size());
        *(pick == 0 ? len0 : len1) = b.size();
    }
    return 0;
}

// rebel_pbs.rs:831-892 (stats: positions, values that differ, strategies that differ).
int oracle_check_value_separates_configs(int* stats3, char* msg, size_t cap) {
    const oracle::Net net = random_net(0xBEEF);
    SolveCfg cfg;
    cfg.depth = 2;
    cfg.iters = 8;
    cfg.snapshots = true;
    std::vector<std::array<int, 3>> per(80, {0, 0, 0});  // per seed: pairs, values differ, strategies differ
    parallel_seeds(1, 80, [&](uint64_t seed) {
        State s;
        Ctx ctx;
        Belief bel[2];
        if (!position_with_ambiguous_facedown(seed, &s, &ctx, bel)) return;
        const uint8_t me = s.to_act();
        auto t = build_tree(s, ctx, cfg, bel);
        oracle::Solver sv(*t, &net);
        sv.multistep(cfg.iters);
        std::vector<float> root(bel[0].p);
        root.insert(root.end(), bel[1].p.begin(), bel[1].p.end());
        auto vals = sv.value_under({root});
        const float* v = vals[0].data() + (me == 0 ? 0 : bel[0].cfg.size());
        std::array<int, 3>& st = per[seed];
        for (size_t i = 0; i < bel[me].cfg.size(); ++i)
            for (size_t j = 0; j < i; ++j) {
                if (std::memcmp(bel[me].cfg[i].hand, bel[me].cfg[j].hand, NSLOT) != 0) continue;
                ++st[0];
                if (std::fabs(v[i] - v[j]) > 1e-9f) ++st[1];
                std::vector<float> a = root_row(sv, *t, i), b = root_row(sv, *t, j);
                bool d = false;
                for (size_t k = 0; k < a.size() && k < b.size(); ++k) d = d || std::fabs(a[k] - b[k]) > 1e-9f;
                if (d) ++st[2];
            }
    });
    int positions = 0, val_differs = 0, strat_differs = 0;
    for (const auto& st : per) {
        positions += st[0];
        val_differs += st[1];
        strat_differs += st[2];
    }
    stats3[0] = positions;
    stats3[1] = val_differs;
    stats3[2] = strat_differs;
    if (positions <= 50) return failf(msg, cap, "only " + std::to_string(positions) + " same-hand pairs found");
    if ((double)val_differs / positions <= 0.9) return failf(msg, cap, "too few same-hand pairs got distinct values");
    if ((double)strat_differs / positions <= 0.5) return failf(msg, cap, "too few same-hand pairs got distinct play");
    return 0;
}

// rebel_pbs.rs:898-927.
int oracle_check_normalized_weights(int* checked, char* msg, size_t cap) {
    Rng rng(0xB33F);
    *checked = 0;
    for (uint64_t seed = 0; seed < 400; ++seed) {
        Rng r(seed * 0x9E3779B9ull);
        uint8_t res[NSLOT];
        for (int k = 0; k < NSLOT; ++k) res[k] = (uint8_t)r.below(6);
        const uint8_t hs = (uint8_t)r.below(4), fs = (uint8_t)r.below(4);
        std::vector<Config> cfgs = enumerate_configs(res, hs, fs, false);
        if (cfgs.empty()) continue;
        std::vector<float> w(cfgs.size(), 0.0f);
        if (seed % 17 != 0)
            for (float& x : w) x = (float)rng.unit_f64();
        std::vector<float> got(cfgs.size());
        normalize_weights(w.data(), w.size(), got.data());
        Belief b;
        b.cfg = cfgs;
        b.p = w;
        b.normalize();
        for (size_t i = 0; i < got.size(); ++i)
            if (std::fabs(got[i] - b.p[i]) >= 2e-7f) return failf(msg, cap, "normalize_weights differs from Belief::normalize");
        ++*checked;
    }
    if (*checked <= 100) return failf(msg, cap, "only " + std::to_string(*checked) + " weight vectors exercised");
    return 0;
}

// rebel_pbs.rs:929-958.
int oracle_check_from_pairs_keeps_zero_weight(char* msg, size_t cap) {
    Config a, b, c;
    b.hand[0] = 1;
    c.fd[0] = 1;
    Belief bel = Belief::from_pairs({{b, 0.25f}, {c, -0.5f}, {a, 0.0f}});
    if (bel.cfg.size() != 2 || !(bel.cfg[0] == a) || !(bel.cfg[1] == b))
        return failf(msg, cap, "zero-weight config must stay in the support");
    if (bel.p[0] != 0.0f) return failf(msg, cap, "the kept config's weight stays exactly zero");
    if (bel.p[1] != 1.0f) return failf(msg, cap, "kept configs are renormalized");
    return 0;
}

// rebel_pbs.rs:960-1105.
int oracle_check_zero_weight_walk_update(char* msg, size_t cap) {
    const oracle::Net empty;  // no network: every non-terminal leaf is valued 0
    Rng rng(777);
    for (int game = 0; game < 200; ++game) {
        State s = make_game(rng, false);
        const size_t n = 40 + rng.below(60);
        for (size_t i = 0; i < n; ++i) {
            if (s.is_terminal()) break;
            std::vector<Action> acts = s.legal_actions();
            if (acts.empty()) break;
            s.apply_inplace(acts[rng.below(acts.size())]);
        }
        while (!s.is_terminal() && s.is_chance()) random_apply(s, rng);
        if (s.is_terminal() || s.is_chance() || s.pending.kind != C_MAINPLAY) continue;
        const Ctx ctx = Ctx::make(s);
        const uint8_t me = s.to_act();
        Belief bel[2];
        bool ok = true;
        for (uint8_t p = 0; p < 2 && ok; ++p) {
            bel[p] = uniform_belief(s, ctx, p);
            ok = bel[p].cfg.size() >= 2;
        }
        if (!ok) continue;
        bel[me].p[0] = (float)1e-46;  // every product with a probability underflows to 0
        bel[me].normalize();
        SolveCfg cfg;
        cfg.depth = 2;
        cfg.iters = 8;
        cfg.snapshots = false;
        auto t = build_tree(s, ctx, cfg, bel);
        oracle::Solver sv(*t, &empty);
        sv.multistep(8);
        const NodeRec& n0 = t->nodes[0];
        const uint32_t lo1 = t->legal_off[n0.row_off + 1], hi1 = t->legal_off[n0.row_off + 2];
        if (lo1 == hi1) continue;
        const uint32_t chosen = t->legal_action[t->soff[0] + lo1];
        const uint32_t child = t->child[n0.child_off + t->obs_child[n0.act_off + chosen]];
        if (t->nodes[child].kind == NK_CHANCE) continue;
        const uint32_t obs = obs_key(t->acts[n0.act_off + chosen]);
        std::vector<std::pair<Config, float>> pairs;
        for (size_t ci = 0; ci < bel[me].cfg.size(); ++ci) {
            std::vector<float> row = root_row(sv, *t, ci);
            const uint32_t lo = t->legal_off[n0.row_off + ci];
            for (size_t k = 0; k < row.size(); ++k) {
                const uint32_t a = t->legal_action[t->soff[0] + lo + k];
                if (obs_key(t->acts[n0.act_off + a]) != obs) continue;
                Config nx;
                if (advance_config(bel[me].cfg[ci], t->aslot[n0.act_off + a], t->fdown[n0.act_off + a] != 0, &nx))
                    pairs.emplace_back(nx, bel[me].p[ci] * row[k]);
            }
        }
        const Belief nb = Belief::from_pairs(std::move(pairs));
        const std::vector<Config>& kids = t->supports[t->nodes[child].sup[me]];
        if (kids.size() != nb.cfg.size() || !std::equal(kids.begin(), kids.end(), nb.cfg.begin()))
            return failf(msg, cap, "walk update dropped a reachable config (weight underflow)");
        return 0;
    }
    return failf(msg, cap, "no usable position in 200 random games");
}

}  // extern "C"
