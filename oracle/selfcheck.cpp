// TEST INFRASTRUCTURE (CPU only, never linked into the product library).
//
// Known-answer and invariant checks of the host rules / PBS code, restating
// the reference engine's own tests so the shared host sources (and with them
// the oracle) are pinned to the reference's behaviour:
//   engine/tests/invariants.rs   random playouts: coin conservation, board
//                                structure, markers, hand cap, in-flight coin,
//                                winner and horizon payoff (:46-171); random
//                                drafts are disjoint (:182-205); the board
//                                tables (:211-241)
//   engine/tests/scenarios.rs:923 action encode / decode round trip (here over
//                                every legal action the playouts meet)
//   engine/src/rebel.rs:1401-1583 DrawScratch::run against the per-draw
//                                composition (hand-built cases and a fuzz)
// Each check returns 0 or writes a message and returns nonzero.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../war-chest-bot-9000-_b200/csrc/host/pbs.h"
#include "../war-chest-bot-9000-_b200/csrc/host/roots.h"

using namespace wc;

namespace {

int failf(char* msg, size_t cap, const std::string& s) {
    if (msg && cap) {
        std::snprintf(msg, cap, "%s", s.c_str());
    }
    return 1;
}

const uint16_t DRAFT_POOL[19] = {1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 16, 17, 18, 19, 52, 53, 54};

// invariants.rs:13-31
void random_draft(Rng& rng, uint16_t* w, uint16_t* b, uint8_t* first) {
    auto pick4 = [&](uint16_t* out) {
        int n = 0;
        while (n < 4) {
            uint16_t id = DRAFT_POOL[rng.below(19)];
            bool dup = false;
            for (int i = 0; i < n; ++i) dup |= out[i] == id;
            if (!dup) out[n++] = id;
        }
    };
    pick4(w);
    pick4(b);
    *first = (rng.next_u64() & 1) == 0 ? WHITE : BLACK;
}

// invariants.rs:34-44
void initial_totals(const uint16_t* units, uint16_t* t) {
    for (int u = 0; u < N_UNITS; ++u) t[u] = 0;
    for (int i = 0; i < 4; ++i) {
        int u = index_of_id(units[i]);
        t[u] += def((uint8_t)u).coins;
    }
    t[ROYAL_COIN] += 1;
}

// invariants.rs:46-117
std::string check_invariants(const State& s, const uint16_t init[2][N_UNITS]) {
    char buf[256];
    for (int p = 0; p < 2; ++p)
        for (int u = 0; u < N_UNITS; ++u)
            if (s.total_coins((uint8_t)p, u) != init[p][u]) {
                std::snprintf(buf, sizeof buf, "coin conservation broke: player %d unit %d got %d want %d", p, u,
                              s.total_coins((uint8_t)p, u), init[p][u]);
                return buf;
            }
    const Board& b = board();
    for (int h = 0; h < N_HEXES; ++h) {
        if (s.hex_type[h] != NONE) {
            if (s.hex_owner[h] != WHITE && s.hex_owner[h] != BLACK) return "deployed stack without an owner";
            if (s.hex_height[h] < 1) return "deployed stack must be >= 1";
        } else if (s.hex_height[h] != 0 || s.hex_owner[h] != NONE) {
            return "empty hex with a height or an owner";
        }
        if (s.loc_marker[h] != NONE && !b.is_location[h]) return "marker on a non-location hex";
    }
    for (int p = 0; p < 2; ++p) {
        int on = s.markers_on_board((uint8_t)p);
        if (on > 6) return "more than 6 markers on the board";
        if (on + s.markers_hand[p] != 6) return "marker count broke";
        if (s.hand_size((uint8_t)p) > 3) return "hand held more than 3 coins";
        int owed = (s.pending.kind == C_WPPLAY && s.pending.a == p) ? 1 : 0;
        for (int i = 0; i < s.conts.n; ++i) owed += (s.conts.v[i].kind == C_WPPLAY && s.conts.v[i].a == p) ? 1 : 0;
        int flight = 0;
        for (int u = 0; u < N_UNITS; ++u) flight += s.zones[p][Z_INFLIGHT][u];
        if (s.is_terminal()) {
            if (flight != 0) return "a terminal has spent the in-flight coin";
        } else if (flight != owed) {
            return "in-flight zone must match the continuation tree";
        }
        if (flight > 1) return "at most one coin in flight";
    }
    if (s.winner != NONE && s.markers_on_board(s.winner) != 6) return "winner must have 6 markers";
    if (s.is_terminal() && s.winner == NONE) {
        float a = s.utility(0), c = s.utility(1);
        if (std::fabs(a + c) >= 1e-6f) return "utility must be zero-sum";
        if (std::fabs(a) >= 1.0f) return "horizon payoff must stay inside +/-1";
    }
    return "";
}

}  // namespace

extern "C" {

// invariants_random_playouts (invariants.rs:119-171) plus the encode / decode
// round trip (scenarios.rs:923-1010) of every legal action met on the way.
// stats4: games, total applies, cap hits, actions round-tripped.
int oracle_check_playouts(uint64_t seed, int n_games, int cap, uint64_t* stats4, char* msg, size_t msg_cap) {
    Rng rng(seed);
    uint64_t applies_total = 0, cap_hits = 0, tripped = 0;
    std::vector<Action> acts;
    for (int g = 0; g < n_games; ++g) {
        uint16_t w[4], b[4];
        uint8_t first;
        random_draft(rng, w, b, &first);
        uint16_t init[2][N_UNITS];
        initial_totals(w, init[0]);
        initial_totals(b, init[1]);
        State s = State::from_draft(w, b, first);
        std::string e = check_invariants(s, init);
        if (!e.empty()) return failf(msg, msg_cap, "game " + std::to_string(g) + " at setup: " + e);
        int n = 0;
        while (!s.is_terminal() && n < cap) {
            s.legal_actions_into(acts);
            if (acts.empty())
                return failf(msg, msg_cap, "game " + std::to_string(g) + ": no legal actions at a non-terminal state");
            for (const Action& a : acts) {
                Action back;
                if (!Action::decode(a.encode(), &back) || !(back == a) || back.encode() != a.encode())
                    return failf(msg, msg_cap, "action code " + std::to_string(a.encode()) + " does not round-trip");
                ++tripped;
            }
            s.apply_inplace(acts[rng.below(acts.size())]);
            e = check_invariants(s, init);
            if (!e.empty())
                return failf(msg, msg_cap, "game " + std::to_string(g) + " after " + std::to_string(n + 1) +
                                               " actions: " + e);
            ++n;
        }
        applies_total += n;
        if (!s.is_terminal()) ++cap_hits;
    }
    if (stats4) {
        stats4[0] = (uint64_t)n_games;
        stats4[1] = applies_total;
        stats4[2] = cap_hits;
        stats4[3] = tripped;
    }
    return 0;
}

// random_drafts_never_duplicate_a_unit_card (invariants.rs:182-205).
int oracle_check_drafts(int n_games, char* msg, size_t msg_cap) {
    for (int g = 0; g < n_games; ++g) {
        Rng rng((uint64_t)g);
        State s = make_game(rng, true);
        for (int u = 0; u < N_UNITS; ++u) {
            if (u == ROYAL_COIN) continue;
            int a = s.total_coins(0, u), c = s.total_coins(1, u);
            if (a != 0 && c != 0)
                return failf(msg, msg_cap, "game " + std::to_string(g) + ": unit " + std::to_string(u) +
                                               " drafted by both players");
            if (a + c > def((uint8_t)u).coins)
                return failf(msg, msg_cap, "game " + std::to_string(g) + ": unit " + std::to_string(u) +
                                               " has more coins in play than the card");
        }
    }
    return 0;
}

// the_exported_board_tables_describe_the_board (invariants.rs:211-241): the
// neighbour relation is symmetric and the location list is the marked hexes.
int oracle_check_board(char* msg, size_t msg_cap) {
    const Board& bd = board();
    for (int h = 0; h < N_HEXES; ++h)
        for (int d = 0; d < 6; ++d) {
            int n = bd.neighbors[h][d];
            if (n == NONE) continue;
            if (n >= N_HEXES) return failf(msg, msg_cap, "neighbour out of range");
            bool back = false;
            for (int e = 0; e < 6; ++e) back |= bd.neighbors[n][e] == h;
            if (!back) return failf(msg, msg_cap, "neighbour relation is not symmetric at hex " + std::to_string(h));
        }
    std::vector<int> marked, listed;
    for (int h = 0; h < N_HEXES; ++h)
        if (bd.is_location[h]) marked.push_back(h);
    for (int i = 0; i < N_LOCATIONS; ++i) listed.push_back(bd.location_hexes[i]);
    std::sort(listed.begin(), listed.end());
    if (marked != listed) return failf(msg, msg_cap, "location_hexes must be the marked hexes");
    return 0;
}

}  // extern "C"

namespace {

// rebel.rs:1407-1439 (`composed`): one transition per draw, composed; a step
// that finds the bag empty refills from the face-up pile.
void composed(const std::vector<Config>& cfg, const uint8_t* res0, const uint8_t* fu0, uint8_t k,
              std::vector<Config>& cur, DrawMap& draw) {
    DrawScratch sc;
    uint8_t res[NSLOT], fu[NSLOT];
    std::memcpy(res, res0, NSLOT);
    std::memcpy(fu, fu0, NSLOT);
    cur = cfg;
    std::vector<Config> next;
    DrawMap step, acc;
    draw = DrawMap();
    for (uint8_t j = 0; j < k; ++j) {
        uint8_t bag[NSLOT];
        cur[0].bag(res, bag);
        bool empty = true;
        for (int s = 0; s < NSLOT; ++s) empty &= bag[s] == 0;
        sc.transition(cur, res, fu, next, step, false);
        if (j == 0) {
            std::swap(draw, step);
        } else {
            sc.compose(draw, step, next.size(), acc);
            std::swap(draw, acc);
        }
        std::swap(cur, next);
        if (empty)
            for (int s = 0; s < NSLOT; ++s) {
                res[s] += fu[s];
                fu[s] = 0;
            }
    }
}

// rebel.rs:1441-1474 (`assert_same`)
std::string same(const std::vector<Config>& cfg, const uint8_t* res, const uint8_t* fu, uint8_t k, const char* what) {
    std::vector<Config> want_sup, sup;
    DrawMap want, map;
    composed(cfg, res, fu, k, want_sup, want);
    DrawScratch sc;
    sc.run(cfg, res, fu, k, sup, map);
    std::string w = what;
    if (sup.size() != want_sup.size()) return w + ": support size";
    for (size_t i = 0; i < sup.size(); ++i)
        if (!(sup[i] == want_sup[i])) return w + ": support";
    if (map.rows() != want.rows()) return w + ": rows";
    for (size_t i = 0; i < map.rows(); ++i) {
        std::vector<std::pair<uint32_t, float>> got, wnt;
        for (uint32_t e = map.start[i]; e < map.start[i + 1]; ++e) got.push_back({map.to[e], map.p[e]});
        for (uint32_t e = want.start[i]; e < want.start[i + 1]; ++e) wnt.push_back({want.to[e], want.p[e]});
        auto by_child = [](const std::pair<uint32_t, float>& a, const std::pair<uint32_t, float>& b) {
            return a.first < b.first;
        };
        std::sort(got.begin(), got.end(), by_child);
        std::sort(wnt.begin(), wnt.end(), by_child);
        if (got.size() != wnt.size()) return w + ": row " + std::to_string(i) + " children";
        float tot = 0.0f;
        for (size_t e = 0; e < got.size(); ++e) {
            if (got[e].first != wnt[e].first) return w + ": row " + std::to_string(i) + " children";
            if (std::fabs(got[e].second - wnt[e].second) >= 1e-5f) return w + ": row " + std::to_string(i) + " prob";
            tot += got[e].second;
        }
        if (std::fabs(tot - 1.0f) >= 1e-5f) return w + ": row " + std::to_string(i) + " does not sum to 1";
    }
    return "";
}

// rebel.rs:1477-1492 (`spread`)
bool spread(Rng& rng, uint8_t total, const uint8_t* cap, const uint8_t* used, uint8_t* out) {
    std::memset(out, 0, NSLOT);
    for (uint8_t t = 0; t < total; ++t) {
        bool placed = false;
        for (int tries = 0; tries < 32 && !placed; ++tries) {
            size_t s = rng.next_u64() % NSLOT;
            if (used[s] + out[s] < cap[s]) {
                out[s] += 1;
                placed = true;
            }
        }
        if (!placed) return false;
    }
    return true;
}

Config mk(std::initializer_list<int> hand, std::initializer_list<int> fd) {
    Config c;
    int i = 0;
    for (int v : hand) c.hand[i++] = (uint8_t)v;
    i = 0;
    for (int v : fd) c.fd[i++] = (uint8_t)v;
    return c;
}

}  // namespace

extern "C" {

// run_matches_composition (rebel.rs:1494-1583): five hand-built cases, then
// `n_fuzz` random supports from Rng(0xD12A). Returns the cases checked.
int oracle_check_draw_runs(int n_fuzz, int* checked, char* msg, size_t msg_cap) {
    struct Case {
        std::vector<Config> cfg;
        uint8_t res[NSLOT], fu[NSLOT];
        uint8_t k;
        const char* what;
    };
    std::vector<Case> cases = {
        {{mk({0, 0, 0, 0, 0}, {1, 1, 0, 0, 0}), mk({0, 0, 0, 0, 0}, {0, 0, 1, 1, 0})},
         {5, 4, 3, 2, 5}, {1, 0, 2, 0, 0}, 3, "plenty"},
        {{mk({0, 0, 0, 0, 0}, {2, 1, 0, 0, 0}), mk({0, 0, 0, 0, 0}, {2, 0, 1, 0, 0}),
          mk({0, 0, 0, 0, 0}, {1, 1, 1, 0, 0})},
         {2, 1, 1, 0, 0}, {1, 2, 0, 0, 0}, 3, "refill"},
        {{mk({1, 0, 0, 0, 0}, {0, 0, 0, 0, 0})}, {2, 0, 0, 0, 0}, {0, 0, 0, 0, 0}, 2, "empty refill"},
        {{mk({0, 0, 0, 0, 0}, {0, 0, 0, 0, 0})}, {0, 0, 0, 0, 0}, {2, 0, 0, 0, 0}, 3, "shortage"},
        {{mk({0, 0, 0, 0, 0}, {0, 0, 0, 0, 0})}, {1, 1, 0, 0, 0}, {1, 0, 0, 0, 0}, 3, "exact dry"},
    };
    int n = 0;
    for (const Case& c : cases) {
        std::string e = same(c.cfg, c.res, c.fu, c.k, c.what);
        if (!e.empty()) return failf(msg, msg_cap, e);
        ++n;
    }
    Rng rng(0xD12A);
    int done = 0;
    while (done < n_fuzz) {
        uint8_t res[NSLOT], fu[NSLOT];
        for (int s = 0; s < NSLOT; ++s) res[s] = (uint8_t)(rng.next_u64() % 4);
        for (int s = 0; s < NSLOT; ++s) fu[s] = (uint8_t)(rng.next_u64() % 2);
        uint8_t ht = (uint8_t)(rng.next_u64() % 3);
        uint8_t fdt = (uint8_t)(rng.next_u64() % 4);
        uint8_t k = (uint8_t)(3 - ht);
        std::vector<Config> cfgs;
        const uint8_t zero[NSLOT] = {0, 0, 0, 0, 0};
        for (int i = 0; i < 6; ++i) {
            Config c;
            if (!spread(rng, ht, res, zero, c.hand)) continue;
            if (!spread(rng, fdt, res, c.hand, c.fd)) continue;
            cfgs.push_back(c);
        }
        if (cfgs.empty()) continue;
        std::sort(cfgs.begin(), cfgs.end());
        cfgs.erase(std::unique(cfgs.begin(), cfgs.end()), cfgs.end());
        std::string e = same(cfgs, res, fu, k, "fuzz");
        if (!e.empty()) return failf(msg, msg_cap, e + " (fuzz case " + std::to_string(done) + ")");
        ++done;
        ++n;
    }
    if (checked) *checked = n;
    return 0;
}

}  // extern "C"
