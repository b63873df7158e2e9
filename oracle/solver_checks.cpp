// TEST INFRASTRUCTURE (CPU only, never linked into the product library).
//
// Structural tests of the subgame tree from engine/tests/rebel_solver.rs,
// restated over the host tree builder and the CPU solver:
//   :449  draw_pass_through_consistency
//   :612  warrior_priest_draw_walks_through_the_tree
//   :753  depth_is_spent_on_coin_plays_not_micro_choices
// (the tabular-CFR agreement :167 and snapshot_iters :579 are in
// oracle_capi.cpp / tests/test_solver_oracle.py). Each returns 0, or writes a
// message and returns nonzero.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../war-chest-bot-9000-_b200/csrc/host/roots.h"
#include "cfr_cpu.h"

using namespace wc;

namespace {

int failf(char* msg, size_t cap, const std::string& s) {
    if (msg && cap) std::snprintf(msg, cap, "%s", s.c_str());
    return 1;
}

// rebel_solver.rs:396-437: a real board reached by random play, both hands
// forced to one coin (the rest into the bag) so the round boundary and its
// draws fall inside the last `plies` main plays.
bool draw_position(uint64_t seed, size_t warmup, uint16_t plies, State* out) {
    Rng rng(seed);
    State s = make_game(rng, false);
    for (size_t i = 0; i < warmup; ++i) {
        if (s.is_terminal()) return false;
        std::vector<Action> acts = s.legal_actions();
        s.apply_inplace(acts[rng.below(acts.size())]);
    }
    if (s.is_terminal() || s.pending.kind != C_MAINPLAY) return false;
    const Ctx ctx = Ctx::make(s);
    for (uint8_t p = 0; p < 2; ++p) {
        for (int u = 0; u < N_UNITS; ++u) {
            s.zones[p][Z_BAG][u] += s.zones[p][Z_HAND][u];
            s.zones[p][Z_HAND][u] = 0;
            s.zones[p][Z_BAG][u] += s.zones[p][Z_FACEDOWN][u];
            s.zones[p][Z_FACEDOWN][u] = 0;
        }
        int hand_slot = NSLOT;
        for (int k = 0; k < NSLOT; ++k)
            if (s.zones[p][Z_BAG][ctx.slots[p][k]] > 0) {
                hand_slot = k;
                break;
            }
        if (hand_slot == NSLOT) return false;
        Config cfg;
        cfg.hand[hand_slot] = 1;
        set_config(s, p, ctx, cfg);
    }
    s.main_plays = (uint16_t)(MAX_MAIN_PLAYS - plies);
    *out = s;
    return true;
}

const std::vector<Config>& sup(const Tree& t, uint32_t node, int p) { return t.supports[t.nodes[node].sup[p]]; }

bool same_support(const std::vector<Config>& a, const std::vector<Config>& b) {
    return a.size() == b.size() && std::equal(a.begin(), a.end(), b.begin());
}

std::vector<float> flat_root(const Belief* bel) {
    std::vector<float> r(bel[0].p);
    r.insert(r.end(), bel[1].p.begin(), bel[1].p.end());
    return r;
}

}  // namespace

extern "C" {

// rebel_solver.rs:449-573. stats: rejected, built, too large, no chance node, solved.
int oracle_check_draw_pass_through(int* stats5, char* msg, size_t cap) {
    const oracle::Net empty;
    int cnt[5] = {0, 0, 0, 0, 0}, checked = 0;
    for (uint64_t seed = 0; seed < 4000; ++seed) {
        State s;
        if (!draw_position(seed, 60 + (size_t)(seed % 120), 4, &s)) {
            ++cnt[0];
            continue;
        }
        const Ctx ctx = Ctx::make(s);
        const Belief bel[2] = {uniform_belief(s, ctx, 0), uniform_belief(s, ctx, 1)};
        if (bel[0].size() * bel[1].size() > 1000) {
            ++cnt[0];
            continue;
        }
        {
            std::vector<Action> acts;
            std::vector<int8_t> aslot;
            std::vector<uint8_t> fdown;
            node_actions(s, s.to_act(), ctx, bel[s.to_act()].cfg, acts, aslot, fdown);
            if (acts.size() > 14) {
                ++cnt[0];
                continue;
            }
        }
        SolveCfg cfg;
        cfg.depth = 5;
        cfg.iters = 80;
        cfg.snapshots = true;
        cfg.keep_states = true;
        cfg.node_cap = 20001;
        auto t = build_tree(s, ctx, cfg, bel);
        if (t->capped || t->nodes.size() > 20000) {
            ++cnt[2];
            continue;
        }
        bool any_chance = false;
        for (const NodeRec& n : t->nodes) any_chance = any_chance || n.kind == NK_CHANCE;
        if (!any_chance) {
            ++cnt[3];
            continue;
        }
        ++cnt[1];
        for (uint32_t i = 0; i < t->nodes.size(); ++i) {
            const NodeRec& n = t->nodes[i];
            if (n.kind != NK_CHANCE) continue;
            if (n.nch != 1) return failf(msg, cap, "a draw must have exactly one public child");
            const int me = n.player;
            const uint32_t ch = t->child[n.child_off];
            if (!same_support(sup(*t, ch, 1 - me), sup(*t, i, 1 - me)))
                return failf(msg, cap, "idle player's support must pass through the draw untouched");
            if (n.draw_steps < 1) return failf(msg, cap, "a draw node covers at least one draw");
            State ws = t->states[i];
            Belief b;
            b.cfg = sup(*t, i, me);
            b.p.assign(b.cfg.size(), 1.0f);
            for (int step = 0; step < n.draw_steps; ++step) {
                uint8_t res[NSLOT], fu[NSLOT];
                reserve(ws, n.player, ctx, res);
                faceup_counts(ws, n.player, ctx, fu);
                b = belief_after_draw(b, res, fu, false);
                std::vector<Action> acts = ws.legal_actions();
                ws.apply_inplace(acts[0]);
            }
            if (!same_support(sup(*t, ch, me), b.cfg))
                return failf(msg, cap, "post-draw support must equal belief_after_draw's, in order (seed " +
                                           std::to_string(seed) + ")");
            const size_t rows = sup(*t, i, me).size();
            for (size_t ci = 0; ci < rows; ++ci) {
                float sum = 0.0f;
                for (uint32_t e = t->draw_start[n.draw_off + ci]; e < t->draw_start[n.draw_off + ci + 1]; ++e)
                    sum += t->draw_p[e];
                if (std::fabs(sum - 1.0f) >= 1e-5f)
                    return failf(msg, cap, "draw row " + std::to_string(ci) + " sums to " + std::to_string(sum));
            }
            if (t->states[ch].hand_size(n.player) != t->states[i].hand_size(n.player) + n.draw_steps)
                return failf(msg, cap, "each covered draw adds exactly one coin to the hand");
        }
        oracle::Solver sv(*t, &empty);
        sv.multistep(80);
        auto vals = sv.value_under({flat_root(bel)});
        double v0 = 0.0, v1 = 0.0;
        for (size_t c = 0; c < bel[0].size(); ++c) v0 += (double)bel[0].p[c] * (double)vals[0][c];
        for (size_t c = 0; c < bel[1].size(); ++c) v1 += (double)bel[1].p[c] * (double)vals[0][bel[0].size() + c];
        if (std::fabs(v0 + v1) >= 0.05) {
            char m[160];
            std::snprintf(m, sizeof m, "seed %llu: root values not zero-sum with draws in the tree: %.4f + %.4f",
                          (unsigned long long)seed, v0, v1);
            return failf(msg, cap, m);
        }
        ++checked;
        ++cnt[4];
        if (checked >= 6) break;
    }
    for (int i = 0; i < 5; ++i) stats5[i] = cnt[i];
    if (checked < 4) return failf(msg, cap, "only " + std::to_string(checked) + " draw positions exercised");
    return 0;
}

// rebel_solver.rs:612-751.
int oracle_check_warrior_priest_draw_walk(char* msg, size_t cap) {
    const oracle::Net empty;
    State s = State::blank(WHITE);
    s.set_unit(17, WHITE, WARRIOR_PRIEST, 1);
    s.set_unit(19, BLACK, FOOTMAN, 3);
    for (uint8_t u : {WARRIOR_PRIEST, SWORDSMAN, PIKEMAN, CROSSBOWMAN, ROYAL_COIN}) s.add_zone(WHITE, Z_BAG, u, 1);
    for (uint8_t u : {FOOTMAN, ARCHER, CAVALRY, LANCER, ROYAL_COIN}) s.add_zone(BLACK, Z_BAG, u, 1);
    s.add_zone(WHITE, Z_HAND, WARRIOR_PRIEST, 1);
    const Ctx ctx = Ctx::make(s);
    const int wp = ctx.slot_of[0][WARRIOR_PRIEST], sw = ctx.slot_of[0][SWORDSMAN];
    if (wp == sw) return failf(msg, cap, "slots collide");
    Config c1;
    c1.hand[wp] = 1;
    const Belief bel[2] = {Belief::point(c1), Belief::point(Config())};
    SolveCfg cfg;
    cfg.depth = 2;
    cfg.iters = 8;
    cfg.snapshots = true;
    cfg.keep_states = true;
    auto t = build_tree(s, ctx, cfg, bel);
    std::vector<uint32_t> draws;
    for (uint32_t i = 0; i < t->nodes.size(); ++i)
        if (t->nodes[i].kind == NK_CHANCE && t->states[i].pending.kind == C_WPDRAW) draws.push_back(i);
    if (draws.size() != 1) return failf(msg, cap, "exactly one WP draw in the tree, found " + std::to_string(draws.size()));
    const uint32_t d = draws[0];
    const NodeRec& n = t->nodes[d];
    if (n.nch != 1) return failf(msg, cap, "a draw has exactly one public child");
    if (n.draw_steps != 1) return failf(msg, cap, "a WP draw is a single draw");
    uint8_t res[NSLOT], fu[NSLOT];
    reserve(t->states[d], n.player, ctx, res);
    faceup_counts(t->states[d], n.player, ctx, fu);
    Belief pre;
    pre.cfg = sup(*t, d, n.player);
    pre.p.assign(pre.cfg.size(), 1.0f);
    const Belief post = belief_after_draw(pre, res, fu, true);
    const uint32_t ch = t->child[n.child_off];
    if (!same_support(sup(*t, ch, n.player), post.cfg))
        return failf(msg, cap, "post-draw support must equal belief_after_draw's, in order");
    for (const Config& c : sup(*t, ch, n.player))
        if (c.inflight < 0) return failf(msg, cap, "a WP draw child carries its coin");
    for (size_t ci = 0; ci < pre.cfg.size(); ++ci) {
        float sum = 0.0f;
        for (uint32_t e = t->draw_start[n.draw_off + ci]; e < t->draw_start[n.draw_off + ci + 1]; ++e) sum += t->draw_p[e];
        if (std::fabs(sum - 1.0f) >= 1e-5f) return failf(msg, cap, "a draw row is not a distribution");
    }
    // the child is the forced-play decision node; its legality is the in-flight coin
    const NodeRec& w = t->nodes[ch];
    if (t->states[ch].pending.kind != C_WPPLAY) return failf(msg, cap, "the draw's child is not a WarriorPriestPlay");
    if (w.kind != NK_DECISION || w.na == 0) return failf(msg, cap, "the forced play is not a decision node with actions");
    const int me = w.player;
    const std::vector<Config>& wc = sup(*t, ch, me);
    std::vector<int> drawn;
    for (size_t ci = 0; ci < wc.size(); ++ci) {
        const int pend = wc[ci].inflight;
        if (pend < 0) return failf(msg, cap, "a forced-play config has no coin in flight");
        drawn.push_back(pend);
        const uint32_t lo = t->soff[ch] + t->legal_off[w.row_off + ci], hi = t->soff[ch] + t->legal_off[w.row_off + ci + 1];
        for (uint32_t a = 0; a < w.na; ++a) {
            bool legal = false;
            for (uint32_t cell = lo; cell < hi; ++cell) legal = legal || t->legal_action[cell] == a;
            if (legal != (t->aslot[w.act_off + a] == pend))
                return failf(msg, cap, "WP play legality must be the in-flight coin");
        }
    }
    std::sort(drawn.begin(), drawn.end());
    drawn.erase(std::unique(drawn.begin(), drawn.end()), drawn.end());
    if (drawn.size() < 2) return failf(msg, cap, "expected both drawn coins in the support");
    for (uint32_t k = 0; k < w.nch; ++k)
        for (const Config& cc : sup(*t, t->child[w.child_off + k], me))
            if (cc.inflight >= 0) return failf(msg, cap, "the forced play spends the coin");
    for (uint32_t i = 0; i < t->nodes.size(); ++i)
        if (t->nodes[i].kind == NK_LEAF && !t->states[i].is_terminal() && t->states[i].pending.kind != C_MAINPLAY)
            return failf(msg, cap, "non-terminal leaf " + std::to_string(i) + " is not a MainPlay state");
    oracle::Solver sv(*t, &empty);
    sv.multistep(8);
    auto vals = sv.value_under({flat_root(bel)});
    for (float v : vals[0])
        if (!std::isfinite(v)) return failf(msg, cap, "a root value is not finite");
    return 0;
}

// rebel_solver.rs:753-835.
int oracle_check_depth_counts_coin_plays(char* msg, size_t cap) {
    const oracle::Net empty;
    Rng rng(1234);
    for (int game = 0; game < 400; ++game) {
        State s = make_game(rng, false);
        while (!s.is_terminal()) {
            if (s.is_chance()) {
                std::vector<Action> acts = s.legal_actions();
                s.apply_inplace(acts[rng.below(acts.size())]);
                continue;
            }
            std::vector<Action> acts = s.legal_actions();
            bool free_child = false;
            for (const Action& a : acts) {
                if (action_coin(a, s) != NONE) continue;
                State cs = s;
                cs.apply_inplace(a);
                free_child = free_child || (!cs.is_terminal() && !cs.is_chance());
            }
            if (free_child) {
                const Ctx ctx = Ctx::make(s);
                const Belief bel[2] = {uniform_belief(s, ctx, 0), uniform_belief(s, ctx, 1)};
                const uint8_t root_player = s.to_act();
                SolveCfg cfg;
                cfg.depth = 1;
                cfg.iters = 4;
                cfg.snapshots = false;
                auto t1 = build_tree(s, ctx, cfg, bel);
                oracle::Solver sv1(*t1, &empty);
                sv1.multistep(4);
                bool expanded = false;
                for (size_t i = 1; i < t1->nodes.size(); ++i) expanded = expanded || t1->nodes[i].kind != NK_LEAF;
                if (!expanded)
                    return failf(msg, cap, "depth 1 was consumed by a tactic micro-choice: nothing expanded below the root");
                cfg.depth = 2;
                auto t2 = build_tree(s, ctx, cfg, bel);
                oracle::Solver sv2(*t2, &empty);
                sv2.multistep(4);
                bool opp = false, opp_expanded = false;
                for (const NodeRec& n : t2->nodes) {
                    if (n.player == root_player) continue;
                    opp = true;
                    opp_expanded = opp_expanded || n.kind != NK_LEAF;
                }
                if (opp && !opp_expanded)
                    return failf(msg, cap, "depth 2 contained only leaf opponent nodes: the opponent's move never got expanded");
                return 0;
            }
            s.apply_inplace(acts[rng.below(acts.size())]);
        }
    }
    return failf(msg, cap, "no position with a free micro-choice found in 400 random games");
}

}  // extern "C"
