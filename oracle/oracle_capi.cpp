// TEST INFRASTRUCTURE — C entry points of the CPU oracle, for tests/,
// __graft_entry__.smoke() and bench.py's CPU-baseline leg. Never linked by the
// product library.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <memory>
#include <cstring>
#include <map>
#include <thread>
#include <vector>

#include "../war-chest-bot-9000-_b200/csrc/host/roots.h"
#include "../war-chest-bot-9000-_b200/csrc/host/walk.h"
#include "cfr_cpu.h"

using namespace oracle;

namespace {

thread_local std::string g_err;

struct OracleCfg {
    int32_t depth, iters, snapshots, pad;
    float alpha, beta, gamma, predict;
    uint64_t node_cap;
};

wc::SolveCfg to_cfg(const OracleCfg* c) {
    wc::SolveCfg s;
    s.depth = c->depth;
    s.iters = c->iters;
    s.snapshots = c->snapshots != 0;
    s.cfr = {c->alpha, c->beta, c->gamma, c->predict};
    s.node_cap = (size_t)c->node_cap;
    return s;
}

struct Handle {
    wc::Root root;
    std::unique_ptr<wc::Tree> tree;
    Net net;
    std::unique_ptr<Solver> sv;
};

// --------------------------------------------- tabular vanilla CFR (f64)
// tests/rebel_solver.rs:66-165: textbook CFR over world states, information
// sets keyed by the public observation history plus the actor's own config.

struct Tab {
    std::map<std::pair<std::vector<uint32_t>, uint64_t>, std::vector<double>> regret, strat;
};

std::vector<double> regret_match(const std::vector<double>& r) {
    std::vector<double> pos(r.size());
    double s = 0.0;
    for (size_t i = 0; i < r.size(); ++i) { pos[i] = r[i] > 0.0 ? r[i] : 0.0; s += pos[i]; }
    if (s > 0.0) for (double& x : pos) x /= s;
    else for (double& x : pos) x = 1.0 / (double)r.size();
    return pos;
}

double tab_cfr(Tab& t, const wc::State& s, const wc::Ctx& ctx, std::vector<uint32_t>& hist, double reach[2], int trav) {
    if (s.is_terminal()) return (double)s.utility(trav);
    uint8_t p = s.to_act();
    wc::Config cfg = wc::true_config(s, p, ctx);
    std::vector<wc::Action> acts;
    std::vector<int8_t> aslot;
    std::vector<uint8_t> fdown;
    wc::node_actions(s, p, ctx, std::vector<wc::Config>{cfg}, acts, aslot, fdown);
    auto key = std::make_pair(hist, cfg.key());
    size_t n = acts.size();
    auto& reg = t.regret[key];
    if (reg.empty()) reg.assign(n, 0.0);
    std::vector<double> sigma = regret_match(reg);
    std::vector<double> util(n);
    double node_util = 0.0;
    for (size_t i = 0; i < n; ++i) {
        wc::State ns = s.apply(acts[i]);
        double r[2] = {reach[0], reach[1]};
        r[p] *= sigma[i];
        hist.push_back(wc::obs_key(acts[i]));
        util[i] = tab_cfr(t, ns, ctx, hist, r, trav);
        hist.pop_back();
        node_util += sigma[i] * util[i];
    }
    if (p == trav) {
        double opp = reach[1 - trav];
        auto& rg = t.regret[key];
        for (size_t i = 0; i < n; ++i) rg[i] += opp * (util[i] - node_util);
        auto& st = t.strat[key];
        if (st.empty()) st.assign(n, 0.0);
        for (size_t i = 0; i < n; ++i) st[i] += reach[trav] * sigma[i];
    }
    return node_util;
}

}  // namespace

extern "C" {

const char* oracle_last_error() { return g_err.c_str(); }

void oracle_set_cap_marker_value(float v) { wc::set_cap_marker_value(v); }

int oracle_root_generate(uint64_t seed, int plies, int random_draft, uint8_t* buf, size_t cap, size_t* len) {
    wc::Root r;
    if (!wc::make_root(seed, plies, random_draft != 0, &r)) { g_err = "game ended before the root"; return 1; }
    std::vector<uint8_t> b = wc::root_to_bytes(r);
    *len = b.size();
    if (b.size() > cap) { g_err = "buffer too small"; return 2; }
    std::memcpy(buf, b.data(), b.size());
    return 0;
}

// micro_position + uniform beliefs of tests/rebel_solver.rs:28-64.
int oracle_micro_root(uint64_t seed, int warmup, int plies, uint8_t* buf, size_t cap, size_t* len) {
    wc::Rng rng(seed);
    wc::State s = wc::make_game(rng, false);
    std::vector<wc::Action> acts;
    for (int i = 0; i < warmup; ++i) {
        if (s.is_terminal()) return 1;
        s.legal_actions_into(acts);
        s.apply_inplace(acts[rng.below(acts.size())]);
    }
    if (s.is_terminal() || s.is_chance() || s.pending.kind != wc::C_MAINPLAY) return 1;
    if (s.hand_size(0) < 2 || s.hand_size(1) < 2) return 1;
    s.main_plays = (uint16_t)(wc::MAX_MAIN_PLAYS - plies);
    wc::Root r;
    r.s = s;
    r.ctx = wc::Ctx::make(s);
    r.bel[0] = wc::uniform_belief(s, r.ctx, 0);
    r.bel[1] = wc::uniform_belief(s, r.ctx, 1);
    std::vector<uint8_t> b = wc::root_to_bytes(r);
    *len = b.size();
    if (b.size() > cap) return 2;
    std::memcpy(buf, b.data(), b.size());
    return 0;
}

// tests/rebel_solver.rs:136-162.
double oracle_tabular_value(const uint8_t* root, size_t len, int iters) {
    wc::Root r;
    if (!wc::root_from_bytes(root, len, &r)) return std::nan("");
    Tab t;
    double value = 0.0;
    for (int it = 0; it < iters; ++it) {
        int trav = it % 2;
        double total = 0.0;
        for (size_t i0 = 0; i0 < r.bel[0].size(); ++i0)
            for (size_t i1 = 0; i1 < r.bel[1].size(); ++i1) {
                wc::State w = r.s;
                wc::set_config(w, 0, r.ctx, r.bel[0].cfg[i0]);
                wc::set_config(w, 1, r.ctx, r.bel[1].cfg[i1]);
                double pr[2] = {(double)r.bel[0].p[i0], (double)r.bel[1].p[i1]};
                std::vector<uint32_t> hist;
                double v = tab_cfr(t, w, r.ctx, hist, pr, trav);
                if (trav == 0) total += pr[0] * pr[1] * v;
            }
        if (trav == 0 && it * 2 >= iters) value += total;
    }
    return value / ((double)iters / 4.0);
}

void* oracle_solver_new(const uint8_t* root, size_t len, const OracleCfg* cfg, const float* w, const float* b,
                        const float* ln) {
    try {
        auto h = std::make_unique<Handle>();
        if (!wc::root_from_bytes(root, len, &h->root)) { g_err = "bad root bytes"; return nullptr; }
        h->tree = wc::build_tree(h->root.s, h->root.ctx, to_cfg(cfg), h->root.bel);
        if (h->tree->capped) { g_err = "tree hit the node cap"; return nullptr; }
        if (w) {
            h->net.w.assign(w, w + h->net.L.w_len);
            h->net.b.assign(b, b + h->net.L.b_len);
            h->net.ln.assign(ln, ln + h->net.L.ln_len);
            h->net.empty = false;
        }
        h->sv = std::make_unique<Solver>(*h->tree, &h->net);
        return h.release();
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}

void oracle_solver_free(void* p) { delete static_cast<Handle*>(p); }

// Tree shape: nodes, cells, rows, terminal leaves, ncfg, levels, all-leaves-terminal.
void oracle_solver_shape(void* p, uint64_t* out7) {
    const wc::Tree& t = *static_cast<Handle*>(p)->tree;
    bool all_term = true;
    for (const wc::NodeRec& n : t.nodes)
        if (n.kind == wc::NK_LEAF && !n.terminal) all_term = false;
    out7[0] = t.nodes.size();
    out7[1] = t.ncells();
    out7[2] = t.leaf_rows.size();
    out7[3] = t.term_leaves.size();
    out7[4] = t.ncfg;
    out7[5] = (uint64_t)t.max_depth() + 1;
    out7[6] = all_term ? 1 : 0;
}

// Distinct terminal utilities for player 0, scaled by 1000 and truncated.
int oracle_solver_outcomes(void* p) {
    const wc::Tree& t = *static_cast<Handle*>(p)->tree;
    std::vector<int> o;
    for (const wc::NodeRec& n : t.nodes)
        if (n.kind == wc::NK_LEAF && n.terminal) o.push_back((int)((n.player == 0 ? n.util : -n.util) * 1000.0f));
    std::sort(o.begin(), o.end());
    return (int)(std::unique(o.begin(), o.end()) - o.begin());
}

void oracle_solver_multistep(void* p, int iters) { static_cast<Handle*>(p)->sv->multistep(iters); }

size_t oracle_solver_ncells(void* p) { return static_cast<Handle*>(p)->tree->ncells(); }
size_t oracle_solver_nsnaps(void* p) { return static_cast<Handle*>(p)->sv->snaps.size(); }

int oracle_solver_snapshot(void* p, size_t which, float* out) {
    Solver& sv = *static_cast<Handle*>(p)->sv;
    if (which >= sv.snaps.size()) return 1;
    std::memcpy(out, sv.snaps[which].data(), sv.snaps[which].size() * 4);
    return 0;
}

void oracle_root_sizes(void* p, uint64_t* out2) {
    const wc::Tree& t = *static_cast<Handle*>(p)->tree;
    out2[0] = t.nc(0, 0);
    out2[1] = t.nc(0, 1);
}

// roots: nroots x (nc0 + nc1) floats; out: same shape.
int oracle_value_under(void* p, const float* roots, size_t nroots, float* out) {
    Handle& h = *static_cast<Handle*>(p);
    size_t w = h.tree->nc(0, 0) + h.tree->nc(0, 1);
    std::vector<std::vector<float>> rv;
    for (size_t i = 0; i < nroots; ++i) rv.emplace_back(roots + i * w, roots + (i + 1) * w);
    auto res = h.sv->value_under(rv);
    for (size_t i = 0; i < nroots; ++i) std::memcpy(out + i * w, res[i].data(), w * 4);
    return 0;
}

void oracle_nash_conv(void* p, float* nash, float* zs) { static_cast<Handle*>(p)->sv->nash_conv(nash, zs); }

// Replace the solver's latest strategy snapshot with an external average
// strategy (reference cell layout), so nash_conv and value_under evaluate it:
// the exploitability of another solver's output under this network.
int oracle_set_strategy(void* p, const float* strat, size_t n) {
    Solver& sv = *static_cast<Handle*>(p)->sv;
    if (n != sv.cur.size()) return 1;
    std::vector<float> s(strat, strat + n);
    if (sv.snaps.empty()) sv.snaps.push_back(std::move(s));
    else sv.snaps.back() = std::move(s);
    return 0;
}

// Exit leaves in result order: network rows, then terminal leaves.
size_t oracle_exit_leaves(void* p, uint32_t* out) {
    const wc::Tree& t = *static_cast<Handle*>(p)->tree;
    size_t n = 0;
    for (uint32_t i : t.leaf_rows) { if (out) out[n] = i; ++n; }
    for (uint32_t i : t.term_leaves) { if (out) out[n] = i; ++n; }
    return n;
}

// (nsnaps - 1) x (nc0 + nc1) floats at `leaf`.
int oracle_carried_beliefs(void* p, uint32_t leaf, float* out) {
    Handle& h = *static_cast<Handle*>(p);
    auto res = h.sv->carried_beliefs(leaf);
    size_t at = 0;
    for (auto& v : res) { std::memcpy(out + at, v.data(), v.size() * 4); at += v.size(); }
    return 0;
}

uint64_t oracle_leaf_node(void* p, size_t leaf_index) {
    return static_cast<Handle*>(p)->tree->leaf_rows[leaf_index];
}

// Leaf-network pieces for per-stage parity: P[rows, 256], jp[rows, 128],
// f[ncfg, 256], g[ncfg, 64], and h[rows, 256] for `player` under the current
// pooled beliefs.
int oracle_net_pieces(void* p, float* pb, float* jp, float* f, float* g) {
    Solver& sv = *static_cast<Handle*>(p)->sv;
    sv.ensure_leaf_batch();
    if (!sv.net_ready()) return 1;
    if (pb) std::memcpy(pb, sv.pb.data(), sv.pb.size() * 4);
    if (jp) std::memcpy(jp, sv.jp.data(), sv.jp.size() * 4);
    if (f) std::memcpy(f, sv.cf.data(), sv.cf.size() * 4);
    if (g) std::memcpy(g, sv.cg.data(), sv.cg.size() * 4);
    return 0;
}

// Leaf values for traverser p at the solver's initial reaches (search.rs:1550):
// network rows in leaf_rows order, each row's p-configs in support order.
// With out == NULL only the count is returned (nothing is evaluated).
size_t oracle_leaf_values(void* h, int p, float* out) {
    Solver& sv = *static_cast<Handle*>(h)->sv;
    const wc::Tree& t = *static_cast<Handle*>(h)->tree;
    if (!out) {
        size_t n = 0;
        for (uint32_t i : t.leaf_rows) n += t.nc(i, p);
        return n;
    }
    sv.leaf_values(p);
    size_t at = 0;
    for (uint32_t i : t.leaf_rows) {
        size_t n = t.nc(i, p);
        if (out) std::memcpy(out + at, sv.vals.data() + sv.voff[i], 4 * n);
        at += n;
    }
    return at;
}

// The readout's inputs behind oracle_leaf_values(p): the join output h of
// every network row (rows x 256), the opponent's reach mass per row, and the
// config index (into the f table of oracle_net_pieces) of every value.
int oracle_leaf_parts(void* h, int p, float* hout, float* opp_reach, uint32_t* cidx) {
    Solver& sv = *static_cast<Handle*>(h)->sv;
    const wc::Tree& t = *static_cast<Handle*>(h)->tree;
    if (!sv.net_ready()) return 1;
    sv.leaf_values(p);
    std::memcpy(hout, sv.h.data(), 4 * t.leaf_rows.size() * 256);
    size_t at = 0;
    for (size_t r = 0; r < t.leaf_rows.size(); ++r) {
        uint32_t i = t.leaf_rows[r];
        const float* ro = sv.reach_of(i, 1 - p);
        float s = 0.0f;
        for (size_t c = 0; c < t.nc(i, 1 - p); ++c) s += ro[c];
        opp_reach[r] = s;
        const uint32_t* idx = t.leaf_cidx.data() + t.leaf_coff[2 * r + p];
        for (size_t c = 0; c < t.nc(i, p); ++c) cidx[at++] = idx[c];
    }
    return 0;
}

// The continual re-solving walk (the host Game, selfplay.rs:466-905) with
// every subgame solved here by the CPU solver, which carries its exit beliefs
// in f32 as the reference's CPU walk does. Writes the game's counters and
// its final state and beliefs in the root encoding.
int oracle_walk(uint64_t seed, int random_draft, const OracleCfg* cfg, const float* w, const float* b,
                const float* ln, uint32_t max_solves, int64_t* counters8, uint8_t* root_out, size_t cap,
                size_t* len) {
    try {
        auto net = std::make_shared<Net>();
        if (w) {
            net->w.assign(w, w + net->L.w_len);
            net->b.assign(b, b + net->L.b_len);
            net->ln.assign(ln, ln + net->L.ln_len);
            net->empty = false;
        }
        wc::Game g(seed, random_draft != 0, to_cfg(cfg));
        g.set_max_solves(max_solves);
        while (g.advance() == wc::Game::NEED_SOLVE) {
            std::shared_ptr<wc::Tree> tree(g.take_pending_tree().release());
            auto sv = std::make_shared<Solver>(*tree, net.get());
            sv->multistep(tree->cfg.iters);
            std::vector<std::vector<float>> roots;
            const size_t w0 = tree->nc(0, 0) + tree->nc(0, 1);
            for (uint32_t r = 0; r < g.pending_nroots(); ++r)
                roots.emplace_back(g.pending_roots().begin() + r * w0, g.pending_roots().begin() + (r + 1) * w0);
            sv->value_under(roots);  // Phase 2, as the solve would run it
            wc::WalkResult res;
            res.strategy = sv->average();
            res.cpu_carried = [tree, sv, net](uint32_t node) { return sv->carried_beliefs(node); };
            g.resume(res);
        }
        g.counters(counters8);
        wc::Root r;
        r.s = g.state();
        r.ctx = g.ctx();
        r.bel[0] = g.belief(0);
        r.bel[1] = g.belief(1);
        std::vector<uint8_t> bytes = wc::root_to_bytes(r);
        if (len) *len = bytes.size();
        if (!root_out || bytes.size() > cap) { g_err = "root buffer too small"; return 2; }
        std::memcpy(root_out, bytes.data(), bytes.size());
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return 1;
    }
}

// Per network row, the number of player-p configs it carries (the row
// structure of oracle_leaf_values / oracle_leaf_parts). Returns the rows.
size_t oracle_leaf_row_counts(void* h, int p, uint32_t* out) {
    const wc::Tree& t = *static_cast<Handle*>(h)->tree;
    if (out)
        for (size_t r = 0; r < t.leaf_rows.size(); ++r) out[r] = (uint32_t)t.nc(t.leaf_rows[r], p);
    return t.leaf_rows.size();
}

// Fraction of network leaf rows whose player-q reach mass is exactly zero at
// the solver's current reaches (the rows whose values for the other player
// are all zero).
double oracle_zero_mass_fraction(void* h, int q) {
    Solver& sv = *static_cast<Handle*>(h)->sv;
    const wc::Tree& t = *static_cast<Handle*>(h)->tree;
    if (t.leaf_rows.empty()) return 0.0;
    size_t zero = 0;
    for (uint32_t i : t.leaf_rows) {
        const float* ro = sv.reach_of(i, q);
        float s = 0.0f;
        for (size_t c = 0; c < t.nc(i, q); ++c) s += ro[c];
        zero += s == 0.0f;
    }
    return (double)zero / (double)t.leaf_rows.size();
}

void oracle_layout(uint64_t* out3) {
    Layout L;
    out3[0] = L.w_len;
    out3[1] = L.b_len;
    out3[2] = L.ln_len;
}

// (gamma offset, width) of every LayerNorm, for seeding test weights.
size_t oracle_norms(uint64_t* g_off, uint64_t* width) {
    Layout L;
    for (size_t i = 0; i < L.norm_g.size(); ++i) {
        if (g_off) g_off[i] = L.norm_g[i];
        if (width) width[i] = L.norm_width[i];
    }
    return L.norm_g.size();
}

// CPU baseline: solve `n` roots with `threads` threads, one subgame per
// thread at a time (rayon over games in the reference). Returns node-updates
// (public nodes x iterations) in *node_updates.
int oracle_solve_many(const uint8_t* const* roots, const size_t* lens, size_t n, const OracleCfg* cfg,
                      const float* w, const float* b, const float* ln, int threads, double* node_updates) {
    std::vector<double> upd(n, 0.0);
    std::vector<std::thread> pool;
    std::atomic<size_t> next{0};
    Net net;
    if (w) {
        net.w.assign(w, w + net.L.w_len);
        net.b.assign(b, b + net.L.b_len);
        net.ln.assign(ln, ln + net.L.ln_len);
        net.empty = false;
    }
    wc::SolveCfg sc = to_cfg(cfg);
    for (int th = 0; th < threads; ++th)
        pool.emplace_back([&]() {
            for (;;) {
                size_t i = next.fetch_add(1);
                if (i >= n) return;
                wc::Root r;
                if (!wc::root_from_bytes(roots[i], lens[i], &r)) continue;
                auto t = wc::build_tree(r.s, r.ctx, sc, r.bel);
                Solver sv(*t, &net);
                sv.multistep(sc.iters);
                std::vector<std::vector<float>> rt(1);
                rt[0] = r.bel[0].p;
                rt[0].insert(rt[0].end(), r.bel[1].p.begin(), r.bel[1].p.end());
                sv.value_under(rt);
                upd[i] = (double)t->nodes.size() * (double)sc.iters;
            }
        });
    for (auto& th : pool) th.join();
    double s = 0.0;
    for (double x : upd) s += x;
    *node_updates = s;
    return 0;
}

// Bounded CPU baseline. Each of `threads` threads takes one subgame: it
// times the solver build plus the first k1 iterations (which includes the
// once-per-solve network pieces), then k2 more iterations, and projects the
// full solve as t1 + (iters - k1) * t2 / k2 plus one Phase-2 pass (about two
// iterations). out[0] = sum over subgames of nodes * iters / projected time
// (aggregate node-updates/s of `threads` busy threads), out[1] = measured
// wall seconds, out[2] = subgames sampled.
int oracle_bench(const uint8_t* const* roots, const size_t* lens, size_t n, const OracleCfg* cfg, const float* w,
                 const float* b, const float* ln, int threads, int k1, int k2, double* out) {
    Net net;
    if (w) {
        net.w.assign(w, w + net.L.w_len);
        net.b.assign(b, b + net.L.b_len);
        net.ln.assign(ln, ln + net.L.ln_len);
        net.empty = false;
    }
    wc::SolveCfg sc = to_cfg(cfg);
    wc::SolveCfg part = sc;
    size_t m = std::min<size_t>(n, (size_t)threads);
    std::vector<double> rate(m, 0.0);
    auto wall0 = std::chrono::steady_clock::now();
    std::vector<std::thread> pool;
    for (size_t i = 0; i < m; ++i)
        pool.emplace_back([&, i]() {
            wc::Root r;
            if (!wc::root_from_bytes(roots[i], lens[i], &r)) return;
            auto t0 = std::chrono::steady_clock::now();
            auto t = wc::build_tree(r.s, r.ctx, part, r.bel);
            Solver sv(*t, &net);
            sv.multistep(k1);
            auto t1 = std::chrono::steady_clock::now();
            sv.multistep(k2);
            auto t2 = std::chrono::steady_clock::now();
            double a = std::chrono::duration<double>(t1 - t0).count();
            double it = std::chrono::duration<double>(t2 - t1).count() / k2;
            double full = a + (sc.iters - k1) * it + 2.0 * it;
            rate[i] = (double)t->nodes.size() * sc.iters / full;
        });
    for (auto& th : pool) th.join();
    double sum = 0.0;
    for (double x : rate) sum += x;
    out[0] = sum;
    out[1] = std::chrono::duration<double>(std::chrono::steady_clock::now() - wall0).count();
    out[2] = (double)m;
    return 0;
}

}  // extern "C"
