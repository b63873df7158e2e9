// Public subgame tree construction (engine/src/search.rs:724-1462).
#include "tree.h"
#include "flatmap.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <stdexcept>

namespace wc {

CfrRule CfrRule::plus() {
    return {std::numeric_limits<float>::infinity(), -std::numeric_limits<float>::infinity(), 2.0f, 0.0f};
}
CfrRule CfrRule::pcfr() {
    return {std::numeric_limits<float>::infinity(), -std::numeric_limits<float>::infinity(), 2.0f, 1.0f};
}
CfrRule CfrRule::sapcfr() {
    return {std::numeric_limits<float>::infinity(), -std::numeric_limits<float>::infinity(), 2.0f, 1.0f / 3.0f};
}
bool CfrRule::named(const char* name, CfrRule* out) {
    if (!std::strcmp(name, "linear")) { *out = linear(); return true; }
    if (!std::strcmp(name, "plus")) { *out = plus(); return true; }
    if (!std::strcmp(name, "dcfr")) { *out = dcfr(); return true; }
    if (!std::strcmp(name, "pcfr")) { *out = pcfr(); return true; }
    if (!std::strcmp(name, "sapcfr")) { *out = sapcfr(); return true; }
    return false;
}

float cfr_factor(float t, float p) {
    if (std::isinf(p)) return p > 0.0f ? 1.0f : 0.0f;
    float x = std::pow(t, p);
    return x / (x + 1.0f);
}

std::vector<int> snapshot_iters(int iters) {
    std::vector<int> out;
    for (int t = 0; t <= iters; ++t)
        if (t == 0 || (t & (t - 1)) == 0 || t == iters) out.push_back(t);
    return out;
}

int Tree::max_depth() const {
    int m = 0;
    for (const NodeRec& n : nodes) m = std::max<int>(m, (int)n.depth);
    return m;
}

uint8_t action_coin(const Action& a, const State& s) {
    switch (a.kind) {
        case K_DEPLOY: case K_BOLSTER: case K_CLAIM: case K_RECRUIT: case K_PASS: case K_TAC_FOOTMAN:
            return a.a;
        case K_ROYALGUARD: return ROYAL_COIN;
        case K_ENSIGN: return ENSIGN;
        case K_MARSHAL: return MARSHAL;
        case K_MOVE: case K_CONTROL: case K_ATTACK: case K_ARCHER: case K_CAVMOVE: case K_CROSSBOW:
        case K_LANCER: case K_LIGHTCAV:
            return s.hex_type[a.a];
        default: return NONE;
    }
}

void node_actions(const State& s, uint8_t player, const Ctx& ctx, const std::vector<Config>& cfgs,
                  std::vector<Action>& acts, std::vector<int8_t>& aslot, std::vector<uint8_t>& fdown) {
    acts.clear(); aslot.clear(); fdown.clear();
    std::vector<uint32_t> seen;
    std::vector<Action> la;
    State probe = s;
    bool forced = s.pending.kind == C_WPPLAY;
    auto held = [&](int k) {
        for (const Config& c : cfgs)
            if (forced ? c.inflight == k : c.hand[k] > 0) return true;
        return false;
    };
    if (s.pending.kind == C_MAINPLAY || forced) {
        uint8_t res[NSLOT];
        reserve(s, player, ctx, res);
        for (int k = 0; k < NSLOT; ++k) {
            if (res[k] == 0) continue;
            if (!cfgs.empty() && !held(k)) continue;
            Config one;
            if (forced) one.inflight = (int8_t)k; else one.hand[k] = 1;
            set_config(probe, player, ctx, one);
            probe.legal_actions_into(la);
            for (const Action& a : la) {
                uint32_t key = a.encode();
                if (std::find(seen.begin(), seen.end(), key) != seen.end()) continue;
                seen.push_back(key);
                uint8_t coin = action_coin(a, probe);
                int slot = coin == NONE ? -1 : ctx.slot_of[player][coin];
                if (slot >= 0 && !cfgs.empty() && !held(slot)) continue;
                aslot.push_back((int8_t)slot);
                fdown.push_back(is_facedown_play(a) ? 1 : 0);
                acts.push_back(a);
            }
        }
    } else {
        s.legal_actions_into(la);
        for (const Action& a : la) {
            uint32_t key = a.encode();
            if (std::find(seen.begin(), seen.end(), key) != seen.end()) continue;
            seen.push_back(key);
            acts.push_back(a);
            aslot.push_back(-1);
            fdown.push_back(0);
        }
    }
}

namespace {

struct Builder {
    Tree& t;
    DrawScratch draw_scratch;
    FlatMap cmap;  // (player, config counts) -> interned config id
    // runs of interned ids already in leaf_cidx, by a hash of (configs,
    // player, reserve); run_index maps the hash to an entry of runs
    struct LeafRun {
        uint32_t sup, off;
        uint8_t p, res[NSLOT];
    };
    std::vector<LeafRun> runs;
    FlatMap run_index;
    static_assert(sizeof(Config) == 2 * NSLOT + 1, "configs compare bytewise: no padding");
    // draw transitions already in the tree, by a hash of their inputs (the
    // drawer's configs, reserve, face-up counts, steps, Warrior Priest draw):
    // the first node's rows start at t.draw_start[start_at]; its child's
    // support is out_sup
    struct DrawRun {
        uint32_t in_sup, out_sup, start_at;
        uint8_t res[NSLOT], fu[NSLOT], steps, wp;
    };
    std::vector<DrawRun> draw_runs;
    FlatMap draw_index;

    static bool same_configs(const std::vector<Config>& a, const std::vector<Config>& b) {
        return a.size() == b.size() && (a.data() == b.data() || std::memcmp(a.data(), b.data(), a.size() * sizeof(Config)) == 0);
    }
    std::vector<std::pair<uint64_t, uint32_t>> cell_order;
    std::vector<Config> adv;  // a decision node's successor config per cell

    explicit Builder(Tree& tree) : t(tree) {}

    uint32_t intern_config(const Config& c, const uint8_t* res, int p) {
        uint8_t cnt[CCOUNTS];
        config_counts(c, res, cnt);
        uint64_t key = (uint64_t)p;
        for (int k = 0; k < CCOUNTS; ++k) key = (key << 4) | cnt[k];
        if (const uint32_t* v = cmap.find(key)) return *v;
        uint32_t i = (uint32_t)t.ncfg++;
        for (int k = 0; k < CCOUNTS; ++k) t.cphi.push_back((float)cnt[k] / CNORM);
        t.cplayer.push_back((uint8_t)p);
        cmap.insert(key, i);
        return i;
    }

    // search.rs:1375-1425. The public row is packed at the leaf; the configs'
    // interning waits for the end of the build (finish_leaves, in leaf order,
    // so the ids are those of interning at each leaf) and is skipped for a
    // tree that hits the node cap, which is never solved.
    struct PendingLeaf {
        uint32_t sup[2];
        uint8_t res[2][NSLOT];
    };
    std::vector<PendingLeaf> pending;

    void push_leaf(uint32_t id, const State& s, const uint32_t sup[2]) {
        if (s.is_terminal()) {
            t.term_leaves.push_back(id);
            return;
        }
        size_t at = t.gpu_rows.size();
        t.gpu_rows.resize(at + GPU_ROW_BYTES);
        pack_gpu_row(s, t.ctx, t.gpu_rows.data() + at);
        PendingLeaf pl;
        for (int p = 0; p < 2; ++p) {
            pl.sup[p] = sup[p];
            reserve(s, (uint8_t)p, t.ctx, pl.res[p]);
        }
        pending.push_back(pl);
        t.leaf_rows.push_back(id);
    }

    // A leaf's config ids depend only on its configs, the player and the
    // player's reserve, and nearly every leaf repeats an earlier leaf's three
    // (the same configs reached along other public paths): such a leaf copies
    // that leaf's run, found by a hash and confirmed field by field. Every
    // config of a copied run is interned already, so no id is assigned out of
    // the first-seen order.
    void finish_leaves() {
        for (const PendingLeaf& pl : pending)
            for (int p = 0; p < 2; ++p) intern_leaf(pl.sup, pl.res[p], p);
        pending.clear();
    }

    void intern_leaf(const uint32_t sup[2], const uint8_t* res, int p) {
        const size_t base = t.leaf_cidx.size();
        t.leaf_coff.push_back((uint32_t)base);
        const std::vector<Config>& cfgs = t.supports[sup[p]];
        uint64_t h = FlatMap::mix(((uint64_t)p << 40) | ((uint64_t)res[0] << 32) | ((uint64_t)res[1] << 24) |
                                  ((uint64_t)res[2] << 16) | ((uint64_t)res[3] << 8) | res[4]);
        for (const Config& c : cfgs) h = FlatMap::mix(h ^ c.key());
        if (h == FlatMap::FREE) h = 0;
        const uint32_t* e = run_index.find(h);
        if (e) {
            const LeafRun& r = runs[*e];
            const std::vector<Config>& prev = t.supports[r.sup];
            if (r.p == p && std::memcmp(r.res, res, NSLOT) == 0 && prev.size() == cfgs.size() &&
                (r.sup == sup[p] || std::memcmp(prev.data(), cfgs.data(), cfgs.size() * sizeof(Config)) == 0)) {
                t.leaf_cidx.resize(base + cfgs.size());
                std::copy(t.leaf_cidx.begin() + r.off, t.leaf_cidx.begin() + r.off + cfgs.size(),
                          t.leaf_cidx.begin() + base);
                return;
            }
        }
        for (const Config& c : cfgs) t.leaf_cidx.push_back(intern_config(c, res, p));
        if (!e) {  // (a hash taken by other contents keeps its first run)
            LeafRun r{sup[p], (uint32_t)base, (uint8_t)p, {}};
            std::memcpy(r.res, res, NSLOT);
            run_index.insert(h, (uint32_t)runs.size());
            runs.push_back(r);
        }
    }

    uint32_t push_support(std::vector<Config>&& v) {
        t.supports.push_back(std::move(v));
        return (uint32_t)(t.supports.size() - 1);
    }

    // search.rs:942-1253.
    uint32_t build(const State& s, int depth, const uint32_t sup_in[2], uint32_t level) {
        uint8_t player = s.to_act();
        bool draw_pass = s.pending.kind == C_DRAW || s.pending.kind == C_WPDRAW;
        bool mainplay = s.pending.kind == C_MAINPLAY;
        bool leaf = s.is_terminal();
        if (!leaf && !draw_pass && depth == 0) leaf = mainplay;
        uint32_t id = (uint32_t)t.nodes.size();
        NodeRec nr;
        std::memset(&nr, 0, sizeof nr);
        nr.util = (leaf && s.is_terminal()) ? s.utility(player) : 0.0f;
        nr.player = player;
        nr.kind = leaf ? NK_LEAF : NK_DECISION;
        nr.terminal = (leaf && s.is_terminal()) ? 1 : 0;
        nr.sup[0] = sup_in[0];
        nr.sup[1] = sup_in[1];
        nr.act_off = (uint32_t)t.acts.size();
        nr.child_off = (uint32_t)t.child.size();
        nr.obs_off = (uint32_t)t.obs_start.size();
        nr.row_off = (uint32_t)t.legal_off.size();
        nr.aoff_off = (uint32_t)t.action_off.size();
        nr.draw_off = (uint32_t)t.draw_start.size();
        nr.depth = level;
        t.nodes.push_back(nr);
        if (t.cfg.keep_states) t.states.push_back(s);
        t.soff.push_back((uint32_t)t.legal_action.size());
        if (t.cfg.node_cap > 0 && t.nodes.size() >= t.cfg.node_cap) {
            t.capped = true;
            return id;
        }
        if (leaf) {
            push_leaf(id, s, sup_in);
            return id;
        }

        if (draw_pass) {
            int me = player;
            State cs = s;
            uint8_t res[NSLOT], fu[NSLOT];
            reserve(cs, player, t.ctx, res);
            faceup_counts(cs, player, t.ctx, fu);
            bool wp = s.pending.kind == C_WPDRAW;
            uint8_t steps = 0;
            for (;;) {
                int unit = cs.first_drawable(player);
                cs.apply_inplace(Action::make(K_DRAW, unit < 0 ? NONE : (uint8_t)unit));
                steps += 1;
                if (!(cs.pending.kind == C_DRAW && cs.to_act() == player)) break;
            }
            // the same inputs give the same transition (rebel.rs:570-771 read
            // nothing else): a repeat copies the first node's rows and child
            // support, found by a hash and confirmed field by field
            const std::vector<Config>& in = t.supports[sup_in[me]];
            uint64_t h = FlatMap::mix(((uint64_t)steps << 1) | (wp ? 1u : 0u));
            for (int k = 0; k < NSLOT; ++k) h = FlatMap::mix(h ^ ((uint64_t)res[k] << 8 | fu[k]));
            for (const Config& c : in) h = FlatMap::mix(h ^ c.key());
            if (h == FlatMap::FREE) h = 0;
            const uint32_t* e = draw_index.find(h);
            const DrawRun* hit = nullptr;
            if (e) {
                const DrawRun& r = draw_runs[*e];
                if (r.steps == steps && r.wp == (wp ? 1 : 0) && std::memcmp(r.res, res, NSLOT) == 0 &&
                    std::memcmp(r.fu, fu, NSLOT) == 0 && same_configs(t.supports[r.in_sup], in))
                    hit = &r;
            }
            const uint32_t start_at = (uint32_t)t.draw_start.size();
            uint32_t base = (uint32_t)t.draw_to.size();
            std::vector<Config> support;
            if (hit) {
                const uint32_t b0 = t.draw_start[hit->start_at], rows = (uint32_t)in.size();
                for (uint32_t r = 0; r <= rows; ++r) {
                    const uint32_t x = t.draw_start[hit->start_at + r] - b0;
                    t.draw_start.push_back(base + x);
                }
                const uint32_t n = t.draw_start.back() - base;
                t.draw_to.resize(base + n);
                std::copy(t.draw_to.begin() + b0, t.draw_to.begin() + b0 + n, t.draw_to.begin() + base);
                t.draw_p.resize(base + n);
                std::copy(t.draw_p.begin() + b0, t.draw_p.begin() + b0 + n, t.draw_p.begin() + base);
                support = t.supports[hit->out_sup];
            } else {
                DrawMap draw;
                if (wp) draw_scratch.transition(in, res, fu, support, draw, true);
                else draw_scratch.run(in, res, fu, steps, support, draw);
                // store the map: rows + 1 global offsets
                for (uint32_t x : draw.start) t.draw_start.push_back(base + x);
                t.draw_to.insert(t.draw_to.end(), draw.to.begin(), draw.to.end());
                t.draw_p.insert(t.draw_p.end(), draw.p.begin(), draw.p.end());
            }
            t.child.push_back(0);
            t.nodes[id].kind = NK_CHANCE;
            t.nodes[id].nch = 1;
            t.nodes[id].draw_steps = steps;
            uint32_t cc[2] = {sup_in[0], sup_in[1]};
            const uint32_t in_sup = sup_in[me];
            cc[me] = push_support(std::move(support));
            if (!hit && !e) {  // (a hash taken by other inputs keeps its first transition)
                DrawRun r{in_sup, cc[me], start_at, {}, {}, steps, (uint8_t)(wp ? 1 : 0)};
                std::memcpy(r.res, res, NSLOT);
                std::memcpy(r.fu, fu, NSLOT);
                draw_index.insert(h, (uint32_t)draw_runs.size());
                draw_runs.push_back(r);
            }
            uint32_t ch = build(cs, depth, cc, level + 1);
            t.child[t.nodes[id].child_off] = ch;
            return id;
        }

        int me = player;
        const std::vector<Config>& mine0 = t.supports[sup_in[me]];
        std::vector<Config> mine = mine0;  // supports may reallocate during recursion
        size_t nc = mine.size();
        std::vector<Action> acts;
        std::vector<int8_t> aslot;
        std::vector<uint8_t> fdown;
        node_actions(s, player, t.ctx, mine, acts, aslot, fdown);
        uint32_t na = (uint32_t)acts.size();
        if (na == 0) throw std::logic_error("a decision node must offer a reachable action");

        // legal cells, config-major
        uint32_t cell0 = (uint32_t)t.legal_action.size();
        t.legal_off.push_back(0);
        for (size_t ci = 0; ci < nc; ++ci) {
            for (uint32_t a = 0; a < na; ++a) {
                if (action_legal(mine[ci], aslot[a])) {
                    t.legal_action.push_back(a);
                    t.legal_child.push_back(0);
                    t.legal_trans.push_back(NO_TRANS);
                    t.cell_row.push_back((uint32_t)ci);
                }
            }
            t.legal_off.push_back((uint32_t)(t.legal_action.size() - cell0));
        }
        uint32_t ncell = (uint32_t)t.legal_action.size() - cell0;

        // observation grouping (first appearance order)
        std::vector<uint32_t> obs_keys;
        std::vector<uint32_t> obs_child(na);
        for (uint32_t a = 0; a < na; ++a) {
            uint32_t k = obs_key(acts[a]);
            auto it = std::find(obs_keys.begin(), obs_keys.end(), k);
            if (it == obs_keys.end()) { obs_keys.push_back(k); obs_child[a] = (uint32_t)obs_keys.size() - 1; }
            else obs_child[a] = (uint32_t)(it - obs_keys.begin());
        }
        uint32_t nch = (uint32_t)obs_keys.size();
        std::vector<uint32_t> obs_start(nch + 1, 0);
        for (uint32_t a = 0; a < na; ++a) obs_start[obs_child[a] + 1] += 1;
        for (uint32_t ch = 0; ch < nch; ++ch) obs_start[ch + 1] += obs_start[ch];
        std::vector<uint32_t> fill(obs_start.begin(), obs_start.end() - 1);
        std::vector<uint32_t> obs_act(na);
        for (uint32_t a = 0; a < na; ++a) obs_act[fill[obs_child[a]]++] = a;

        for (uint32_t cell = 0; cell < ncell; ++cell)
            t.legal_child[cell0 + cell] = obs_child[t.legal_action[cell0 + cell]];
        std::vector<uint32_t> action_off(na + 1, 0);
        for (uint32_t cell = 0; cell < ncell; ++cell) action_off[t.legal_action[cell0 + cell] + 1] += 1;
        for (uint32_t a = 0; a < na; ++a) action_off[a + 1] += action_off[a];
        std::vector<uint32_t> afill(action_off.begin(), action_off.end() - 1);
        std::vector<uint32_t> action_cell(ncell);
        for (uint32_t cell = 0; cell < ncell; ++cell) action_cell[afill[t.legal_action[cell0 + cell]]++] = cell;

        // child supports, by sorted config key (search.rs:1164-1197); each
        // cell's successor config is computed once (adv, by cell)
        std::vector<std::vector<Config>> child_cfgs(nch);
        adv.resize(ncell);
        for (uint32_t ch = 0; ch < nch; ++ch) {
            cell_order.clear();
            for (uint32_t j = obs_start[ch]; j < obs_start[ch + 1]; ++j) {
                uint32_t a = obs_act[j];
                for (uint32_t x = action_off[a]; x < action_off[a + 1]; ++x) {
                    uint32_t cell = action_cell[x];
                    if (t.legal_child[cell0 + cell] != ch) continue;
                    uint32_t ci = t.cell_row[cell0 + cell];
                    if (advance_config(mine[ci], aslot[a], fdown[a], &adv[cell])) cell_order.emplace_back(adv[cell].key(), cell);
                }
            }
            std::sort(cell_order.begin(), cell_order.end());
            std::vector<Config>& sup = child_cfgs[ch];
            uint64_t prev = ~0ull;
            for (auto& kc : cell_order) {
                uint32_t cell = kc.second;
                if (kc.first != prev) {
                    prev = kc.first;
                    sup.push_back(adv[cell]);
                }
                t.legal_trans[cell0 + cell] = (uint32_t)(sup.size() - 1);
            }
        }

        // write the node's flat arrays before its children are built
        NodeRec& n = t.nodes[id];
        n.na = na;
        n.nch = nch;
        t.acts.insert(t.acts.end(), acts.begin(), acts.end());
        t.aslot.insert(t.aslot.end(), aslot.begin(), aslot.end());
        t.fdown.insert(t.fdown.end(), fdown.begin(), fdown.end());
        t.obs_child.insert(t.obs_child.end(), obs_child.begin(), obs_child.end());
        t.obs_start.insert(t.obs_start.end(), obs_start.begin(), obs_start.end());
        t.obs_act.insert(t.obs_act.end(), obs_act.begin(), obs_act.end());
        t.action_off.insert(t.action_off.end(), action_off.begin(), action_off.end());
        t.action_cell.insert(t.action_cell.end(), action_cell.begin(), action_cell.end());
        uint32_t child_off = (uint32_t)t.child.size();
        t.child.resize(child_off + nch, 0);

        bool spends = s.pending.kind == C_MAINPLAY;
        for (uint32_t ch = 0; ch < nch; ++ch) {
            uint32_t a = obs_act[obs_start[ch]];
            const Config* rep = nullptr;
            for (const Config& c : mine)
                if (action_legal(c, aslot[a])) { rep = &c; break; }
            if (!rep) throw std::logic_error("a kept action is playable by some config in the support");
            State cs = s;
            set_config(cs, player, t.ctx, *rep);
            cs.apply_inplace(acts[a]);
            uint32_t cc[2] = {sup_in[0], sup_in[1]};
            cc[me] = push_support(std::move(child_cfgs[ch]));
            uint32_t cid = build(cs, depth - (spends ? 1 : 0), cc, level + 1);
            t.child[child_off + ch] = cid;
        }
        for (uint32_t cell = 0; cell < ncell; ++cell)
            t.legal_child[cell0 + cell] = t.child[child_off + t.legal_child[cell0 + cell]];
        return id;
    }
};

}  // namespace

std::unique_ptr<Tree> build_tree(const State& root, const Ctx& ctx, const SolveCfg& cfg, const Belief bel[2]) {
    auto t = std::make_unique<Tree>();
    t->ctx = ctx;
    t->cfg = cfg;
    t->root_belief[0] = bel[0];
    t->root_belief[1] = bel[1];
    for (int view = 0; view < 2; ++view)
        for (int ty = 0; ty < NTYPE; ++ty) {
            int physical = view == 0 ? ty / NSLOT : 1 - ty / NSLOT;
            t->ids[view][ty] = ctx.slots[physical][ty % NSLOT];
        }
    Builder b(*t);
    uint32_t sup[2];
    sup[0] = b.push_support(std::vector<Config>(bel[0].cfg));
    sup[1] = b.push_support(std::vector<Config>(bel[1].cfg));
    b.build(root, std::max(cfg.depth, 1), sup, 0);
    if (!t->capped) b.finish_leaves();
    t->soff.push_back((uint32_t)t->legal_action.size());
    t->leaf_coff.push_back((uint32_t)t->leaf_cidx.size());
    return t;
}

}  // namespace wc
