// Continual re-solving walk (engine/src/selfplay.rs:466-905).
#include "walk.h"

#include <cstring>
#include <stdexcept>

namespace wc {

std::shared_ptr<const WalkTree> WalkTree::from(const Tree& t) {
    auto w = std::make_shared<WalkTree>();
    const size_t n = t.nodes.size();
    w->kind.resize(n);
    w->player.resize(n);
    w->draw_steps.resize(n);
    w->row_off.resize(n);
    w->act_off.resize(n);
    w->na.resize(n);
    w->child_off.resize(n);
    w->nch.resize(n);
    w->sup.resize(2 * n);
    for (size_t i = 0; i < n; ++i) {
        const NodeRec& r = t.nodes[i];
        w->kind[i] = r.kind;
        w->player[i] = r.player;
        w->draw_steps[i] = r.draw_steps;
        w->row_off[i] = r.row_off;
        w->act_off[i] = r.act_off;
        w->na[i] = r.na;
        w->child_off[i] = r.child_off;
        w->nch[i] = r.nch;
        w->sup[2 * i] = r.sup[0];
        w->sup[2 * i + 1] = r.sup[1];
    }
    w->soff = t.soff;
    w->legal_off = t.legal_off;
    w->obs_child = t.obs_child;
    w->child = t.child;
    w->supports = t.supports;
    return w;
}

namespace {

// IEEE binary16 -> binary32 (exact: every half is a float).
float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal: man * 2^-24
            float m = (float)man * (1.0f / 16777216.0f);
            std::memcpy(&bits, &m, 4);
            bits |= sign;
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// client.rs:78-92: decode, then normalise to sum 1 when the sum is positive.
void decode_probability(const uint16_t* src, size_t n, std::vector<float>& out) {
    size_t at = out.size();
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        out.push_back(half_to_float(src[i]));
        sum += out.back();
    }
    if (sum > 0.0f)
        for (size_t i = 0; i < n; ++i) out[at + i] /= sum;
}

bool same_support(const std::vector<Config>& a, const std::vector<Config>& b) {
    return a.size() == b.size() && std::equal(a.begin(), a.end(), b.begin());
}

}  // namespace

Game::Game(uint64_t seed, bool random_draft, const SolveCfg& cfg) : rng_(seed), cfg_(cfg) {
    s_ = make_game(rng_, random_draft);
    ctx_ = Ctx::make(s_);
    bel_[0] = Belief::point(Config());
    bel_[1] = Belief::point(Config());
    cfg_.snapshots = true;
}

Game::Game(const Root& root, uint64_t seed, const SolveCfg& cfg) : rng_(seed), cfg_(cfg) {
    s_ = root.s;
    ctx_ = root.ctx;
    bel_[0] = root.bel[0];
    bel_[1] = root.bel[1];
    cfg_.snapshots = true;
}

// finish_walk (selfplay.rs:466-488) with CarryStore::select (client.rs:
// 41-58): the exit node's beliefs under every kept per-iterate average but
// the last, then the live belief, as the next subgame's carried roots.
void Game::end_walk() {
    const WalkTree& t = *tree_;
    if (res_.cpu_carried) {
        carried_.clear();
        std::vector<std::vector<float>> v = res_.cpu_carried(node_);
        for (const auto& x : v) carried_.insert(carried_.end(), x.begin(), x.end());
        carried_.insert(carried_.end(), bel_[0].p.begin(), bel_[0].p.end());
        carried_.insert(carried_.end(), bel_[1].p.begin(), bel_[1].p.end());
        ncarried_ = (uint32_t)v.size() + 1;
        walking_ = false;
        tree_.reset();
        res_ = WalkResult();
        if (max_solves_ && solves_ >= (int64_t)max_solves_) stopped_ = true;
        return;
    }
    size_t e = 0;
    while (e < res_.exit_nodes.size() && res_.exit_nodes[e] != node_) ++e;
    if (e == res_.exit_nodes.size()) throw std::logic_error("carry store has no exit node " + std::to_string(node_));
    const size_t n0 = t.support(node_, 0).size(), n1 = t.support(node_, 1).size();
    if (res_.carry_off[e + 1] - res_.carry_off[e] != n0 + n1) throw std::logic_error("carry row does not fit its node");
    carried_.clear();
    for (uint32_t sn = 0; sn < res_.carry_snapshots; ++sn) {
        const uint16_t* row = res_.carries.data() + (size_t)sn * res_.carry_width + res_.carry_off[e];
        decode_probability(row, n0, carried_);
        decode_probability(row + n0, n1, carried_);
    }
    carried_.insert(carried_.end(), bel_[0].p.begin(), bel_[0].p.end());
    carried_.insert(carried_.end(), bel_[1].p.begin(), bel_[1].p.end());
    ncarried_ = res_.carry_snapshots + 1;
    walking_ = false;
    tree_.reset();
    if (max_solves_ && solves_ >= (int64_t)max_solves_) stopped_ = true;
}

// Game::advance (selfplay.rs:588-905) with both seats ReBeL agents that
// collect (snapshots on), no exploration.
Game::Step Game::advance() {
    if (pending_) throw std::logic_error("a solve is pending: resume first");
    while (!s_.is_terminal() && !stopped_) {
        const uint8_t player = s_.to_act();
        if (s_.is_chance()) {
            uint8_t res[NSLOT], fu[NSLOT];
            reserve(s_, player, ctx_, res);
            faceup_counts(s_, player, ctx_, fu);
            const bool wp = s_.pending.kind == C_WPDRAW;
            bel_[player] = belief_after_draw(bel_[player], res, fu, wp);
            resolve_chance(s_, player, rng_);
            if (walking_) {
                const WalkTree& t = *tree_;
                if (t.kind[node_] != NK_CHANCE || t.player[node_] != player) throw std::logic_error("walk not at the draw");
                ++walk_draws_;
                if (++drawn_ == t.draw_steps[node_]) {
                    drawn_ = 0;
                    const uint32_t child = t.child[t.child_off[node_]];
                    if (!same_support(t.support(child, player), bel_[player].cfg))
                        throw std::logic_error("walk desync: post-draw support does not match the game belief");
                    node_ = child;
                    if (t.kind[child] == NK_LEAF) end_walk();
                }
            }
            continue;
        }
        const std::vector<Config> cfgs = bel_[player].cfg;
        const int true_ci = bel_[player].index_of(true_config(s_, player, ctx_));
        if (true_ci < 0) throw std::logic_error("belief filter dropped the true config");
        ++decisions_;
        NodePolicy np;
        if (!walking_) {
            // a new subgame at this decision (selfplay.rs:683-756)
            auto tree = build_tree(s_, ctx_, cfg_, bel_);
            if (tree->capped) {
                carried_.clear();
                ncarried_ = 0;
                ++capped_;
                np = NodePolicy::uniform(s_, ctx_, player, cfgs);
            } else {
                if (ncarried_ == 0) {
                    pending_roots_ = bel_[0].p;
                    pending_roots_.insert(pending_roots_.end(), bel_[1].p.begin(), bel_[1].p.end());
                    pending_nroots_ = 1;
                } else {
                    pending_roots_ = std::move(carried_);
                    pending_nroots_ = ncarried_;
                    carried_.clear();
                    ncarried_ = 0;
                }
                pending_walk_ = WalkTree::from(*tree);
                pending_ = std::move(tree);
                --decisions_;  // counted again when the walk plays it
                return NEED_SOLVE;
            }
        } else {
            const WalkTree& t = *tree_;
            if (t.player[node_] != player || !same_support(t.support(node_, player), cfgs))
                throw std::logic_error("walk desync: subgame tree no longer matches the game belief");
            np = NodePolicy::frame(s_, ctx_, player, cfgs);
            if (np.acts.size() != t.na[node_]) throw std::logic_error("walk desync: the node's actions differ");
            // act on the CFR average: the strategy rows of this node
            for (size_t ci = 0; ci < cfgs.size(); ++ci) {
                const uint32_t lo = t.legal_off[t.row_off[node_] + ci], hi = t.legal_off[t.row_off[node_] + ci + 1];
                if (hi - lo != np.legal_off[ci + 1] - np.legal_off[ci])
                    throw std::logic_error("walk desync: a legal row differs from the tree's");
                std::memcpy(np.probs.data() + np.legal_off[ci], res_.strategy.data() + t.soff[node_] + lo,
                            4 * (size_t)(hi - lo));
            }
            ++walk_decisions_;
        }
        const size_t chosen_cell = np.sample(rng_, (size_t)true_ci);
        const uint32_t chosen = np.legal_action[chosen_cell];
        bel_[player] = np.posterior(bel_[player], obs_key(np.acts[chosen]));
        s_.apply_inplace(np.acts[chosen]);
        if (walking_) {
            node_ = tree_->child_for_action(node_, chosen);
            if (tree_->kind[node_] == NK_LEAF) end_walk();
        }
    }
    return ENDED;
}

// Game::resume (selfplay.rs:907-946): the walk starts at the subgame root.
void Game::resume(const WalkResult& r) {
    if (!pending_walk_) throw std::logic_error("no solve is pending");
    tree_ = std::move(pending_walk_);
    pending_.reset();
    pending_roots_.clear();
    pending_nroots_ = 0;
    res_ = r;
    if (res_.strategy.size() != tree_->soff.back()) throw std::logic_error("the strategy does not fit the subgame");
    walking_ = true;
    node_ = 0;
    drawn_ = 0;
    ++solves_;
}

void Game::counters(int64_t* out) const {
    out[0] = decisions_;
    out[1] = solves_;
    out[2] = capped_;
    out[3] = walk_decisions_;
    out[4] = walk_draws_;
    out[5] = (s_.is_terminal() || stopped_) ? 1 : 0;
    out[6] = s_.winner == NONE ? -1 : (int64_t)s_.winner;
    out[7] = walking_ ? 1 : 0;
}

}  // namespace wc
