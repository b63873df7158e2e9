// Seeded root generation (selfplay.rs / policy.rs of the reference).
#include "roots.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <stdexcept>

namespace wc {

// selfplay.rs:45-52.
static const uint16_t STARTER_WHITE[4] = {17, 12, 4, 9};
static const uint16_t STARTER_BLACK[4] = {1, 3, 8, 16};
static const uint16_t DRAFT_POOL[19] = {1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 16, 17, 18, 19, 52, 53, 54};

// selfplay.rs:59-81.
State make_game(Rng& rng, bool random_draft) {
    uint8_t first = (rng.next_u64() & 1) == 0 ? WHITE : BLACK;
    if (!random_draft) return State::from_draft(STARTER_WHITE, STARTER_BLACK, first);
    uint16_t pool[19];
    std::memcpy(pool, DRAFT_POOL, sizeof pool);
    for (size_t i = 18; i >= 1; --i) {
        size_t j = rng.below(i + 1);
        uint16_t tmp = pool[i]; pool[i] = pool[j]; pool[j] = tmp;
    }
    return State::from_draft(pool, pool + 4, first);
}

// policy.rs:41-63.
NodePolicy NodePolicy::frame(const State& s, const Ctx& ctx, uint8_t player, const std::vector<Config>& cfgs) {
    NodePolicy np;
    node_actions(s, player, ctx, cfgs, np.acts, np.aslot, np.fdown);
    size_t na = np.acts.size();
    np.legal_off.push_back(0);
    for (const Config& c : cfgs) {
        for (size_t a = 0; a < na; ++a)
            if (action_legal(c, np.aslot[a])) np.legal_action.push_back((uint32_t)a);
        np.legal_off.push_back((uint32_t)np.legal_action.size());
    }
    np.probs.assign(np.legal_action.size(), 0.0f);
    return np;
}

// policy.rs:127-139.
NodePolicy NodePolicy::uniform(const State& s, const Ctx& ctx, uint8_t player, const std::vector<Config>& cfgs) {
    NodePolicy np = frame(s, ctx, player, cfgs);
    for (size_t ci = 0; ci < cfgs.size(); ++ci) {
        uint32_t lo = np.legal_off[ci], hi = np.legal_off[ci + 1];
        float k = (float)(hi - lo);
        for (uint32_t cell = lo; cell < hi; ++cell) np.probs[cell] = 1.0f / k;
    }
    return np;
}

// policy.rs:79-90.
size_t NodePolicy::sample(Rng& rng, size_t c) const {
    uint32_t lo = legal_off[c], hi = legal_off[c + 1];
    std::vector<double> w;
    double tot = 0.0;
    for (uint32_t cell = lo; cell < hi; ++cell) {
        double x = probs[cell] > 0.0f ? (double)probs[cell] : 0.0;
        w.push_back(x);
        tot += x;
    }
    if (tot > 0.0) return lo + rng.weighted_index(w.data(), w.size());
    return lo + rng.below(w.size() > 0 ? w.size() : 1);
}

// policy.rs:95-109.
Belief NodePolicy::posterior(const Belief& prior, uint32_t obs) const {
    std::vector<std::pair<Config, float>> pairs;
    for (size_t ci = 0; ci < prior.cfg.size(); ++ci) {
        for (uint32_t cell = legal_off[ci]; cell < legal_off[ci + 1]; ++cell) {
            uint32_t a = legal_action[cell];
            if (obs_key(acts[a]) != obs) continue;
            Config next;
            if (advance_config(prior.cfg[ci], aslot[a], fdown[a] != 0, &next))
                pairs.emplace_back(next, prior.p[ci] * probs[cell]);
        }
    }
    return Belief::from_pairs(std::move(pairs));
}

// selfplay.rs:1148-1156.
static uint8_t effective_bag_count(const State& s, uint8_t p, uint8_t unit) {
    int bag_total = 0;
    for (int u = 0; u < N_UNITS; ++u) bag_total += s.zones[p][Z_BAG][u];
    if (bag_total > 0) return s.zones[p][Z_BAG][unit];
    return (uint8_t)(s.zones[p][Z_FACEUP][unit] + s.zones[p][Z_FACEDOWN][unit]);
}

// selfplay.rs:1124-1146.
void resolve_chance(State& s, uint8_t player, Rng& rng) {
    std::vector<Action> acts = s.legal_actions();
    std::vector<double> w;
    bool any = false;
    for (const Action& a : acts) {
        int c = (a.kind == K_DRAW && a.a != NONE) ? effective_bag_count(s, player, a.a) : 1;
        any |= c > 0;
        w.push_back((double)c);
    }
    if (!any)
        for (double& x : w) x = 1.0;
    Action drawn = acts[rng.weighted_index(w.data(), w.size())];
    s.apply_inplace(drawn);
}

bool make_root(uint64_t seed, int plies, bool random_draft, Root* out) {
    Rng rng(seed);
    State s = make_game(rng, random_draft);
    Ctx ctx = Ctx::make(s);
    Belief bel[2] = {Belief::point(Config()), Belief::point(Config())};
    int decisions = 0;
    while (!s.is_terminal()) {
        uint8_t player = s.to_act();
        if (s.is_chance()) {
            uint8_t res[NSLOT], fu[NSLOT];
            reserve(s, player, ctx, res);
            faceup_counts(s, player, ctx, fu);
            bool wp = s.pending.kind == C_WPDRAW;
            bel[player] = belief_after_draw(bel[player], res, fu, wp);
            resolve_chance(s, player, rng);
            continue;
        }
        if (decisions >= plies && s.pending.kind == C_MAINPLAY) {
            out->s = s;
            out->ctx = ctx;
            out->bel[0] = bel[0];
            out->bel[1] = bel[1];
            return true;
        }
        const std::vector<Config>& cfgs = bel[player].cfg;
        int true_ci = bel[player].index_of(true_config(s, player, ctx));
        if (true_ci < 0) throw std::logic_error("belief filter dropped the true config");
        NodePolicy np = NodePolicy::uniform(s, ctx, player, cfgs);
        size_t cell = np.sample(rng, (size_t)true_ci);
        uint32_t chosen = np.legal_action[cell];
        bel[player] = np.posterior(bel[player], obs_key(np.acts[chosen]));
        s.apply_inplace(np.acts[chosen]);
        ++decisions;
    }
    return false;
}

Belief uniform_belief(const State& s, const Ctx& ctx, uint8_t p) {
    uint8_t res[NSLOT];
    reserve(s, p, ctx, res);
    Config truth = true_config(s, p, ctx);
    Belief b;
    b.cfg = enumerate_configs(res, truth.hand_size(), truth.fd_size(), truth.inflight >= 0);
    float n = (float)b.cfg.size();
    b.p.assign(b.cfg.size(), 1.0f / n);
    return b;
}

bool make_wide_root(uint64_t seed, int plies, bool random_draft, uint32_t ncfg, Root* out) {
    if (!make_root(seed, plies, random_draft, out)) return false;
    Rng rng(seed ^ 0x5EEDB17EF0C0FFEEull);  // a stream of its own, apart from the game's
    for (int p = 0; p < 2; ++p) {
        Belief all = uniform_belief(out->s, out->ctx, (uint8_t)p);
        std::vector<Config>& c = all.cfg;
        // the true config first, then a partial Fisher-Yates draw of the rest
        const int ti = all.index_of(true_config(out->s, (uint8_t)p, out->ctx));
        if (ti > 0) std::swap(c[0], c[(size_t)ti]);
        const size_t k = std::max<size_t>(1, std::min<size_t>(ncfg, c.size()));
        for (size_t i = 1; i < k; ++i) std::swap(c[i], c[i + rng.below(c.size() - i)]);
        std::vector<double> e(k);
        double tot = 0.0;
        for (size_t i = 0; i < k; ++i) {
            e[i] = -std::log(1.0 - rng.unit_f64());  // unit exponential; 1 - u is in (0, 1]
            tot += e[i];
        }
        std::vector<std::pair<Config, float>> pairs;
        pairs.reserve(k);
        for (size_t i = 0; i < k; ++i) pairs.emplace_back(c[i], (float)(e[i] / tot));
        out->bel[p] = Belief::from_pairs(std::move(pairs));
    }
    return true;
}

std::vector<uint8_t> root_to_bytes(const Root& r) {
    std::vector<uint8_t> out(sizeof(State));
    std::memcpy(out.data(), &r.s, sizeof(State));
    for (int p = 0; p < 2; ++p) {
        uint32_t n = (uint32_t)r.bel[p].cfg.size();
        const uint8_t* np = reinterpret_cast<const uint8_t*>(&n);
        out.insert(out.end(), np, np + 4);
        for (const Config& c : r.bel[p].cfg) {
            out.insert(out.end(), c.hand, c.hand + NSLOT);
            out.insert(out.end(), c.fd, c.fd + NSLOT);
            out.push_back((uint8_t)c.inflight);
        }
        const uint8_t* wp = reinterpret_cast<const uint8_t*>(r.bel[p].p.data());
        out.insert(out.end(), wp, wp + 4 * n);
    }
    return out;
}

bool root_from_bytes(const uint8_t* data, size_t n, Root* out) {
    if (n < sizeof(State)) return false;
    std::memcpy(&out->s, data, sizeof(State));
    size_t at = sizeof(State);
    for (int p = 0; p < 2; ++p) {
        if (at + 4 > n) return false;
        uint32_t cnt;
        std::memcpy(&cnt, data + at, 4);
        at += 4;
        if (at + (size_t)cnt * 11 > n) return false;
        out->bel[p].cfg.resize(cnt);
        for (uint32_t i = 0; i < cnt; ++i) {
            Config& c = out->bel[p].cfg[i];
            std::memcpy(c.hand, data + at, NSLOT);
            std::memcpy(c.fd, data + at + NSLOT, NSLOT);
            c.inflight = (int8_t)data[at + 2 * NSLOT];
            at += 11;
        }
        if (at + (size_t)cnt * 4 > n) return false;
        out->bel[p].p.resize(cnt);
        std::memcpy(out->bel[p].p.data(), data + at, (size_t)cnt * 4);
        at += (size_t)cnt * 4;
    }
    try {
        out->ctx = Ctx::make(out->s);
    } catch (...) {
        return false;
    }
    return at == n;
}

}  // namespace wc
