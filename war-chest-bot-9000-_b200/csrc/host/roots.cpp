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

// ------------------------------------------------------------ root bytes
// The reference's root encoding, format v3 (engine/src/roots.rs:247-313,
// write_root / read_root): the State field by field in little-endian
// (write_state, roots.rs:150-180), then per player u32 n, n configs
// (hand[5], fd[5], inflight or 0xff) and n f32 weights. Cont tags and
// payloads follow write_cont (roots.rs:49-104); the Cont kinds here are
// numbered as those tags.

namespace {

struct Writer {
    std::vector<uint8_t>& out;
    void u8(uint8_t x) { out.push_back(x); }
    void u32(uint32_t x) { for (int i = 0; i < 4; ++i) out.push_back((uint8_t)(x >> (8 * i))); }
    void u64(uint64_t x) { for (int i = 0; i < 8; ++i) out.push_back((uint8_t)(x >> (8 * i))); }
    void f32(float x) { uint32_t u; std::memcpy(&u, &x, 4); u32(u); }
};

struct Reader {
    const uint8_t* p;
    size_t n, at = 0;
    bool ok = true;
    bool need(size_t k) { if (!ok || at + k > n) ok = false; return ok; }
    uint8_t u8() { if (!need(1)) return 0; return p[at++]; }
    uint32_t u32() {
        if (!need(4)) return 0;
        uint32_t x = 0;
        for (int i = 0; i < 4; ++i) x |= (uint32_t)p[at + i] << (8 * i);
        at += 4;
        return x;
    }
    uint64_t u64() {
        if (!need(8)) return 0;
        uint64_t x = 0;
        for (int i = 0; i < 8; ++i) x |= (uint64_t)p[at + i] << (8 * i);
        at += 8;
        return x;
    }
    float f32() { uint32_t u = u32(); float x; std::memcpy(&x, &u, 4); return x; }
};

void write_cont(Writer& w, const Cont& c) {
    w.u8(c.kind);
    switch (c.kind) {
        case C_MAINPLAY: break;
        case C_RGCHOICE: case C_WPDRAW: w.u8(c.a); w.u8(c.b); break;
        case C_BERSCHAIN: w.u8(c.a); w.u8(c.b ? 1 : 0); break;
        case C_FOOTMAN: w.u64(c.hexes); break;
        default: w.u8(c.a); break;  // Draw, SwordsmanMove, CavalryAttack, Mercenary, FID, WPPlay, _AttackPost
    }
}

bool read_cont(Reader& r, Cont* c) {
    const uint8_t tag = r.u8();
    if (tag > C_ATKPOST) return false;
    *c = Cont::make(tag);
    switch (tag) {
        case C_MAINPLAY: break;
        case C_RGCHOICE: case C_WPDRAW: c->a = r.u8(); c->b = r.u8(); break;
        case C_BERSCHAIN: c->a = r.u8(); c->b = r.u8() != 0 ? 1 : 0; break;
        case C_FOOTMAN: c->hexes = r.u64(); break;
        default: c->a = r.u8(); break;
    }
    return r.ok;
}

}  // namespace

// Every index a State carries is in range: units < N_UNITS, hexes <
// N_HEXES, players 0 / 1 (NONE where the field allows it). The engine indexes
// tables with these fields unchecked, so bytes from outside are checked once
// here.
bool state_in_range(const State& s) {
    auto unit = [](uint8_t u) { return u < N_UNITS; };
    auto hex = [](uint8_t h) { return h < N_HEXES; };
    auto player = [](uint8_t p) { return p < 2; };
    for (int h = 0; h < N_HEXES; ++h) {
        const bool empty = s.hex_type[h] == NONE;
        if (!empty && (!unit(s.hex_type[h]) || !player(s.hex_owner[h]))) return false;
        if (empty && s.hex_owner[h] != NONE) return false;
        if (s.loc_marker[h] != NONE && !player(s.loc_marker[h])) return false;
    }
    if (!player(s.initiative) || !player(s.first_player) || !player(s.active)) return false;
    if (s.winner != NONE && !player(s.winner)) return false;
    auto cont_ok = [&](const Cont& c) {
        switch (c.kind) {
            case C_MAINPLAY: return true;
            case C_DRAW: case C_WPPLAY: return player(c.a);
            case C_RGCHOICE: return player(c.a) && hex(c.b);
            case C_WPDRAW: return player(c.a) && (c.b == NONE || hex(c.b));
            case C_BERSCHAIN: return hex(c.a);
            case C_FOOTMAN: return (c.hexes >> N_HEXES) == 0;
            case C_FID: return unit(c.a);
            default: return hex(c.a);  // SwordsmanMove, CavalryAttack, Mercenary, _AttackPost
        }
    };
    if (!cont_ok(s.pending)) return false;
    for (int i = 0; i < s.conts.n; ++i)
        if (!cont_ok(s.conts.v[i])) return false;
    return true;
}

bool action_well_formed(const State& s, const Action& a) {
    auto unit = [](uint8_t u) { return u < N_UNITS; };
    auto hex = [](uint8_t h) { return h < N_HEXES; };
    auto unit_at = [&](uint8_t h) { return hex(h) && s.hex_type[h] != NONE; };
    switch (a.kind) {
        case K_DEPLOY: case K_BOLSTER: return unit(a.a) && hex(a.b);
        case K_CLAIM: case K_PASS: case K_TAC_FOOTMAN: return unit(a.a);
        case K_RECRUIT: return unit(a.a) && unit(a.b);
        case K_DRAW: return a.a == NONE || unit(a.a);
        case K_RG_SUPPLY: case K_RG_STACK: case K_SWORD_DECLINE: case K_BERS_STOP: case K_MERC_DECLINE:
        case K_FID_DECLINE: return true;
        case K_FID_DEPLOY: return hex(a.a);
        case K_CONTROL: case K_FOOTCTRL: case K_BERS_CTRL: case K_MERC_CTRL: case K_GRANT_CTRL: return unit_at(a.a);
        case K_LANCER: return unit_at(a.a) && hex(a.b) && hex(a.c);
        default: return unit_at(a.a) && hex(a.b);  // the two-hex maneuvers, attacks and tactics
    }
}

void write_state(std::vector<uint8_t>& out, const State& s) {
    Writer w{out};
    for (int h = 0; h < N_HEXES; ++h) {
        w.u8(s.hex_type[h]);
        w.u8(s.hex_owner[h]);
        w.u8(s.hex_height[h]);
        w.u8(s.loc_marker[h]);
    }
    for (int p = 0; p < N_PLAYERS; ++p)
        for (int z = 0; z < N_ZONES; ++z)
            for (int u = 0; u < N_UNITS; ++u) w.u8(s.zones[p][z][u]);
    w.u8(s.markers_hand[0]);
    w.u8(s.markers_hand[1]);
    w.u8(s.initiative);
    w.u8(s.initiative_moved ? 1 : 0);
    w.u32(s.round);
    w.u8(s.first_player);
    w.u8(s.active);
    w.u8(s.turns_taken[0]);
    w.u8(s.turns_taken[1]);
    w.u32(s.main_plays);
    w.u8(s.winner);
    w.u8(s.adjudicated_draw ? 1 : 0);
    write_cont(w, s.pending);
    w.u8(s.conts.n);
    for (int i = (int)s.conts.n - 1; i >= 0; --i) write_cont(w, s.conts.v[i]);  // pop order: top first
    w.u8(s.wp_v2_triggered ? 1 : 0);
    w.u8(s.interrupt ? 1 : 0);
}

bool read_state(const uint8_t* data, size_t n, size_t* at, State* out) {
    Reader r{data, n, *at};
    State s = State::blank(0);
    for (int h = 0; h < N_HEXES; ++h) {
        s.hex_type[h] = r.u8();
        s.hex_owner[h] = r.u8();
        s.hex_height[h] = r.u8();
        s.loc_marker[h] = r.u8();
    }
    for (int p = 0; p < N_PLAYERS; ++p)
        for (int z = 0; z < N_ZONES; ++z)
            for (int u = 0; u < N_UNITS; ++u) s.zones[p][z][u] = r.u8();
    s.markers_hand[0] = r.u8();
    s.markers_hand[1] = r.u8();
    s.initiative = r.u8();
    s.initiative_moved = r.u8() != 0;
    s.round = (uint16_t)r.u32();
    s.first_player = r.u8();
    s.active = r.u8();
    s.turns_taken[0] = r.u8();
    s.turns_taken[1] = r.u8();
    s.main_plays = (uint16_t)r.u32();
    s.winner = r.u8();
    s.adjudicated_draw = r.u8() != 0;
    if (!read_cont(r, &s.pending)) return false;
    const uint8_t nc = r.u8();
    if (!r.ok || nc > CONT_CAP) return false;
    Cont items[CONT_CAP];
    for (int i = 0; i < nc; ++i)
        if (!read_cont(r, &items[i])) return false;
    s.conts.clear();
    for (int i = (int)nc - 1; i >= 0; --i) s.conts.push(items[i]);  // written top first
    s.wp_v2_triggered = r.u8() != 0;
    s.interrupt = r.u8() != 0;
    if (!r.ok || !state_in_range(s)) return false;
    *out = s;
    *at = r.at;
    return true;
}

std::vector<uint8_t> root_to_bytes(const Root& r) {
    std::vector<uint8_t> out;
    write_state(out, r.s);
    Writer w{out};
    for (int p = 0; p < 2; ++p) {
        const Belief& b = r.bel[p];
        w.u32((uint32_t)b.cfg.size());
        for (const Config& c : b.cfg) {
            for (int k = 0; k < NSLOT; ++k) w.u8(c.hand[k]);
            for (int k = 0; k < NSLOT; ++k) w.u8(c.fd[k]);
            w.u8(c.inflight < 0 ? 0xff : (uint8_t)c.inflight);
        }
        for (float x : b.p) w.f32(x);
    }
    return out;
}

bool root_from_bytes(const uint8_t* data, size_t n, Root* out, size_t* used) {
    size_t at = 0;
    if (!read_state(data, n, &at, &out->s)) return false;
    Reader r{data, n, at};
    for (int p = 0; p < 2; ++p) {
        const uint32_t cnt = r.u32();
        if (!r.ok || cnt > 100000 || (size_t)cnt * 15 > n - r.at) return false;  // read_root's bound
        Belief& b = out->bel[p];
        b.cfg.resize(cnt);
        for (uint32_t i = 0; i < cnt; ++i) {
            Config& c = b.cfg[i];
            for (int k = 0; k < NSLOT; ++k) c.hand[k] = r.u8();
            for (int k = 0; k < NSLOT; ++k) c.fd[k] = r.u8();
            const uint8_t f = r.u8();
            c.inflight = f == 0xff ? (int8_t)-1 : (int8_t)f;
        }
        b.p.resize(cnt);
        for (uint32_t i = 0; i < cnt; ++i) b.p[i] = r.f32();
        if (!r.ok) return false;
    }
    try {
        out->ctx = Ctx::make(out->s);
    } catch (...) {
        return false;
    }
    // a coin in flight is in none (0xff) or one of the five slots: the builder
    // indexes a config's slots by it (read_root takes any other byte as a slot
    // index, which its indexing then refuses). Counts beyond the player's
    // coins are left as read_root leaves them: a root may carry a stale belief.
    for (int p = 0; p < 2; ++p)
        for (const Config& c : out->bel[p].cfg)
            if (c.inflight < -1 || c.inflight >= NSLOT) return false;
    if (used) {
        *used = r.at;
        return true;
    }
    return r.at == n;
}

bool roots_file_split(const uint8_t* data, size_t n, std::vector<std::pair<size_t, size_t>>* spans) {
    Reader r{data, n};
    if (r.u32() != ROOTS_MAGIC || r.u32() != ROOTS_VERSION) return false;
    const uint32_t count = r.u32();
    if (!r.ok) return false;
    spans->clear();
    size_t at = r.at;
    for (uint32_t i = 0; i < count; ++i) {
        Root tmp;
        size_t used = 0;
        if (!root_from_bytes(data + at, n - at, &tmp, &used)) return false;
        spans->emplace_back(at, used);
        at += used;
    }
    return at == n;
}

}  // namespace wc
