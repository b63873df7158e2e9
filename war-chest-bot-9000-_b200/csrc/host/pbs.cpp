// Public belief states, restating engine/src/rebel.rs of the reference.
#include "pbs.h"

#include <algorithm>
#include <cstring>
#include <stdexcept>

namespace wc {

// rebel.rs:87-103.
Ctx Ctx::make(const State& s) {
    Ctx c;
    for (int p = 0; p < 2; ++p) {
        for (int u = 0; u < N_UNITS; ++u) c.slot_of[p][u] = -1;
        int n = 0;
        for (int u = 0; u < N_UNITS; ++u) {
            if (s.total_coins((uint8_t)p, u) > 0) {
                if (n >= NSLOT) throw std::invalid_argument("a player may own at most 5 coin types");
                c.slots[p][n] = (uint8_t)u;
                c.slot_of[p][u] = (int8_t)n;
                ++n;
            }
        }
        if (n != NSLOT) throw std::invalid_argument("expected exactly 5 coin types per player");
    }
    return c;
}

Ctx Ctx::mirrored() const {
    Ctx m;
    for (int k = 0; k < NSLOT; ++k) { m.slots[0][k] = slots[1][k]; m.slots[1][k] = slots[0][k]; }
    for (int u = 0; u < N_UNITS; ++u) { m.slot_of[0][u] = slot_of[1][u]; m.slot_of[1][u] = slot_of[0][u]; }
    return m;
}

// rebel.rs:184-191.
void config_counts(const Config& c, const uint8_t* res, uint8_t* out) {
    for (int k = 0; k < NSLOT; ++k) {
        int inflight = c.inflight == k ? 1 : 0;
        out[k] = c.hand[k];
        out[NSLOT + k] = c.fd[k];
        int used = c.hand[k] + c.fd[k] + inflight;
        out[2 * NSLOT + k] = res[k] > used ? (uint8_t)(res[k] - used) : 0;
    }
}

// rebel.rs:208-218.
void reserve(const State& s, uint8_t p, const Ctx& ctx, uint8_t* out) {
    for (int k = 0; k < NSLOT; ++k) {
        int u = ctx.slots[p][k];
        out[k] = (uint8_t)(s.zones[p][Z_BAG][u] + s.zones[p][Z_HAND][u] + s.zones[p][Z_FACEDOWN][u] +
                           s.zones[p][Z_INFLIGHT][u]);
    }
}

void faceup_counts(const State& s, uint8_t p, const Ctx& ctx, uint8_t* out) {
    for (int k = 0; k < NSLOT; ++k) out[k] = s.zones[p][Z_FACEUP][ctx.slots[p][k]];
}

Config true_config(const State& s, uint8_t p, const Ctx& ctx) {
    Config c;
    for (int k = 0; k < NSLOT; ++k) {
        int u = ctx.slots[p][k];
        c.hand[k] = s.zones[p][Z_HAND][u];
        c.fd[k] = s.zones[p][Z_FACEDOWN][u];
        if (s.zones[p][Z_INFLIGHT][u] > 0) c.inflight = (int8_t)k;
    }
    return c;
}

// rebel.rs:239-261.
void set_config(State& s, uint8_t p, const Ctx& ctx, const Config& c) {
    for (int k = 0; k < NSLOT; ++k) {
        int u = ctx.slots[p][k];
        uint8_t inflight = c.inflight == k ? 1 : 0;
        uint8_t res = (uint8_t)(s.zones[p][Z_BAG][u] + s.zones[p][Z_HAND][u] + s.zones[p][Z_FACEDOWN][u] +
                                s.zones[p][Z_INFLIGHT][u]);
        s.zones[p][Z_HAND][u] = c.hand[k];
        s.zones[p][Z_FACEDOWN][u] = c.fd[k];
        s.zones[p][Z_INFLIGHT][u] = inflight;
        s.zones[p][Z_BAG][u] = (uint8_t)(res - c.hand[k] - c.fd[k] - inflight);
    }
}

// rebel.rs:270-345.
std::vector<Config> enumerate_configs(const uint8_t* res, uint8_t hand_size, uint8_t fd_size, bool inflight) {
    std::vector<Config> out;
    uint8_t hand[NSLOT] = {0, 0, 0, 0, 0};
    uint8_t fd[NSLOT] = {0, 0, 0, 0, 0};
    auto push = [&](int8_t infl) {
        Config c;
        for (int k = 0; k < NSLOT; ++k) { c.hand[k] = hand[k]; c.fd[k] = fd[k]; }
        c.inflight = infl;
        out.push_back(c);
    };
    auto rec_fd = [&](auto&& self, int k, int left) -> void {
        if (k == NSLOT - 1) {
            if (left + hand[k] <= res[k]) {
                fd[k] = (uint8_t)left;
                if (inflight) {
                    for (int s = 0; s < NSLOT; ++s)
                        if (hand[s] + fd[s] < res[s]) push((int8_t)s);
                } else {
                    push(-1);
                }
                fd[k] = 0;
            }
            return;
        }
        int lim = res[k] > hand[k] ? res[k] - hand[k] : 0;
        lim = std::min(lim, left);
        for (int t = 0; t <= lim; ++t) {
            fd[k] = (uint8_t)t;
            self(self, k + 1, left - t);
        }
        fd[k] = 0;
    };
    auto rec_hand = [&](auto&& self, int k, int left) -> void {
        if (k == NSLOT - 1) {
            if (left <= res[k]) {
                hand[k] = (uint8_t)left;
                for (int i = 0; i < NSLOT; ++i) fd[i] = 0;
                rec_fd(rec_fd, 0, fd_size);
                hand[k] = 0;
            }
            return;
        }
        int lim = std::min<int>(left, res[k]);
        for (int t = 0; t <= lim; ++t) {
            hand[k] = (uint8_t)t;
            self(self, k + 1, left - t);
        }
        hand[k] = 0;
    };
    rec_hand(rec_hand, 0, hand_size);
    return out;
}

// rebel.rs:377-399. Duplicates merge in a stable order (the reference uses an
// unstable sort; only the ulp-level sum of duplicate weights can differ).
Belief Belief::from_pairs(std::vector<std::pair<Config, float>> pairs) {
    std::stable_sort(pairs.begin(), pairs.end(),
                     [](const std::pair<Config, float>& x, const std::pair<Config, float>& y) {
                         return x.first.key() < y.first.key();
                     });
    Belief b;
    b.cfg.reserve(pairs.size());
    b.p.reserve(pairs.size());
    for (auto& pr : pairs) {
        if (pr.second < 0.0f) continue;
        if (!b.cfg.empty() && b.cfg.back() == pr.first) {
            b.p.back() += pr.second;
        } else {
            b.cfg.push_back(pr.first);
            b.p.push_back(pr.second);
        }
    }
    b.normalize();
    return b;
}

// rebel.rs:401-413.
void Belief::normalize() {
    float s = 0.0f;
    for (float v : p) s += v;
    if (s > SMOOTH) {
        for (float& v : p) v /= s;
    } else {
        float n = (float)std::max<size_t>(p.size(), 1);
        for (float& v : p) v = 1.0f / n;
    }
}

int Belief::index_of(const Config& c) const {
    auto it = std::lower_bound(cfg.begin(), cfg.end(), c);
    if (it != cfg.end() && *it == c) return (int)(it - cfg.begin());
    return -1;
}

// rebel.rs:425-430.
bool action_legal(const Config& c, int slot) {
    if (c.inflight >= 0) return slot == c.inflight;
    return slot < 0 || c.hand[slot] > 0;
}

// rebel.rs:440-465.
bool advance_config(const Config& c, int slot, bool facedown, Config* out) {
    if (c.inflight >= 0) {
        int k = c.inflight;
        if (slot != k) return false;
        Config n = c;
        n.inflight = -1;
        if (facedown) n.fd[k] += 1;
        *out = n;
        return true;
    }
    if (slot < 0) { *out = c; return true; }
    if (c.hand[slot] == 0) return false;
    Config n = c;
    n.hand[slot] -= 1;
    if (facedown) n.fd[slot] += 1;
    *out = n;
    return true;
}

// rebel.rs:831-843.
static void draw_source(const Config& c, const uint8_t* res, const uint8_t* faceup, uint8_t* src, Config* base) {
    uint8_t bag[NSLOT];
    c.bag(res, bag);
    bool any = false;
    for (int k = 0; k < NSLOT; ++k) any |= bag[k] > 0;
    if (any) {
        for (int k = 0; k < NSLOT; ++k) src[k] = bag[k];
        *base = c;
        return;
    }
    for (int k = 0; k < NSLOT; ++k) src[k] = (uint8_t)(faceup[k] + c.fd[k]);
    *base = c;
    for (int k = 0; k < NSLOT; ++k) base->fd[k] = 0;
}

// rebel.rs:474-506.
Belief belief_after_draw(const Belief& b, const uint8_t* res, const uint8_t* faceup, bool set_pending) {
    std::vector<std::pair<Config, float>> pairs;
    pairs.reserve(b.size() * NSLOT);
    for (size_t i = 0; i < b.size(); ++i) {
        const Config& c = b.cfg[i];
        float w = b.p[i];
        uint8_t src[NSLOT];
        Config base;
        draw_source(c, res, faceup, src, &base);
        uint32_t total = 0;
        for (int k = 0; k < NSLOT; ++k) total += src[k];
        if (total == 0) { pairs.emplace_back(c, w); continue; }
        for (int k = 0; k < NSLOT; ++k) {
            if (src[k] == 0) continue;
            Config n = base;
            if (set_pending) {
                n.inflight = (int8_t)k;
                pairs.emplace_back(n, w * (float)src[k] / (float)total);
            } else {
                n.hand[k] += 1;
                if (n.hand_size() <= HAND_CAP) pairs.emplace_back(n, w * (float)src[k] / (float)total);
            }
        }
    }
    return Belief::from_pairs(std::move(pairs));
}

// rebel.rs:570-615.
void DrawScratch::transition(const std::vector<Config>& cfg, const uint8_t* res, const uint8_t* faceup,
                             std::vector<Config>& support, DrawMap& map, bool set_pending) {
    kid.clear();
    prob.clear();
    map.start.clear();
    map.start.push_back(0);
    for (const Config& c : cfg) {
        uint8_t src[NSLOT];
        Config base;
        draw_source(c, res, faceup, src, &base);
        uint32_t total = 0;
        for (int k = 0; k < NSLOT; ++k) total += src[k];
        if (total == 0) {
            kid.push_back(c);
            prob.push_back(1.0f);
        } else {
            float inv = 1.0f / (float)total;
            for (int k = 0; k < NSLOT; ++k) {
                if (src[k] == 0) continue;
                Config n = base;
                if (set_pending) {
                    n.inflight = (int8_t)k;
                    kid.push_back(n);
                    prob.push_back((float)src[k] * inv);
                } else {
                    n.hand[k] += 1;
                    if (n.hand_size() <= HAND_CAP) {
                        kid.push_back(n);
                        prob.push_back((float)src[k] * inv);
                    }
                }
            }
        }
        map.start.push_back((uint32_t)kid.size());
    }
    pack(support, map);
}

// rebel.rs:629-685.
void DrawScratch::run(const std::vector<Config>& cfg, const uint8_t* res, const uint8_t* faceup, uint8_t k8,
                      std::vector<Config>& support, DrawMap& map) {
    kid.clear();
    prob.clear();
    map.start.clear();
    map.start.push_back(0);
    uint32_t k = k8;
    for (const Config& c : cfg) {
        uint8_t bag[NSLOT];
        c.bag(res, bag);
        uint32_t b = 0;
        for (int s = 0; s < NSLOT; ++s) b += bag[s];
        if (b >= k) {
            deal(bag, k, c);
        } else {
            Config base = c;
            for (int s = 0; s < NSLOT; ++s) base.hand[s] += bag[s];
            uint8_t r[NSLOT];
            uint32_t rt = 0;
            for (int s = 0; s < NSLOT; ++s) { r[s] = (uint8_t)(faceup[s] + c.fd[s]); rt += r[s]; }
            uint32_t left = k - b;
            if (rt == 0) {
                kid.push_back(base);
                prob.push_back(1.0f);
            } else {
                for (int s = 0; s < NSLOT; ++s) base.fd[s] = 0;
                if (rt <= left) {
                    for (int s = 0; s < NSLOT; ++s) base.hand[s] += r[s];
                    kid.push_back(base);
                    prob.push_back(1.0f);
                } else {
                    deal(r, left, base);
                }
            }
        }
        map.start.push_back((uint32_t)kid.size());
    }
    pack(support, map);
}

// rebel.rs:690-738: every way to draw k coins from src, hypergeometric weight,
// computed in f64 as a product of (n - i) / (i + 1) factors.
static double choose(uint32_t n, uint32_t k) {
    double r = 1.0;
    for (uint32_t i = 0; i < k; ++i) r *= (double)(n - i) / (double)(i + 1);
    return r;
}

// Slot by slot, x coins from this slot for x ascending; `take` packs the
// coins taken so far (byte s: slot s). Only the counts that leave no more
// coins than the later slots hold are visited (suf[s]: coins in slots s..):
// the other branches deal nothing, so the dealt hands, their order and their
// products are those of the full enumeration.
static void deal_rec(const uint8_t* src, const uint32_t* suf, int slot, uint32_t left, double num, uint64_t take,
                     double denom, std::vector<uint64_t>& out, std::vector<float>& prob) {
    if (slot == NSLOT) {
        out.push_back(take);
        prob.push_back((float)(num / denom));
        return;
    }
    const uint32_t hi = std::min<uint32_t>(left, src[slot]);
    const uint32_t lo = left > suf[slot + 1] ? left - suf[slot + 1] : 0;
    for (uint32_t x = lo; x <= hi; ++x)
        deal_rec(src, suf, slot + 1, left - x, num * choose(src[slot], x), take | ((uint64_t)x << (8 * slot)), denom,
                 out, prob);
}

// The hands of a (source, k) pair depend on nothing else: each pair is
// enumerated once per scratch and its hands are added to every base config
// that draws from it.
void DrawScratch::deal(const uint8_t* src, uint32_t k, const Config& base) {
    uint64_t key = k;
    for (int s = 0; s < NSLOT; ++s) key = (key << 8) | src[s];
    uint32_t entry;
    if (const uint32_t* e = deal_index.find(key)) {
        entry = *e;
    } else {
        uint32_t suf[NSLOT + 1];
        suf[NSLOT] = 0;
        for (int s = NSLOT - 1; s >= 0; --s) suf[s] = suf[s + 1] + src[s];
        const uint32_t first = (uint32_t)deal_take.size();
        if (k <= suf[0])  // else no hand: more coins than the source holds
            deal_rec(src, suf, 0, k, 1.0, 0, choose(suf[0], k), deal_take, deal_p);
        entry = (uint32_t)deal_span.size();
        deal_span.emplace_back(first, (uint32_t)deal_take.size() - first);
        deal_index.insert(key, entry);
    }
    const auto [first, n] = deal_span[entry];
    for (uint32_t i = first; i < first + n; ++i) {
        Config c = base;
        const uint64_t take = deal_take[i];
        for (int s = 0; s < NSLOT; ++s) c.hand[s] = (uint8_t)(c.hand[s] + (uint8_t)(take >> (8 * s)));
        kid.push_back(c);
        prob.push_back(deal_p[i]);
    }
}

// rebel.rs:743-771.
void DrawScratch::pack(std::vector<Config>& support, DrawMap& map) {
    constexpr uint32_t IDX_BITS = 24;
    if (kid.size() >= (1u << IDX_BITS)) throw std::runtime_error("draw fan-out over the index width");
    order.clear();
    order.reserve(kid.size());
    for (size_t i = 0; i < kid.size(); ++i) order.push_back((kid[i].key() << IDX_BITS) | (uint64_t)i);
    std::sort(order.begin(), order.end());
    support.clear();
    map.to.assign(kid.size(), 0);
    map.p.assign(prob.begin(), prob.end());
    uint64_t prev = ~0ull;
    for (uint64_t packed : order) {
        uint64_t key = packed >> IDX_BITS;
        size_t i = (size_t)(packed & ((1ull << IDX_BITS) - 1));
        if (key != prev) {
            prev = key;
            support.push_back(kid[i]);
        }
        map.to[i] = (uint32_t)(support.size() - 1);
    }
}

// rebel.rs:777-812.
void DrawScratch::compose(const DrawMap& a, const DrawMap& b, size_t n_child, DrawMap& out) {
    if (acc.size() < n_child) { acc.resize(n_child, 0.0f); hit.resize(n_child, 0); }
    size_t rows = a.rows();
    out.start.clear(); out.start.push_back(0);
    out.to.clear(); out.p.clear();
    for (size_t i = 0; i < rows; ++i) {
        touched.clear();
        for (uint32_t m = a.start[i]; m < a.start[i + 1]; ++m) {
            uint32_t mid = a.to[m];
            float pm = a.p[m];
            for (uint32_t j = b.start[mid]; j < b.start[mid + 1]; ++j) {
                uint32_t t = b.to[j];
                if (!hit[t]) { hit[t] = 1; touched.push_back(t); }
                acc[t] += pm * b.p[j];
            }
        }
        std::sort(touched.begin(), touched.end());
        for (uint32_t t : touched) {
            out.to.push_back(t);
            out.p.push_back(acc[t]);
            acc[t] = 0.0f;
            hit[t] = 0;
        }
        out.start.push_back((uint32_t)out.to.size());
    }
}

bool is_facedown_play(const Action& a) {
    return a.kind == K_PASS || a.kind == K_CLAIM || a.kind == K_RECRUIT;
}

// rebel.rs:868-875.
uint32_t obs_key(const Action& a) {
    uint32_t code = a.encode();
    if (a.kind == K_PASS || a.kind == K_CLAIM) return code & 63u;
    if (a.kind == K_RECRUIT) return (code & 63u) | ((uint32_t)a.b << 12);
    return code;
}

// rebel.rs:1054-1068.
void normalize_weights(const float* w, size_t n, float* out) {
    float tot = 0.0f;
    for (size_t i = 0; i < n; ++i) tot += w[i];
    float scale, flat;
    if (tot > SMOOTH) { scale = 1.0f / tot; flat = 0.0f; }
    else { scale = 0.0f; flat = 1.0f / (float)std::max<size_t>(n, 1); }
    for (size_t i = 0; i < n; ++i) out[i] = w[i] * scale + flat;
}

// rebel.rs:1274-1306.
// rebel.rs:996-1030: FNV-1a over the tables the expansion depends on (the
// location map, every unit's card facts as f32 bits, the layout constants),
// each mixed in as one u64.
uint64_t rules_table_hash() {
    uint64_t h = 0xcbf29ce484222325ull;
    auto mix = [&](uint64_t x) { h = (h ^ x) * 0x100000001b3ull; };
    const Board& bd = board();
    for (int k = 0; k < N_HEXES; ++k) mix(bd.is_location[k] ? 1u : 0u);
    for (int u = 0; u < N_UNITS; ++u) {
        float f[CARD_FEATS];
        write_card_features((uint8_t)u, f);
        for (float x : f) {
            uint32_t bits;
            std::memcpy(&bits, &x, 4);
            mix(bits);
        }
    }
    for (int c : {PUBFEAT, HEX_FACTS, HEX_CH, CARD_FEATS, NSLOT, NTYPE, N_HEXES, PILE_COUNTS, LOOSE}) mix((uint64_t)c);
    return h;
}

// rebel.rs:1236-1268: the replay row of a live state.
void pack_row(const State& s, const Ctx& ctx, uint8_t* out) {
    const uint32_t version = ROW_FORMAT_VERSION;
    const uint64_t hash = rules_table_hash();
    for (int k = 0; k < 4; ++k) out[ROW_VERSION + k] = (uint8_t)(version >> (8 * k));
    for (int k = 0; k < 8; ++k) out[ROW_HASH + k] = (uint8_t)(hash >> (8 * k));
    for (int t = 0; t < 2 * NSLOT; ++t) out[ROW_IDS + t] = ctx.slots[t / NSLOT][t % NSLOT];
    for (int h = 0; h < N_HEXES; ++h) {
        out[ROW_HEX_OWNER + h] = s.hex_owner[h];
        out[ROW_HEX_SLOT + h] = s.hex_owner[h] == NONE ? NONE : (uint8_t)ctx.slot_of[s.hex_owner[h]][s.hex_type[h]];
        out[ROW_HEX_HEIGHT + h] = s.hex_height[h];
        out[ROW_HEX_MARKER + h] = s.loc_marker[h];
    }
    for (int p = 0; p < 2; ++p) {
        uint8_t res[NSLOT];
        reserve(s, (uint8_t)p, ctx, res);
        for (int k = 0; k < NSLOT; ++k) {
            const int u = ctx.slots[p][k], at = ROW_PILES + (p * NSLOT + k) * PILE_COUNTS;
            out[at] = res[k];
            out[at + 1] = s.zones[p][Z_FACEUP][u];
            out[at + 2] = s.zones[p][Z_SUPPLY][u];
            out[at + 3] = s.zones[p][Z_ELIM][u];
        }
    }
    out[ROW_INITIATIVE] = s.initiative;
    out[ROW_INIT_MOVED] = s.initiative_moved ? 1 : 0;
    out[ROW_TO_ACT] = s.to_act();
    const uint16_t plies = (uint16_t)(MAX_MAIN_PLAYS - std::min<uint16_t>(s.main_plays, MAX_MAIN_PLAYS));
    out[ROW_PLIES] = (uint8_t)(plies & 0xff);
    out[ROW_PLIES + 1] = (uint8_t)(plies >> 8);
}

void pack_gpu_row(const State& s, const Ctx& ctx, uint8_t* out) {
    for (int h = 0; h < N_HEXES; ++h) {
        out[GPU_ROW_HEX_OWNER + h] = s.hex_owner[h];
        out[GPU_ROW_HEX_SLOT + h] =
            s.hex_owner[h] == NONE ? NONE : (uint8_t)ctx.slot_of[s.hex_owner[h]][s.hex_type[h]];
        out[GPU_ROW_HEX_HEIGHT + h] = s.hex_height[h];
        out[GPU_ROW_HEX_MARKER + h] = s.loc_marker[h];
    }
    for (int p = 0; p < 2; ++p) {
        uint8_t res[NSLOT];
        reserve(s, (uint8_t)p, ctx, res);
        for (int k = 0; k < NSLOT; ++k) {
            int u = ctx.slots[p][k];
            int at = GPU_ROW_PILES + (p * NSLOT + k) * PILE_COUNTS;
            out[at] = res[k];
            out[at + 1] = s.zones[p][Z_FACEUP][u];
            out[at + 2] = s.zones[p][Z_SUPPLY][u];
            out[at + 3] = s.zones[p][Z_ELIM][u];
        }
        out[GPU_ROW_MARKERS + p] = s.markers_hand[p];
        out[GPU_ROW_HAND + p] = s.hand_size((uint8_t)p);
        uint8_t fd = 0;
        for (int u = 0; u < N_UNITS; ++u) fd += s.zones[p][Z_FACEDOWN][u];
        out[GPU_ROW_FD + p] = fd;
        out[GPU_ROW_BAG + p] = s.bag_size((uint8_t)p);
    }
    out[GPU_ROW_INITIATIVE] = s.initiative;
    out[GPU_ROW_INIT_MOVED] = s.initiative_moved ? 1 : 0;
    out[GPU_ROW_TO_ACT] = s.to_act();
    uint16_t plies = (uint16_t)(MAX_MAIN_PLAYS - std::min<uint16_t>(s.main_plays, MAX_MAIN_PLAYS));
    out[GPU_ROW_PLIES] = (uint8_t)(plies & 0xff);
    out[GPU_ROW_PLIES + 1] = (uint8_t)(plies >> 8);
}

// rebel.rs:1144-1233: the shared core of the public encoding.
static void write_public_features_raw(const uint8_t* hex_owner, const uint8_t* hex_slot, const uint8_t* hex_height,
                                      const uint8_t* hex_marker, const uint8_t* piles, const uint8_t* ids,
                                      const uint8_t* markers_hand, const uint8_t* hand_size, const uint8_t* fd_size,
                                      const uint8_t* bag_size, uint8_t initiative, bool initiative_moved,
                                      uint8_t to_act, uint16_t plies_remaining, float* out) {
    for (int i = 0; i < PUBFEAT; ++i) out[i] = 0.0f;
    const Board& bd = board();
    int i = 0;
    for (int h = 0; h < N_HEXES; ++h) {
        uint8_t owner = hex_owner[h];
        if (owner != NONE) {
            out[i + owner] = 1.0f;
            out[i + 2] = (float)hex_height[h] / 5.0f;
            if (hex_slot[h] != NONE) out[i + HEX_FACTS + owner * NSLOT + hex_slot[h]] = 1.0f;
        }
        if (hex_marker[h] != NONE) out[i + 3 + hex_marker[h]] = 1.0f;
        out[i + 5] = bd.is_location[h] ? 1.0f : 0.0f;
        i += HEX_CH;
    }
    for (int t = 0; t < NTYPE; ++t) {
        int at = t * PILE_COUNTS;
        for (int j = 0; j < 4; ++j) out[i + j] = (float)piles[at + j] / 5.0f;
        i += PILE_COUNTS;
    }
    for (int t = 0; t < NTYPE; ++t) {
        write_card_features(ids[t], out + i);
        i += CARD_FEATS;
    }
    for (int p = 0; p < 2; ++p) {
        out[i] = (float)markers_hand[p] / 6.0f;
        out[i + 1] = (float)(6 - markers_hand[p]) / 6.0f;
        out[i + 2] = (float)hand_size[p] / 3.0f;
        out[i + 3] = (float)fd_size[p] / MAX_COINS;
        out[i + 4] = (float)bag_size[p] / MAX_COINS;
        out[i + 5] = initiative == p ? 1.0f : 0.0f;
        i += PLAYER_SCALARS;
    }
    out[i] = (float)plies_remaining / (float)MAX_MAIN_PLAYS;
    out[i + 1] = initiative_moved ? 1.0f : 0.0f;
    out[i + 2] = to_act == 0 ? 1.0f : 0.0f;
}

// rebel.rs:1311-1346.
void expand_gpu_row(const uint8_t* row, const uint8_t* ids, float* out) {
    uint16_t plies = (uint16_t)(row[GPU_ROW_PLIES] | (row[GPU_ROW_PLIES + 1] << 8));
    write_public_features_raw(row + GPU_ROW_HEX_OWNER, row + GPU_ROW_HEX_SLOT, row + GPU_ROW_HEX_HEIGHT,
                              row + GPU_ROW_HEX_MARKER, row + GPU_ROW_PILES, ids, row + GPU_ROW_MARKERS,
                              row + GPU_ROW_HAND, row + GPU_ROW_FD, row + GPU_ROW_BAG, row[GPU_ROW_INITIATIVE],
                              row[GPU_ROW_INIT_MOVED] != 0, row[GPU_ROW_TO_ACT], plies, out);
}

// rebel.rs:1079-1138.
void write_public_features(const State& s, const Ctx& ctx, float* out) {
    uint8_t row[GPU_ROW_BYTES];
    pack_gpu_row(s, ctx, row);
    uint8_t ids[NTYPE];
    for (int t = 0; t < NTYPE; ++t) ids[t] = ctx.slots[t / NSLOT][t % NSLOT];
    expand_gpu_row(row, ids, out);
}

}  // namespace wc
