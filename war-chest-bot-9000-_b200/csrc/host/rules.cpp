// Legal-move generation and apply: a line-for-line semantic restatement of
// engine/src/rules.rs. Action order within every listing, the retain-first
// dedup (rules.rs:1018) and the continuation-stack discipline all follow the
// reference, because the public tree is indexed by them.
#include <unordered_set>

#include "game.h"

namespace wc {

namespace {

inline uint8_t other(uint8_t p) { return (uint8_t)(1 - p); }
inline bool occupied(const State& s, int hex) { return s.hex_type[hex] != NONE; }
inline bool is_enemy_unit(const State& s, int hex, uint8_t me) {
    return s.hex_type[hex] != NONE && s.hex_owner[hex] == other(me);
}
inline bool is_friendly_unit(const State& s, int hex, uint8_t me) {
    return s.hex_type[hex] != NONE && s.hex_owner[hex] == me;
}
inline bool controls(const State& s, int hex, uint8_t me) {
    return board().is_location[hex] && s.loc_marker[hex] == me;
}
// Knight immunity against an attacker of effective height h (rules.rs:47-54).
inline bool attack_allowed_h(const State& s, int target_hex, uint8_t h) {
    uint8_t t = s.hex_type[target_hex];
    if (t != NONE && def(t).knight) return h >= 2;
    return true;
}
inline bool attack_allowed(const State& s, int target_hex, int attacker_hex) {
    return attack_allowed_h(s, target_hex, s.hex_height[attacker_hex]);
}
inline bool clear_two_line(const State& s, int from, int target) {
    uint8_t mid = board().between[from][target];
    return mid != NONE && !occupied(s, mid);
}
inline bool controls_target(const State& s, int hex, uint8_t me) {
    return board().is_location[hex] && s.loc_marker[hex] != me;
}

// rules.rs:1018-1021: keep the first occurrence of every encoding.
void dedup(std::vector<Action>& out) {
    size_t n = out.size();
    if (n < 2) return;
    size_t w = 0;
    if (n <= 96) {
        uint32_t seen[96];
        for (size_t i = 0; i < n; ++i) {
            uint32_t k = out[i].encode();
            bool dup = false;
            for (size_t j = 0; j < w; ++j)
                if (seen[j] == k) { dup = true; break; }
            if (!dup) { seen[w] = k; out[w++] = out[i]; }
        }
    } else {
        std::unordered_set<uint32_t> seen;
        seen.reserve(n * 2);
        for (size_t i = 0; i < n; ++i)
            if (seen.insert(out[i].encode()).second) out[w++] = out[i];
    }
    out.resize(w);
}

// Which maneuver variants a context permits, rules.rs:581-660.
enum class ManVariant { Main, Footman, Berserker, BerserkerV2, Merc, CavalryAtk };

uint8_t chain_cost(ManVariant v) {
    return (v == ManVariant::Berserker || v == ManVariant::BerserkerV2) ? 1 : 0;
}
bool allows_move(ManVariant v) { return v != ManVariant::CavalryAtk; }
bool allows_control(ManVariant v) {
    return v == ManVariant::Main || v == ManVariant::Footman || v == ManVariant::Berserker ||
           v == ManVariant::Merc;
}
bool allows_attack(ManVariant) { return true; }
Action mk_move(ManVariant v, uint8_t from, uint8_t to) {
    switch (v) {
        case ManVariant::Footman: return Action::make(K_FOOTMOVE, from, to);
        case ManVariant::Berserker: case ManVariant::BerserkerV2: return Action::make(K_BERS_MOVE, from, to);
        case ManVariant::Merc: return Action::make(K_MERC_MOVE, from, to);
        default: return Action::make(K_MOVE, from, to);
    }
}
Action mk_control(ManVariant v, uint8_t from) {
    switch (v) {
        case ManVariant::Footman: return Action::make(K_FOOTCTRL, from);
        case ManVariant::Berserker: return Action::make(K_BERS_CTRL, from);
        case ManVariant::Merc: return Action::make(K_MERC_CTRL, from);
        default: return Action::make(K_CONTROL, from);
    }
}
Action mk_attack(ManVariant v, uint8_t from, uint8_t target) {
    switch (v) {
        case ManVariant::Footman: return Action::make(K_FOOTATK, from, target);
        case ManVariant::Berserker: case ManVariant::BerserkerV2: return Action::make(K_BERS_ATK, from, target);
        case ManVariant::Merc: return Action::make(K_MERC_ATK, from, target);
        case ManVariant::CavalryAtk: return Action::make(K_CAVATK, from, target);
        default: return Action::make(K_ATTACK, from, target);
    }
}

void adj_empty(const State& s, int from, uint8_t* out, int* n) {
    const Board& b = board();
    *n = 0;
    for (int d = 0; d < 6; ++d) {
        uint8_t nb = b.neighbors[from][d];
        if (nb != NONE && !occupied(s, nb)) out[(*n)++] = nb;
    }
}

void normal_attack_targets(const State& s, int from, uint8_t eff_h, uint8_t* out, int* n) {
    const Board& b = board();
    uint8_t me = s.hex_owner[from];
    *n = 0;
    for (int d = 0; d < 6; ++d) {
        uint8_t nb = b.neighbors[from][d];
        if (nb != NONE && is_enemy_unit(s, nb, me) && attack_allowed_h(s, nb, eff_h)) out[(*n)++] = nb;
    }
}

// Hexes where p has a deployed unit of type `unit`, ascending (rules.rs:665-673).
int hexes_of(const State& s, uint8_t p, uint8_t unit, uint8_t* out) {
    int n = 0;
    for (int h = 0; h < N_HEXES; ++h)
        if (s.hex_owner[h] == p && s.hex_type[h] == unit) out[n++] = (uint8_t)h;
    return n;
}

bool has_deployed(const State& s, uint8_t p, uint8_t unit) {
    for (int h = 0; h < N_HEXES; ++h)
        if (s.hex_owner[h] == p && s.hex_type[h] == unit) return true;
    return false;
}

// rules.rs:510-549.
void list_basic_maneuvers(const State& s, int hex, ManVariant variant, std::vector<Action>& out) {
    uint8_t unit = s.hex_type[hex];
    if (unit == NONE) return;
    uint8_t me = s.hex_owner[hex];
    const UnitDef& d = def(unit);
    uint8_t buf[6];
    int n;
    if (allows_move(variant)) {
        adj_empty(s, hex, buf, &n);
        for (int i = 0; i < n; ++i) out.push_back(mk_move(variant, (uint8_t)hex, buf[i]));
    }
    if (allows_control(variant) && s.markers_hand[me] > 0 && controls_target(s, hex, me))
        out.push_back(mk_control(variant, (uint8_t)hex));
    if (allows_attack(variant) && !d.no_normal_attack) {
        uint8_t eff_h = (uint8_t)(s.hex_height[hex] - chain_cost(variant));
        normal_attack_targets(s, hex, eff_h, buf, &n);
        for (int i = 0; i < n; ++i) out.push_back(mk_attack(variant, (uint8_t)hex, buf[i]));
    }
}

// rules.rs:715-937.
void list_tactics(const State& s, int hex, std::vector<Action>& out) {
    uint8_t unit = s.hex_type[hex];
    uint8_t me = s.hex_owner[hex];
    const Board& b = board();
    switch (def(unit).tactic) {
        case Tactic::None: break;
        case Tactic::Footman:
            out.push_back(Action::make(K_TAC_FOOTMAN, unit));
            break;
        case Tactic::Archer:
            for (int t = 0; t < N_HEXES; ++t)
                if (b.dist[hex][t] == 2 && is_enemy_unit(s, t, me) && attack_allowed(s, t, hex))
                    out.push_back(Action::make(K_ARCHER, (uint8_t)hex, (uint8_t)t));
            break;
        case Tactic::Cavalry: {
            uint8_t h = s.hex_height[hex];
            uint8_t tos[6]; int n;
            adj_empty(s, hex, tos, &n);
            for (int i = 0; i < n; ++i) {
                uint8_t to = tos[i];
                bool has_target = false;
                for (int d = 0; d < 6; ++d) {
                    uint8_t nb = b.neighbors[to][d];
                    if (nb != NONE && is_enemy_unit(s, nb, me) && attack_allowed_h(s, nb, h)) { has_target = true; break; }
                }
                if (has_target) out.push_back(Action::make(K_CAVMOVE, (uint8_t)hex, to));
            }
            break;
        }
        case Tactic::Crossbowman:
            for (int t = 0; t < N_HEXES; ++t)
                if (b.dist[hex][t] == 2 && is_enemy_unit(s, t, me) && clear_two_line(s, hex, t) &&
                    attack_allowed(s, t, hex))
                    out.push_back(Action::make(K_CROSSBOW, (uint8_t)hex, (uint8_t)t));
            break;
        case Tactic::Ensign:
            for (int u = 0; u < N_HEXES; ++u) {
                if (u == hex || !is_friendly_unit(s, u, me) || b.dist[hex][u] > 2) continue;
                for (int d = 0; d < 6; ++d) {
                    uint8_t to = b.neighbors[u][d];
                    if (to == NONE) continue;
                    if (!occupied(s, to) && b.dist[hex][to] <= 2)
                        out.push_back(Action::make(K_ENSIGN, (uint8_t)u, to));
                }
            }
            break;
        case Tactic::Lancer: {
            bool bolstered = s.hex_height[hex] >= 2;
            for (int d = 0; d < 6; ++d) {
                uint8_t s1 = b.step[hex][d];
                if (s1 == NONE || occupied(s, s1)) continue;
                uint8_t beyond1 = b.step[s1][d];
                if (beyond1 != NONE && is_enemy_unit(s, beyond1, me)) {
                    bool knight = def(s.hex_type[beyond1]).knight;
                    if (!knight || bolstered) out.push_back(Action::make(K_LANCER, (uint8_t)hex, s1, beyond1));
                }
                uint8_t s2 = b.step[s1][d];
                if (s2 != NONE && !occupied(s, s2)) {
                    uint8_t beyond2 = b.step[s2][d];
                    if (beyond2 != NONE && is_enemy_unit(s, beyond2, me)) {
                        bool knight = def(s.hex_type[beyond2]).knight;
                        if (!knight || bolstered) out.push_back(Action::make(K_LANCER, (uint8_t)hex, s2, beyond2));
                    }
                }
            }
            break;
        }
        case Tactic::LightCavalry:
            for (int d1 = 0; d1 < 6; ++d1) {
                uint8_t m = b.neighbors[hex][d1];
                if (m == NONE || occupied(s, m)) continue;
                for (int d2 = 0; d2 < 6; ++d2) {
                    uint8_t to = b.neighbors[m][d2];
                    if (to == NONE || to == hex || occupied(s, to)) continue;
                    if (b.dist[hex][to] != 2) continue;
                    out.push_back(Action::make(K_LIGHTCAV, (uint8_t)hex, to));
                }
            }
            break;
        case Tactic::Marshal:
            for (int u = 0; u < N_HEXES; ++u) {
                if (u == hex || !is_friendly_unit(s, u, me) || b.dist[hex][u] > 2) continue;
                if (def(s.hex_type[u]).no_normal_attack) continue;
                uint8_t tg[6]; int n;
                normal_attack_targets(s, u, s.hex_height[u], tg, &n);
                for (int i = 0; i < n; ++i) out.push_back(Action::make(K_MARSHAL, (uint8_t)u, tg[i]));
            }
            break;
        case Tactic::RoyalGuard:
            if (s.zones[me][s.pay_zone()][ROYAL_COIN] == 0) return;
            for (int d1 = 0; d1 < 6; ++d1) {
                uint8_t m = b.neighbors[hex][d1];
                if (m == NONE || occupied(s, m)) continue;
                if (controls(s, m, me)) out.push_back(Action::make(K_ROYALGUARD, (uint8_t)hex, m));
                for (int d2 = 0; d2 < 6; ++d2) {
                    uint8_t to = b.neighbors[m][d2];
                    if (to == NONE || to == hex || occupied(s, to)) continue;
                    if (controls(s, to, me)) out.push_back(Action::make(K_ROYALGUARD, (uint8_t)hex, to));
                }
            }
            break;
    }
}

// rules.rs:946-1013.
void list_main_play(const State& s, uint8_t p, std::vector<Action>& out) {
    bool claim_ok = s.initiative != p && !s.initiative_moved;
    int pay = s.pay_zone();
    uint8_t hx[N_HEXES];
    for (int u = 0; u < N_UNITS; ++u) {
        if (s.zones[p][pay][u] == 0) continue;
        uint8_t unit = (uint8_t)u;
        const UnitDef& d = def(unit);
        if (claim_ok) out.push_back(Action::make(K_CLAIM, unit));
        out.push_back(Action::make(K_PASS, unit));
        for (int r = 0; r < N_UNITS; ++r)
            if (s.zones[p][Z_SUPPLY][r] > 0) out.push_back(Action::make(K_RECRUIT, unit, (uint8_t)r));
        if (d.is_royal_coin) {
            int n = hexes_of(s, p, ROYAL_GUARD, hx);
            for (int i = 0; i < n; ++i) list_tactics(s, hx[i], out);
            continue;
        }
        if (!has_deployed(s, p, unit) || d.two_footmen) {
            int cap = d.two_footmen ? 2 : 1;
            if (hexes_of(s, p, unit, hx) < cap) {
                for (int h = 0; h < N_HEXES; ++h)
                    if (controls(s, h, p) && !occupied(s, h)) out.push_back(Action::make(K_DEPLOY, unit, (uint8_t)h));
                if (d.scout) {
                    const Board& b = board();
                    for (int h = 0; h < N_HEXES; ++h) {
                        if (occupied(s, h)) continue;
                        bool ok = false;
                        for (int dd = 0; dd < 6; ++dd) {
                            uint8_t nb = b.neighbors[h][dd];
                            if (nb != NONE && is_friendly_unit(s, nb, p)) { ok = true; break; }
                        }
                        if (ok) out.push_back(Action::make(K_DEPLOY, unit, (uint8_t)h));
                    }
                }
            }
        }
        int n = hexes_of(s, p, unit, hx);
        for (int i = 0; i < n; ++i) out.push_back(Action::make(K_BOLSTER, unit, hx[i]));
        for (int i = 0; i < n; ++i) {
            list_basic_maneuvers(s, hx[i], ManVariant::Main, out);
            list_tactics(s, hx[i], out);
        }
    }
    dedup(out);
}

}  // namespace

// ------------------------------------------------------- zone primitives

// rules.rs:73-85.
void State::remove_stack_coin(int hex, bool eliminate) {
    uint8_t p = hex_owner[hex];
    uint8_t unit = hex_type[hex];
    int z = eliminate ? Z_ELIM : Z_FACEUP;
    zones[p][z][unit] += 1;
    hex_height[hex] -= 1;
    if (hex_height[hex] == 0) {
        hex_type[hex] = NONE;
        hex_owner[hex] = NONE;
    }
}

void State::move_stack(int from, int to) {
    hex_type[to] = hex_type[from];
    hex_owner[to] = hex_owner[from];
    hex_height[to] = hex_height[from];
    hex_type[from] = NONE;
    hex_owner[from] = NONE;
    hex_height[from] = 0;
}

// rules.rs:101-113.
void State::place_marker(int hex, uint8_t p) {
    uint8_t prev = loc_marker[hex];
    if (prev != NONE && prev != p) markers_hand[prev] += 1;
    if (prev != p) markers_hand[p] -= 1;
    loc_marker[hex] = p;
    if (markers_on_board(p) >= WIN_MARKERS) winner = p;
}

// --------------------------------------------------------- attack engine

// rules.rs:126-153.
void State::queue_maneuver_post(int hex, bool was_attack, bool was_move) {
    if (hex_type[hex] == NONE) return;
    const UnitDef& d = def(hex_type[hex]);
    bool bers = d.berserker_v1 ? true : (d.berserker_v2 ? (was_attack || was_move) : false);
    if (bers && hex_height[hex] >= 2) conts.push(Cont::make(C_BERSCHAIN, (uint8_t)hex, d.berserker_v2 ? 1 : 0));
    if (d.swordsman && was_attack) conts.push(Cont::make(C_SWORDMOVE, (uint8_t)hex));
}

// rules.rs:163-201.
void State::resolve_attack(int atk_hex, int tgt_hex) {
    const Board& b = board();
    bool adjacent = b.dist[atk_hex][tgt_hex] == 1;
    uint8_t tgt_unit = hex_type[tgt_hex];
    uint8_t defender = hex_owner[tgt_hex];
    bool pikeman_reflex = tgt_unit != NONE && def(tgt_unit).pikeman && adjacent;
    bool rg_soak = tgt_unit != NONE && def(tgt_unit).royal_guard &&
                   zones[defender][Z_SUPPLY][ROYAL_GUARD] > 0;
    if (pikeman_reflex) remove_stack_coin(atk_hex, true);
    if (rg_soak) {
        conts.push(Cont::make(C_ATKPOST, (uint8_t)atk_hex));
        pending = Cont::make(C_RGCHOICE, defender, (uint8_t)tgt_hex);
        interrupt = true;
        return;
    }
    if (tgt_unit != NONE) remove_stack_coin(tgt_hex, true);
    queue_maneuver_post(atk_hex, true, false);
}

// ------------------------------------------------- continuation advancing

void State::finish() {
    if (interrupt) {
        interrupt = false;
        return;
    }
    advance();
}

// rules.rs:222-271.
void State::advance() {
    std::vector<Action> probe;
    for (;;) {
        if (winner != NONE) return;
        Cont c;
        if (!conts.pop(&c)) {
            end_turn();
            return;
        }
        if (c.kind == C_ATKPOST) {
            queue_maneuver_post(c.a, true, false);
            continue;
        }
        if (c.kind == C_FOOTMAN || c.kind == C_CAVATK) {
            pending = c;
            legal_actions_into(probe);
            if (probe.empty()) continue;
            return;
        }
        if (c.kind == C_MAINPLAY) {
            begin_main_turn();
            return;
        }
        pending = c;
        return;
    }
}

void State::end_turn() {
    turns_taken[active] += 1;
    wp_v2_triggered = false;
    active = other(active);
    begin_main_turn();
}

// rules.rs:286-305.
void State::begin_main_turn() {
    if (main_plays >= MAX_MAIN_PLAYS) {
        adjudicated_draw = true;
        return;
    }
    uint8_t a = active, o = other(active);
    if (hand_size(a) > 0) {
        pending = Cont::make(C_MAINPLAY);
    } else if (hand_size(o) > 0) {
        active = o;
        pending = Cont::make(C_MAINPLAY);
    } else {
        round += 1;
        first_player = initiative;
        active = initiative;
        start_round_draws();
    }
}

// ------------------------------------------------------ maneuver effects

// rules.rs:315-345.
void State::queue_wp_post(int hex) {
    if (!wp_trigger_ready(hex)) return;
    if (def(hex_type[hex]).warrior_priest_v2) wp_v2_triggered = true;
    conts.push(Cont::make(C_WPDRAW, hex_owner[hex], NONE));
}

bool State::wp_trigger_ready(int hex) const {
    if (hex_type[hex] == NONE) return false;
    const UnitDef& d = def(hex_type[hex]);
    if (!d.warrior_priest) return false;
    if (d.warrior_priest_v2 && wp_v2_triggered) return false;
    return true;
}

void State::do_move(int from, int to) {
    move_stack(from, to);
    queue_maneuver_post(to, false, true);
}

void State::do_control(int hex) {
    uint8_t p = hex_owner[hex];
    place_marker(hex, p);
    queue_maneuver_post(hex, false, false);
    queue_wp_post(hex);
}

// rules.rs:376-397.
void State::do_attack(int from, int target) {
    resolve_attack(from, target);
    if (interrupt) {
        if (wp_trigger_ready(from) && pending.kind == C_RGCHOICE) {
            uint8_t rg_hex = pending.b;
            if (def(hex_type[from]).warrior_priest_v2) wp_v2_triggered = true;
            uint8_t p = hex_owner[from];
            pending = Cont::make(C_WPDRAW, p, rg_hex);
        }
    } else {
        queue_wp_post(from);
    }
}

// ------------------------------------------------------------ draw helpers

void State::refill_bag(uint8_t p) {
    for (int u = 0; u < N_UNITS; ++u) {
        zones[p][Z_BAG][u] += zones[p][Z_FACEUP][u] + zones[p][Z_FACEDOWN][u];
        zones[p][Z_FACEUP][u] = 0;
        zones[p][Z_FACEDOWN][u] = 0;
    }
}

// rules.rs:481-497.
int State::first_drawable(uint8_t p) const {
    for (int u = 0; u < N_UNITS; ++u)
        if (zones[p][Z_BAG][u] > 0) return u;
    for (int u = 0; u < N_UNITS; ++u)
        if (zones[p][Z_BAG][u] + zones[p][Z_FACEUP][u] + zones[p][Z_FACEDOWN][u] > 0) return u;
    return -1;
}

void State::do_draw(uint8_t p, uint8_t unit, int to) {
    bool bag_empty = true;
    for (int u = 0; u < N_UNITS; ++u)
        if (zones[p][Z_BAG][u] > 0) { bag_empty = false; break; }
    if (bag_empty) refill_bag(p);
    zmove(p, Z_BAG, to, unit);
}

// --------------------------------------------------------- legal actions

// Distinct drawable coin types in unit order (rules.rs:443-473).
static void drawable_units(const State& s, uint8_t p, std::vector<Action>& out) {
    bool bag_empty = true;
    for (int u = 0; u < N_UNITS; ++u)
        if (s.zones[p][Z_BAG][u] > 0) { bag_empty = false; break; }
    for (int u = 0; u < N_UNITS; ++u) {
        int c = bag_empty ? s.zones[p][Z_BAG][u] + s.zones[p][Z_FACEUP][u] + s.zones[p][Z_FACEDOWN][u]
                          : s.zones[p][Z_BAG][u];
        if (c > 0) out.push_back(Action::make(K_DRAW, (uint8_t)u));
    }
}

void State::legal_actions_into(std::vector<Action>& out) const {
    out.clear();
    if (winner != NONE) return;
    const State& s = *this;
    switch (pending.kind) {
        case C_DRAW:
            drawable_units(s, pending.a, out);
            break;
        case C_WPDRAW:
            drawable_units(s, pending.a, out);
            if (out.empty()) out.push_back(Action::make(K_DRAW, NONE));
            break;
        case C_MAINPLAY:
            list_main_play(s, active, out);
            break;
        case C_WPPLAY:
            list_main_play(s, pending.a, out);
            break;
        case C_RGCHOICE:
            out.push_back(Action::make(K_RG_SUPPLY));
            out.push_back(Action::make(K_RG_STACK));
            break;
        case C_SWORDMOVE: {
            uint8_t tos[6]; int n;
            adj_empty(s, pending.a, tos, &n);
            for (int i = 0; i < n; ++i) out.push_back(Action::make(K_SWORD_MOVE, pending.a, tos[i]));
            out.push_back(Action::make(K_SWORD_DECLINE));
            break;
        }
        case C_BERSCHAIN:
            list_basic_maneuvers(s, pending.a, pending.b ? ManVariant::BerserkerV2 : ManVariant::Berserker, out);
            out.push_back(Action::make(K_BERS_STOP));
            break;
        case C_MERC:
            list_basic_maneuvers(s, pending.a, ManVariant::Merc, out);
            out.push_back(Action::make(K_MERC_DECLINE));
            break;
        case C_FOOTMAN: {
            uint64_t bits = pending.hexes;
            while (bits) {
                int h = __builtin_ctzll(bits);
                bits &= bits - 1;
                list_basic_maneuvers(s, h, ManVariant::Footman, out);
            }
            break;
        }
        case C_CAVATK:
            list_basic_maneuvers(s, pending.a, ManVariant::CavalryAtk, out);
            break;
        case C_FID: {
            uint8_t p = active;
            uint8_t hx[N_HEXES];
            if (hexes_of(s, p, pending.a, hx) < 2) {
                for (int h = 0; h < N_HEXES; ++h)
                    if (controls(s, h, p) && !occupied(s, h)) out.push_back(Action::make(K_FID_DEPLOY, (uint8_t)h));
            }
            out.push_back(Action::make(K_FID_DECLINE));
            break;
        }
        default:
            break;
    }
    dedup(out);
}

// ------------------------------------------------------------------ apply

// rules.rs:1155-1289.
void State::apply_inplace(const Action& action) {
    switch (pending.kind) {
        case C_DRAW: {
            uint8_t player = pending.a;
            if (action.kind == K_DRAW) do_draw(player, action.a, Z_HAND);
            finish();
            return;
        }
        case C_WPDRAW: {
            uint8_t player = pending.a, rg_hex = pending.b;
            if (action.kind == K_DRAW) {
                bool has_rg = rg_hex != NONE;
                if (action.a == NONE) {
                    if (has_rg) pending = Cont::make(C_RGCHOICE, hex_owner[rg_hex], rg_hex);
                    else finish();
                } else {
                    do_draw(player, action.a, Z_INFLIGHT);
                    if (has_rg) {
                        Cont c = Cont::make(C_RGCHOICE, hex_owner[rg_hex], rg_hex);
                        conts.push(Cont::make(C_WPPLAY, player));
                        pending = c;
                    } else {
                        pending = Cont::make(C_WPPLAY, player);
                    }
                }
            }
            return;
        }
        default:
            break;
    }
    switch (pending.kind) {
        case C_MAINPLAY:
            main_plays += 1;
            apply_main(active, action);
            return;
        case C_WPPLAY:
            apply_main(pending.a, action);
            return;
        case C_RGCHOICE: {
            uint8_t defender = pending.a, rg_hex = pending.b;
            if (action.kind == K_RG_SUPPLY) {
                zones[defender][Z_SUPPLY][ROYAL_GUARD] -= 1;
                zones[defender][Z_ELIM][ROYAL_GUARD] += 1;
            } else if (action.kind == K_RG_STACK) {
                remove_stack_coin(rg_hex, true);
            }
            finish();
            return;
        }
        case C_SWORDMOVE:
            if (action.kind == K_SWORD_MOVE) do_move(action.a, action.b);
            finish();
            return;
        case C_BERSCHAIN:
            apply_berserker(pending.a, action);
            return;
        case C_MERC:
            if (action.kind == K_MERC_MOVE) do_move(action.a, action.b);
            else if (action.kind == K_MERC_CTRL) do_control(action.a);
            else if (action.kind == K_MERC_ATK) do_attack(action.a, action.b);
            finish();
            return;
        case C_FOOTMAN:
            apply_footman(pending.hexes, action);
            return;
        case C_CAVATK:
            if (action.kind == K_CAVATK) do_attack(action.a, action.b);
            finish();
            return;
        case C_FID: {
            uint8_t coin = pending.a;
            if (action.kind == K_FID_DEPLOY) {
                zones[active][Z_FACEUP][coin] -= 1;
                place_unit(active, coin, action.a);
            }
            finish();
            return;
        }
        default:
            return;
    }
}

void State::place_unit(uint8_t p, uint8_t unit, int hex) {
    hex_type[hex] = unit;
    hex_owner[hex] = p;
    hex_height[hex] = 1;
}

// rules.rs:1304-1445.
void State::apply_main(uint8_t p, const Action& a) {
    int pay = pay_zone();
    auto spend_maneuver_coin = [&](int hex) { zmove(p, pay, Z_FACEUP, hex_type[hex]); };
    switch (a.kind) {
        case K_DEPLOY:
            zones[p][pay][a.a] -= 1;
            place_unit(p, a.a, a.b);
            finish();
            break;
        case K_BOLSTER:
            zones[p][pay][a.a] -= 1;
            hex_height[a.b] += 1;
            finish();
            break;
        case K_CLAIM:
            zmove(p, pay, Z_FACEDOWN, a.a);
            initiative = p;
            initiative_moved = true;
            finish();
            break;
        case K_PASS:
            zmove(p, pay, Z_FACEDOWN, a.a);
            finish();
            break;
        case K_RECRUIT: {
            zmove(p, pay, Z_FACEDOWN, a.a);
            uint8_t unit = a.b;
            zones[p][Z_SUPPLY][unit] -= 1;
            zones[p][Z_FACEUP][unit] += 1;
            const UnitDef& d = def(unit);
            if (d.mercenary && has_deployed(*this, p, unit)) {
                uint8_t hx[N_HEXES];
                hexes_of(*this, p, unit, hx);
                conts.push(Cont::make(C_MERC, hx[0]));
            }
            if (d.footman_v2 && has_deployed(*this, p, unit)) conts.push(Cont::make(C_FID, unit));
            finish();
            break;
        }
        case K_MOVE:
            spend_maneuver_coin(a.a);
            do_move(a.a, a.b);
            finish();
            break;
        case K_CONTROL:
            spend_maneuver_coin(a.a);
            do_control(a.a);
            finish();
            break;
        case K_ATTACK: case K_ARCHER: case K_CROSSBOW:
            spend_maneuver_coin(a.a);
            do_attack(a.a, a.b);
            finish();
            break;
        case K_CAVMOVE:
            spend_maneuver_coin(a.a);
            do_move(a.a, a.b);
            conts.push(Cont::make(C_CAVATK, a.b));
            finish();
            break;
        case K_ENSIGN:
            zmove(p, pay, Z_FACEUP, ENSIGN);
            do_move(a.a, a.b);
            finish();
            break;
        case K_LANCER:
            spend_maneuver_coin(a.a);
            move_stack(a.a, a.b);
            do_attack(a.b, a.c);
            finish();
            break;
        case K_LIGHTCAV:
            spend_maneuver_coin(a.a);
            do_move(a.a, a.b);
            finish();
            break;
        case K_MARSHAL:
            zmove(p, pay, Z_FACEUP, MARSHAL);
            do_attack(a.a, a.b);
            finish();
            break;
        case K_ROYALGUARD:
            zmove(p, pay, Z_FACEUP, ROYAL_COIN);
            do_move(a.a, a.b);
            finish();
            break;
        case K_TAC_FOOTMAN: {
            zmove(p, pay, Z_FACEUP, a.a);
            uint64_t hexes = 0;
            uint8_t hx[N_HEXES];
            for (uint8_t u : {(uint8_t)FOOTMAN, (uint8_t)FOOTMAN_V2}) {
                int n = hexes_of(*this, p, u, hx);
                for (int i = 0; i < n; ++i) hexes |= 1ull << hx[i];
            }
            if (hexes) conts.push(Cont::make(C_FOOTMAN, 0, 0, hexes));
            finish();
            break;
        }
        default:
            finish();
            break;
    }
}

// rules.rs:1460-1495.
void State::apply_berserker(uint8_t hex, const Action& a) {
    if (a.kind == K_BERS_STOP) {
        finish();
        return;
    }
    int h = hex;
    uint8_t unit = hex_type[h];
    zones[hex_owner[h]][Z_FACEUP][unit] += 1;
    hex_height[h] -= 1;
    if (a.kind == K_BERS_MOVE) do_move(a.a, a.b);
    else if (a.kind == K_BERS_CTRL) do_control(a.a);
    else if (a.kind == K_BERS_ATK) do_attack(a.a, a.b);
    finish();
}

// rules.rs:1499-1519.
void State::apply_footman(uint64_t hexes, const Action& a) {
    uint8_t from = NONE;
    if (a.kind == K_FOOTMOVE || a.kind == K_FOOTCTRL || a.kind == K_FOOTATK) from = a.a;
    if (a.kind == K_FOOTMOVE) do_move(a.a, a.b);
    else if (a.kind == K_FOOTCTRL) do_control(a.a);
    else if (a.kind == K_FOOTATK) do_attack(a.a, a.b);
    uint64_t rest = hexes;
    if (from < 64) rest &= ~(1ull << from);
    if (rest) conts.push(Cont::make(C_FOOTMAN, 0, 0, rest));
    finish();
}

}  // namespace wc
