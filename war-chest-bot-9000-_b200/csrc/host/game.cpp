// Board geometry, unit cards, action decoding and the State basics.
// Restates engine/src/{board,units,actions,state,rng}.rs of the reference.
#include "game.h"

#include <atomic>
#include <cmath>
#include <cstdio>
#include <stdexcept>
#include <type_traits>

namespace wc {

// ------------------------------------------------------------------ board
// board.rs:12-135: the radius-3 hexagon centred on (3,3), hexes numbered in
// row-major (y, then x) order; neighbour offsets in the site's order.

static const int8_t NEIGHBOR_OFFSETS[6][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}, {1, -1}, {-1, 1}};
static const int8_t LOCATION_COORDS[N_LOCATIONS][2] = {
    {4, 0}, {6, 1}, {0, 5}, {2, 6}, {2, 1}, {3, 2}, {5, 3}, {1, 3}, {3, 4}, {4, 5}};

static bool valid_coord(int x, int y) {
    return std::abs(x - 3) <= 3 && std::abs(y - 3) <= 3 && std::abs(x + y - 6) <= 3;
}

static Board build_board() {
    Board b;
    int n = 0;
    for (int y = 0; y <= 6; ++y)
        for (int x = 0; x <= 6; ++x)
            if (valid_coord(x, y)) { b.coord[n][0] = (int8_t)x; b.coord[n][1] = (int8_t)y; ++n; }
    if (n != N_HEXES) throw std::logic_error("board must have 37 hexes");
    auto index_of = [&](int x, int y) -> uint8_t {
        for (int i = 0; i < N_HEXES; ++i)
            if (b.coord[i][0] == x && b.coord[i][1] == y) return (uint8_t)i;
        return NONE;
    };
    for (int i = 0; i < N_HEXES; ++i)
        for (int d = 0; d < 6; ++d) {
            uint8_t nb = index_of(b.coord[i][0] + NEIGHBOR_OFFSETS[d][0], b.coord[i][1] + NEIGHBOR_OFFSETS[d][1]);
            b.neighbors[i][d] = nb;
            b.step[i][d] = nb;
        }
    for (int a = 0; a < N_HEXES; ++a)
        for (int c = 0; c < N_HEXES; ++c) {
            int dx = b.coord[a][0] - b.coord[c][0], dy = b.coord[a][1] - b.coord[c][1];
            b.dist[a][c] = (uint8_t)((std::abs(dx) + std::abs(dy) + std::abs(dx + dy)) / 2);
        }
    std::memset(b.between, NONE, sizeof(b.between));
    for (int a = 0; a < N_HEXES; ++a)
        for (int d = 0; d < 6; ++d) {
            uint8_t mid = b.step[a][d];
            if (mid == NONE) continue;
            uint8_t far = b.step[mid][d];
            if (far == NONE) continue;
            b.between[a][far] = mid;
        }
    for (int i = 0; i < N_HEXES; ++i) b.is_location[i] = false;
    for (int li = 0; li < N_LOCATIONS; ++li) {
        uint8_t h = index_of(LOCATION_COORDS[li][0], LOCATION_COORDS[li][1]);
        b.is_location[h] = true;
        b.location_hexes[li] = h;
    }
    return b;
}

const Board& board() {
    static const Board b = build_board();
    return b;
}

int mirror_hex(int h) {
    const Board& bd = board();
    for (int k = 0; k < N_HEXES; ++k)
        if (bd.coord[k][0] == 6 - bd.coord[h][0] && bd.coord[k][1] == 6 - bd.coord[h][1]) return k;
    throw std::logic_error("rotation left the board");
}

// ------------------------------------------------------------------ units
// units.rs:163-203: the card table and its attribute flags.

static UnitDef mk(uint16_t id, const char* name, uint8_t coins, Tactic t) {
    UnitDef d{};
    d.id = id; d.name = name; d.coins = coins; d.tactic = t;
    return d;
}

static std::vector<UnitDef> build_units() {
    std::vector<UnitDef> a = {
        mk(1, "Archer", 4, Tactic::Archer), mk(2, "Berserker", 5, Tactic::None),
        mk(3, "Cavalry", 4, Tactic::Cavalry), mk(4, "Crossbowman", 5, Tactic::Crossbowman),
        mk(5, "Ensign", 5, Tactic::Ensign), mk(6, "Footman", 5, Tactic::Footman),
        mk(7, "Knight", 4, Tactic::None), mk(8, "Lancer", 4, Tactic::Lancer),
        mk(9, "Light Cavalry", 5, Tactic::LightCavalry), mk(10, "Marshal", 5, Tactic::Marshal),
        mk(11, "Mercenary", 5, Tactic::None), mk(12, "Pikeman", 4, Tactic::None),
        mk(16, "Scout", 5, Tactic::None), mk(17, "Swordsman", 5, Tactic::None),
        mk(18, "Warrior Priest", 4, Tactic::None), mk(19, "Royal Guard", 5, Tactic::RoyalGuard),
        mk(52, "Berserker V2", 5, Tactic::None), mk(53, "Footman V2", 5, Tactic::Footman),
        mk(54, "Warrior Priest V2", 4, Tactic::None), mk(13, "Royal Coin", 1, Tactic::None)};
    a[ARCHER].no_normal_attack = true;
    a[BERSERKER].berserker_v1 = true;
    a[FOOTMAN].two_footmen = true;
    a[KNIGHT].knight = true;
    a[LANCER].no_normal_attack = true;
    a[MERCENARY].mercenary = true;
    a[PIKEMAN].pikeman = true;
    a[ROYAL_GUARD].royal_guard = true;
    a[SCOUT].scout = true;
    a[SWORDSMAN].swordsman = true;
    a[WARRIOR_PRIEST].warrior_priest = true;
    a[BERSERKER_V2].berserker_v2 = true;
    a[FOOTMAN_V2].two_footmen = true;
    a[FOOTMAN_V2].footman_v2 = true;
    a[WARRIOR_PRIEST_V2].warrior_priest = true;
    a[WARRIOR_PRIEST_V2].warrior_priest_v2 = true;
    a[ROYAL_COIN].is_royal_coin = true;
    return a;
}

const UnitDef& def(uint8_t idx) {
    static const std::vector<UnitDef> units = build_units();
    return units[idx];
}

int index_of_id(uint16_t id) {
    if (id == 13 || id == 14) return ROYAL_COIN;
    for (int i = 0; i < N_UNITS; ++i)
        if (def((uint8_t)i).id == id) return i;
    return -1;
}

void write_card_features(uint8_t u, float* out) {
    const UnitDef& d = def(u);
    for (int i = 0; i < CARD_FEATS; ++i) out[i] = 0.0f;
    out[(int)d.tactic] = 1.0f;
    const bool flags[12] = {d.berserker_v1, d.berserker_v2, d.knight, d.mercenary,
                            d.pikeman, d.royal_guard, d.scout, d.swordsman,
                            d.warrior_priest, d.warrior_priest_v2, d.footman_v2, d.two_footmen};
    for (int i = 0; i < 12; ++i) out[N_TACTICS + i] = flags[i] ? 1.0f : 0.0f;
    out[N_TACTICS + 12] = d.no_normal_attack ? 1.0f : 0.0f;
    out[N_TACTICS + 13] = d.is_royal_coin ? 1.0f : 0.0f;
    out[N_TACTICS + 14] = (float)d.coins / 5.0f;
}

// ---------------------------------------------------------------- actions

bool Action::decode(uint32_t code, Action* out) {
    uint32_t kind = code & 63u;
    auto f = [](uint32_t v) -> uint8_t { return v == 63u ? NONE : (uint8_t)v; };
    uint8_t a = f((code >> 6) & 63u), b = f((code >> 12) & 63u), c = f((code >> 18) & 63u);
    if (kind >= (uint32_t)N_KINDS) return false;
    Action x = Action::make((uint8_t)kind);
    switch (kind) {
        // two-field kinds
        case K_DEPLOY: case K_BOLSTER: case K_RECRUIT: case K_MOVE: case K_ATTACK: case K_ARCHER:
        case K_CAVMOVE: case K_CAVATK: case K_CROSSBOW: case K_ENSIGN: case K_LIGHTCAV:
        case K_MARSHAL: case K_ROYALGUARD: case K_FOOTMOVE: case K_FOOTATK: case K_SWORD_MOVE:
        case K_BERS_MOVE: case K_BERS_ATK: case K_MERC_MOVE: case K_MERC_ATK: case K_GRANT_MOVE:
        case K_GRANT_ATK:
            x.a = a; x.b = b; break;
        case K_LANCER:
            x.a = a; x.b = b; x.c = c; break;
        // one-field kinds
        case K_CLAIM: case K_PASS: case K_CONTROL: case K_FOOTCTRL: case K_DRAW: case K_BERS_CTRL:
        case K_MERC_CTRL: case K_FID_DEPLOY: case K_GRANT_CTRL: case K_TAC_FOOTMAN:
            x.a = a; break;
        default: break;  // field-less kinds
    }
    *out = x;
    return true;
}

std::string Action::to_string() const {
    char buf[96];
    std::snprintf(buf, sizeof buf, "kind=%u a=%u b=%u c=%u", kind, a, b, c);
    return buf;
}

// ------------------------------------------------------------ cap marker

// state.rs:30-43. 0x3E19999A is 0.15f32.
static std::atomic<uint32_t> CAP_MARKER_BITS{0x3E19999Au};

float cap_marker_value() {
    uint32_t u = CAP_MARKER_BITS.load(std::memory_order_relaxed);
    float f; std::memcpy(&f, &u, 4); return f;
}
void set_cap_marker_value(float v) {
    uint32_t u; std::memcpy(&u, &v, 4);
    CAP_MARKER_BITS.store(u, std::memory_order_relaxed);
}

// ----------------------------------------------------------------- state

void ContStack::push(const Cont& c) {
    if (n >= CONT_CAP) throw std::runtime_error("continuation stack overflow: raise CONT_CAP");
    v[n++] = c;
}

static_assert(std::has_unique_object_representations_v<State>,
              "State has no implicit padding, so its bytes (roots, hashes) are fully defined");

State State::blank(uint8_t active) {
    State s;
    std::memset(&s, 0, sizeof s);
    std::memset(s.hex_type, NONE, sizeof s.hex_type);
    std::memset(s.hex_owner, NONE, sizeof s.hex_owner);
    std::memset(s.loc_marker, NONE, sizeof s.loc_marker);
    s.initiative = active;
    s.initiative_moved = false;
    s.round = 1;
    s.first_player = active;
    s.active = active;
    s.main_plays = 0;
    s.winner = NONE;
    s.adjudicated_draw = false;
    s.pending = Cont::make(C_MAINPLAY);
    s.conts = ContStack();
    s.wp_v2_triggered = false;
    s.interrupt = false;
    return s;
}

// state.rs:274-325.
State State::from_draft(const uint16_t* white4, const uint16_t* black4, uint8_t first) {
    State s = blank(first);
    const uint16_t* sides[2] = {white4, black4};
    for (int p = 0; p < 2; ++p) {
        for (int i = 0; i < 4; ++i) {
            int u = index_of_id(sides[p][i]);
            if (u < 0) throw std::invalid_argument("drafted unit must be a known unitTypeId");
            uint8_t total = def((uint8_t)u).coins;
            s.zones[p][Z_BAG][u] += 2;
            s.zones[p][Z_SUPPLY][u] += total - 2;
        }
        s.zones[p][Z_BAG][ROYAL_COIN] += 1;
        s.markers_hand[p] = MARKERS_TOTAL - 2;
    }
    const Board& b = board();
    s.loc_marker[b.location_hexes[0]] = WHITE;
    s.loc_marker[b.location_hexes[1]] = WHITE;
    s.loc_marker[b.location_hexes[2]] = BLACK;
    s.loc_marker[b.location_hexes[3]] = BLACK;
    s.start_round_draws();
    return s;
}

// state.rs:330-387.
void State::start_round_draws() {
    turns_taken[0] = turns_taken[1] = 0;
    initiative_moved = false;
    uint8_t first = first_player, other = (uint8_t)(1 - first);
    auto cap_draws = [&](uint8_t p) -> uint8_t {
        uint8_t hs = hand_size(p);
        uint8_t need = hs >= HAND_MAX ? 0 : (uint8_t)(HAND_MAX - hs);
        uint8_t avail = 0;
        for (int u = 0; u < N_UNITS; ++u)
            avail += zones[p][Z_BAG][u] + zones[p][Z_FACEUP][u] + zones[p][Z_FACEDOWN][u];
        return need < avail ? need : avail;
    };
    uint8_t need_first = cap_draws(first), need_other = cap_draws(other);
    if (need_first == 0 && need_other == 0 && hand_size(first) == 0 && hand_size(other) == 0) {
        adjudicated_draw = true;
        return;
    }
    conts.clear();
    conts.push(Cont::make(C_MAINPLAY));
    for (int i = 0; i < need_other; ++i) conts.push(Cont::make(C_DRAW, other));
    for (int i = 1; i < need_first; ++i) conts.push(Cont::make(C_DRAW, first));
    Cont tmp;
    if (need_first > 0) {
        pending = Cont::make(C_DRAW, first);
    } else if (need_other > 0) {
        conts.pop(&tmp);
        pending = Cont::make(C_DRAW, other);
    } else {
        conts.pop(&tmp);
        pending = Cont::make(C_MAINPLAY);
    }
}

uint8_t State::hand_size(uint8_t p) const {
    uint8_t n = 0;
    for (int u = 0; u < N_UNITS; ++u) n += zones[p][Z_HAND][u];
    return n;
}
uint8_t State::bag_size(uint8_t p) const {
    uint8_t n = 0;
    for (int u = 0; u < N_UNITS; ++u) n += zones[p][Z_BAG][u];
    return n;
}
uint8_t State::markers_on_board(uint8_t p) const {
    uint8_t n = 0;
    for (int h = 0; h < N_HEXES; ++h)
        if (loc_marker[h] == p) ++n;
    return n;
}

// state.rs:439-452.
float State::utility(int player) const {
    if (!is_terminal()) throw std::logic_error("utility is defined only at terminals");
    if (winner != NONE) return winner == player ? 1.0f : -1.0f;
    float me = (float)markers_on_board((uint8_t)player);
    float them = (float)markers_on_board((uint8_t)(1 - player));
    return cap_marker_value() * (me - them);
}

// state.rs:456-464.
uint8_t State::to_act() const {
    switch (pending.kind) {
        case C_DRAW: case C_WPDRAW: case C_WPPLAY: case C_RGCHOICE: return pending.a;
        default: return active;
    }
}

uint8_t State::total_coins(uint8_t p, int unit) const {
    uint8_t n = 0;
    for (int z = 0; z < N_ZONES; ++z) n += zones[p][z][unit];
    for (int h = 0; h < N_HEXES; ++h)
        if (hex_owner[h] == p && hex_type[h] == unit) n += hex_height[h];
    return n;
}

// state.rs:573-595.
State State::mirror() const {
    if (!(pending.kind == C_MAINPLAY && conts.empty()))
        throw std::logic_error("the mirror is defined at a normal coin play");
    auto flip = [](uint8_t p) -> uint8_t { return p == NONE ? NONE : (uint8_t)(1 - p); };
    State m = *this;
    for (int h = 0; h < N_HEXES; ++h) {
        int k = mirror_hex(h);
        m.hex_type[k] = hex_type[h];
        m.hex_height[k] = hex_height[h];
        m.hex_owner[k] = flip(hex_owner[h]);
        m.loc_marker[k] = flip(loc_marker[h]);
    }
    std::memcpy(m.zones[0], zones[1], sizeof zones[0]);
    std::memcpy(m.zones[1], zones[0], sizeof zones[0]);
    m.markers_hand[0] = markers_hand[1]; m.markers_hand[1] = markers_hand[0];
    m.turns_taken[0] = turns_taken[1]; m.turns_taken[1] = turns_taken[0];
    m.initiative = flip(initiative);
    m.first_player = flip(first_player);
    m.active = flip(active);
    m.winner = flip(winner);
    return m;
}

// rng.rs:32-45.
size_t Rng::weighted_index(const double* w, size_t n) {
    double total = 0.0;
    for (size_t i = 0; i < n; ++i) total += w[i];
    if (!(total > 0.0 && std::isfinite(total))) throw std::invalid_argument("weighted_index: bad total");
    double needle = unit_f64() * total;
    for (size_t i = 0; i < n; ++i) {
        if (needle < w[i]) return i;
        needle -= w[i];
    }
    return n - 1;
}

}  // namespace wc
