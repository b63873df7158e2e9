// War Chest rules engine: board geometry, unit cards, the action encoding,
// the flat game state and its continuation stack, legal moves and apply.
//
// A C++ restatement of the reference engine (fplonka/war-chest-bot-9000-):
//   engine/src/board.rs   hex geometry            (board.rs:32-135)
//   engine/src/units.rs   the 20 unit cards       (units.rs:5-218)
//   engine/src/actions.rs action kinds + encoding (actions.rs:50-295)
//   engine/src/state.rs   State, Cont, ContStack  (state.rs:45-606)
//   engine/src/rules.rs   legality and apply      (rules.rs:1-1534)
//   engine/src/rng.rs     xorshift64*             (rng.rs:5-45)
// Legal-action order, dedup order and every state transition must match the
// reference bit for bit, because subgame trees are indexed by them.
#pragma once
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

namespace wc {

constexpr int N_HEXES = 37;
constexpr int N_LOCATIONS = 10;
constexpr uint8_t NONE = 255;
constexpr int N_UNITS = 20;
constexpr int N_PLAYERS = 2;
constexpr uint8_t HAND_MAX = 3;
constexpr uint8_t MARKERS_TOTAL = 6;
constexpr uint8_t WIN_MARKERS = 6;
constexpr uint16_t MAX_MAIN_PLAYS = 256;
constexpr float CAP_MARKER_VALUE_DEFAULT = 0.15f;

// Zones, state.rs:46-56.
constexpr int Z_BAG = 0, Z_HAND = 1, Z_FACEUP = 2, Z_FACEDOWN = 3, Z_SUPPLY = 4, Z_ELIM = 5,
              Z_INFLIGHT = 6, N_ZONES = 7;
constexpr uint8_t WHITE = 0, BLACK = 1;

// ------------------------------------------------------------------ board

struct Board {
    int8_t coord[N_HEXES][2];
    uint8_t neighbors[N_HEXES][6];
    uint8_t dist[N_HEXES][N_HEXES];
    bool is_location[N_HEXES];
    uint8_t location_hexes[N_LOCATIONS];
    uint8_t between[N_HEXES][N_HEXES];
    uint8_t step[N_HEXES][6];
};
const Board& board();
int mirror_hex(int h);

// ------------------------------------------------------------------ units

enum UnitIdx : uint8_t {
    ARCHER = 0, BERSERKER, CAVALRY, CROSSBOWMAN, ENSIGN, FOOTMAN, KNIGHT, LANCER, LIGHT_CAVALRY,
    MARSHAL, MERCENARY, PIKEMAN, SCOUT, SWORDSMAN, WARRIOR_PRIEST, ROYAL_GUARD, BERSERKER_V2,
    FOOTMAN_V2, WARRIOR_PRIEST_V2, ROYAL_COIN
};

enum class Tactic : uint8_t {
    None = 0, Archer, Cavalry, Crossbowman, Ensign, Footman, Lancer, LightCavalry, Marshal, RoyalGuard
};
constexpr int N_TACTICS = 10;
constexpr int CARD_FEATS = N_TACTICS + 12 + 2 + 1;  // units.rs:64

struct UnitDef {
    uint16_t id;
    const char* name;
    uint8_t coins;
    Tactic tactic;
    bool berserker_v1, berserker_v2, knight, mercenary, pikeman, royal_guard, scout, swordsman,
        warrior_priest, warrior_priest_v2, footman_v2, two_footmen, no_normal_attack, is_royal_coin;
};
const UnitDef& def(uint8_t idx);
int index_of_id(uint16_t id);  // -1 if unknown
void write_card_features(uint8_t u, float* out);  // CARD_FEATS floats, units.rs:76

// ---------------------------------------------------------------- actions

// Stable kind numbers, actions.rs:133-171.
enum Kind : uint8_t {
    K_DEPLOY = 0, K_BOLSTER, K_CLAIM, K_RECRUIT, K_PASS, K_MOVE, K_CONTROL, K_ATTACK, K_ARCHER,
    K_CAVMOVE, K_CAVATK, K_CROSSBOW, K_ENSIGN, K_LANCER, K_LIGHTCAV, K_MARSHAL, K_ROYALGUARD,
    K_FOOTMOVE, K_FOOTCTRL, K_FOOTATK, K_DRAW, K_RG_SUPPLY, K_RG_STACK, K_SWORD_MOVE,
    K_SWORD_DECLINE, K_BERS_MOVE, K_BERS_CTRL, K_BERS_ATK, K_BERS_STOP, K_MERC_MOVE, K_MERC_CTRL,
    K_MERC_ATK, K_MERC_DECLINE, K_FID_DEPLOY, K_FID_DECLINE, K_GRANT_MOVE, K_GRANT_ATK,
    K_GRANT_CTRL, K_TAC_FOOTMAN
};
constexpr int N_KINDS = 39;

// One action: the stable kind and up to three 8-bit fields in the order the
// reference encodes them (a, b, c). Fields a variant does not have are 0, so
// `encode` reproduces `Action::encode` (actions.rs:252-295) exactly.
struct Action {
    uint8_t kind = 0, a = 0, b = 0, c = 0;
    static Action make(uint8_t k, uint8_t a = 0, uint8_t b = 0, uint8_t c = 0) {
        Action x; x.kind = k; x.a = a; x.b = b; x.c = c; return x;
    }
    uint32_t encode() const {
        auto e = [](uint8_t v) -> uint32_t { return v == NONE ? 63u : (uint32_t)v; };
        return (uint32_t)kind | (e(a) << 6) | (e(b) << 12) | (e(c) << 18);
    }
    static bool decode(uint32_t code, Action* out);
    bool operator==(const Action& o) const { return encode() == o.encode(); }
    std::string to_string() const;
};

// --------------------------------------------------------- continuations

enum ContKind : uint8_t {
    C_DRAW = 0, C_MAINPLAY, C_RGCHOICE, C_SWORDMOVE, C_BERSCHAIN, C_FOOTMAN, C_CAVATK, C_MERC,
    C_FID, C_WPDRAW, C_WPPLAY, C_ATKPOST
};

// Cont (state.rs:121-164). Field use per kind:
//   Draw{player}=a  RoyalGuardChoice{defender=a, rg_hex=b}  SwordsmanMove{hex=a}
//   BerserkerChain{hex=a, v2=b}  FootmanManeuver{hexes}  CavalryAttack{hex=a}
//   MercenaryManeuver{hex=a}  FootmanInstantDeploy{coin=a}
//   WarriorPriestDraw{player=a, rg_hex=b}  WarriorPriestPlay{player=a}  _AttackPost{atk_hex=a}
struct Cont {
    uint8_t kind = C_MAINPLAY, a = 0, b = 0;
    uint8_t pad_[5] = {0, 0, 0, 0, 0};  // explicit, so a State's bytes are all defined
    uint64_t hexes = 0;
    static Cont make(uint8_t k, uint8_t a = 0, uint8_t b = 0, uint64_t h = 0) {
        Cont c; c.kind = k; c.a = a; c.b = b; c.hexes = h; return c;
    }
    bool operator==(const Cont& o) const {
        return kind == o.kind && a == o.a && b == o.b && hexes == o.hexes;
    }
};

constexpr int CONT_CAP = 16;  // state.rs:172

struct ContStack {
    uint8_t n = 0;
    uint8_t pad_[7] = {0, 0, 0, 0, 0, 0, 0};
    Cont v[CONT_CAP];
    void push(const Cont& c);
    bool pop(Cont* out) {
        if (n == 0) return false;
        --n; *out = v[n]; return true;
    }
    void clear() { n = 0; }
    bool empty() const { return n == 0; }
};

// ----------------------------------------------------------------- state

struct State {
    uint8_t hex_type[N_HEXES];
    uint8_t hex_owner[N_HEXES];
    uint8_t hex_height[N_HEXES];
    uint8_t loc_marker[N_HEXES];
    uint8_t zones[N_PLAYERS][N_ZONES][N_UNITS];
    uint8_t markers_hand[N_PLAYERS];
    uint8_t initiative;
    bool initiative_moved;
    uint16_t round;
    uint8_t first_player;
    uint8_t active;
    uint8_t turns_taken[N_PLAYERS];
    uint16_t main_plays;
    uint8_t winner;
    bool adjudicated_draw;
    uint8_t pad0_[6];  // explicit padding (zeroed by blank()): root bytes are canonical
    Cont pending;
    ContStack conts;
    bool wp_v2_triggered;
    bool interrupt;
    uint8_t pad1_[6];

    static State from_draft(const uint16_t* white4, const uint16_t* black4, uint8_t first);
    static State blank(uint8_t active);
    void start_round_draws();
    void begin_main_turn();

    uint8_t hand_size(uint8_t p) const;
    uint8_t bag_size(uint8_t p) const;
    uint8_t markers_on_board(uint8_t p) const;
    bool is_terminal() const { return winner != NONE || adjudicated_draw; }
    float utility(int player) const;
    uint8_t to_act() const;
    bool is_chance() const { return pending.kind == C_DRAW || pending.kind == C_WPDRAW; }
    uint8_t total_coins(uint8_t p, int unit) const;
    State mirror() const;

    // Legal actions (rules.rs:1027-1124) into a caller-owned buffer.
    void legal_actions_into(std::vector<Action>& out) const;
    std::vector<Action> legal_actions() const { std::vector<Action> v; legal_actions_into(v); return v; }
    void apply_inplace(const Action& a);
    State apply(const Action& a) const { State s = *this; s.apply_inplace(a); return s; }
    int first_drawable(uint8_t p) const;  // -1 when nothing can be drawn

    // test builders, state.rs:501-559
    void set_unit(int hex, uint8_t owner, uint8_t unit, uint8_t height) {
        hex_type[hex] = unit; hex_owner[hex] = owner; hex_height[hex] = height;
    }
    void add_zone(uint8_t p, int zone, uint8_t unit, uint8_t n) { zones[p][zone][unit] += n; }

    // ---- internals (rules.rs) ----
    void zmove(uint8_t p, int from, int to, uint8_t unit) {
        zones[p][from][unit] -= 1; zones[p][to][unit] += 1;
    }
    void remove_stack_coin(int hex, bool eliminate);
    void move_stack(int from, int to);
    void place_marker(int hex, uint8_t p);
    void queue_maneuver_post(int hex, bool was_attack, bool was_move);
    void resolve_attack(int atk_hex, int tgt_hex);
    void finish();
    void advance();
    void end_turn();
    void queue_wp_post(int hex);
    bool wp_trigger_ready(int hex) const;
    void do_move(int from, int to);
    void do_control(int hex);
    void do_attack(int from, int target);
    void refill_bag(uint8_t p);
    int pay_zone() const { return pending.kind == C_WPPLAY ? Z_INFLIGHT : Z_HAND; }
    void do_draw(uint8_t p, uint8_t unit, int to);
    void place_unit(uint8_t p, uint8_t unit, int hex);
    void apply_main(uint8_t p, const Action& a);
    void apply_berserker(uint8_t hex, const Action& a);
    void apply_footman(uint64_t hexes, const Action& a);
};

float cap_marker_value();
void set_cap_marker_value(float v);

// ------------------------------------------------------------------- rng

// xorshift64* (rng.rs:5-45).
struct Rng {
    uint64_t s;
    explicit Rng(uint64_t seed) {
        uint64_t x = seed ^ 0x9E3779B97F4A7C15ull;
        s = x == 0 ? 0xDEADBEEFCAFEF00Dull : x;
    }
    uint64_t next_u64() {
        uint64_t x = s;
        x ^= x >> 12; x ^= x << 25; x ^= x >> 27;
        s = x;
        return x * 0x2545F4914F6CDD1Dull;
    }
    size_t below(size_t n) { return (size_t)(next_u64() % (uint64_t)n); }
    double unit_f64() { return (double)(next_u64() >> 11) * (1.0 / (double)(1ull << 53)); }
    size_t weighted_index(const double* w, size_t n);
};

}  // namespace wc
