// Public belief states: private configs, beliefs, chance transitions of draws,
// observation keys and the public encodings the value network reads.
// Restates engine/src/rebel.rs of the reference (rebel.rs:60-1399).
#pragma once
#include <cstdint>
#include <vector>

#include "flatmap.h"
#include "game.h"

namespace wc {

constexpr int NSLOT = 5;       // rebel.rs:61
constexpr int HAND_CAP = 3;    // rebel.rs:63
constexpr int CCOUNTS = 3 * NSLOT;
constexpr int CFEAT = CCOUNTS;
constexpr float CNORM = 5.0f;  // rebel.rs:74
constexpr float SMOOTH = 1e-30f;  // rebel.rs:359

// Per-game slot tables (rebel.rs:79-111).
struct Ctx {
    uint8_t slots[2][NSLOT];
    int8_t slot_of[2][N_UNITS];
    static Ctx make(const State& s);
    Ctx mirrored() const;
};

// A player's private state (rebel.rs:117-175). inflight = -1 means None.
struct Config {
    uint8_t hand[NSLOT] = {0, 0, 0, 0, 0};
    uint8_t fd[NSLOT] = {0, 0, 0, 0, 0};
    int8_t inflight = -1;
    uint8_t hand_size() const { int n = 0; for (int k = 0; k < NSLOT; ++k) n += hand[k]; return (uint8_t)n; }
    uint8_t fd_size() const { int n = 0; for (int k = 0; k < NSLOT; ++k) n += fd[k]; return (uint8_t)n; }
    // Orders exactly like the reference's derived Ord (hand, fd, inflight).
    uint64_t key() const {
        uint64_t k = 0;
        for (int i = 0; i < NSLOT; ++i) k = (k << 2) | hand[i];
        for (int i = 0; i < NSLOT; ++i) k = (k << 5) | fd[i];
        k = (k << 3) | (uint64_t)(inflight < 0 ? 0 : inflight + 1);
        return k;
    }
    void bag(const uint8_t* reserve, uint8_t* out) const {
        for (int k = 0; k < NSLOT; ++k) {
            int used = hand[k] + fd[k] + (inflight == k ? 1 : 0);
            out[k] = reserve[k] > used ? (uint8_t)(reserve[k] - used) : 0;
        }
    }
    bool operator==(const Config& o) const { return key() == o.key(); }
    bool operator<(const Config& o) const { return key() < o.key(); }
};

void config_counts(const Config& c, const uint8_t* reserve, uint8_t* out /*CCOUNTS*/);
void reserve(const State& s, uint8_t p, const Ctx& ctx, uint8_t* out /*NSLOT*/);
void faceup_counts(const State& s, uint8_t p, const Ctx& ctx, uint8_t* out);
Config true_config(const State& s, uint8_t p, const Ctx& ctx);
void set_config(State& s, uint8_t p, const Ctx& ctx, const Config& c);
std::vector<Config> enumerate_configs(const uint8_t* reserve, uint8_t hand_size, uint8_t fd_size, bool inflight);

// A distribution over one player's configs, support sorted by key.
struct Belief {
    std::vector<Config> cfg;
    std::vector<float> p;
    static Belief point(const Config& c) { Belief b; b.cfg.push_back(c); b.p.push_back(1.0f); return b; }
    static Belief from_pairs(std::vector<std::pair<Config, float>> pairs);
    void normalize();
    int index_of(const Config& c) const;
    size_t size() const { return cfg.size(); }
};

bool action_legal(const Config& c, int slot);
bool advance_config(const Config& c, int slot, bool facedown, Config* out);
Belief belief_after_draw(const Belief& b, const uint8_t* reserve, const uint8_t* faceup, bool set_pending);

// A draw's chance transition, CSR by parent config (rebel.rs:515-531).
struct DrawMap {
    std::vector<uint32_t> start, to;
    std::vector<float> p;
    size_t rows() const { return start.empty() ? 0 : start.size() - 1; }
};

// Reusable scratch for building draw transitions (rebel.rs:546-813).
struct DrawScratch {
    std::vector<Config> kid;
    std::vector<float> prob;
    std::vector<uint64_t> order;
    std::vector<float> acc;
    std::vector<uint8_t> hit;
    std::vector<uint32_t> touched;
    // the hands dealt from each (source counts, k) met so far: the coins
    // taken per slot (5 bytes, packed) and the probability, in enumeration
    // order; deal_span[i] = (first, count) of entry i of deal_index
    FlatMap deal_index;
    std::vector<uint64_t> deal_take;
    std::vector<float> deal_p;
    std::vector<std::pair<uint32_t, uint32_t>> deal_span;
    void transition(const std::vector<Config>& cfg, const uint8_t* reserve, const uint8_t* faceup,
                    std::vector<Config>& support, DrawMap& map, bool set_pending);
    void run(const std::vector<Config>& cfg, const uint8_t* reserve, const uint8_t* faceup, uint8_t k,
             std::vector<Config>& support, DrawMap& map);
    void compose(const DrawMap& a, const DrawMap& b, size_t n_child, DrawMap& out);
    void deal(const uint8_t* src, uint32_t k, const Config& base);
    void pack(std::vector<Config>& support, DrawMap& map);
};

bool is_facedown_play(const Action& a);
uint32_t obs_key(const Action& a);

// --------------------------------------------------------------- features
constexpr int NTYPE = 2 * NSLOT;
constexpr int HEX_FACTS = 6;
constexpr int HEX_CH = HEX_FACTS + NTYPE;
constexpr int HEX_BLOCK = N_HEXES * HEX_CH;
constexpr int PILE_COUNTS = 4;
constexpr int PLAYER_SCALARS = 6;
constexpr int GLOBAL_SCALARS = 3;
constexpr int OFF_PILES = HEX_BLOCK;
constexpr int OFF_CARDS = OFF_PILES + NTYPE * PILE_COUNTS;
constexpr int OFF_LOOSE = OFF_CARDS + NTYPE * CARD_FEATS;
constexpr int LOOSE = 2 * PLAYER_SCALARS + GLOBAL_SCALARS;
constexpr int PUBFEAT = OFF_LOOSE + LOOSE;
constexpr float MAX_COINS = 21.0f;

// Compact public row (rebel.rs:973-986), 201 bytes.
constexpr int GPU_ROW_HEX_OWNER = 0;
constexpr int GPU_ROW_HEX_SLOT = GPU_ROW_HEX_OWNER + N_HEXES;
constexpr int GPU_ROW_HEX_HEIGHT = GPU_ROW_HEX_SLOT + N_HEXES;
constexpr int GPU_ROW_HEX_MARKER = GPU_ROW_HEX_HEIGHT + N_HEXES;
constexpr int GPU_ROW_PILES = GPU_ROW_HEX_MARKER + N_HEXES;
constexpr int GPU_ROW_MARKERS = GPU_ROW_PILES + NTYPE * PILE_COUNTS;
constexpr int GPU_ROW_HAND = GPU_ROW_MARKERS + 2;
constexpr int GPU_ROW_FD = GPU_ROW_HAND + 2;
constexpr int GPU_ROW_BAG = GPU_ROW_FD + 2;
constexpr int GPU_ROW_INITIATIVE = GPU_ROW_BAG + 2;
constexpr int GPU_ROW_INIT_MOVED = GPU_ROW_INITIATIVE + 1;
constexpr int GPU_ROW_TO_ACT = GPU_ROW_INIT_MOVED + 1;
constexpr int GPU_ROW_PLIES = GPU_ROW_TO_ACT + 1;
constexpr int GPU_ROW_BYTES = GPU_ROW_PLIES + 2;

// Replay row (rebel.rs:935-964), 215 bytes: the training buffer's compact
// record of a position; the training batch expands it on the device.
constexpr int ROW_VERSION = 0;
constexpr int ROW_HASH = 4;
constexpr int ROW_IDS = 12;
constexpr int ROW_HEX_OWNER = 22;
constexpr int ROW_HEX_SLOT = ROW_HEX_OWNER + N_HEXES;
constexpr int ROW_HEX_HEIGHT = ROW_HEX_SLOT + N_HEXES;
constexpr int ROW_HEX_MARKER = ROW_HEX_HEIGHT + N_HEXES;
constexpr int ROW_PILES = ROW_HEX_MARKER + N_HEXES;
constexpr int ROW_INITIATIVE = ROW_PILES + 2 * NSLOT * PILE_COUNTS;
constexpr int ROW_INIT_MOVED = ROW_INITIATIVE + 1;
constexpr int ROW_TO_ACT = ROW_INIT_MOVED + 1;
constexpr int ROW_PLIES = ROW_TO_ACT + 1;
constexpr int ROW_BYTES = ROW_PLIES + 2;
constexpr uint32_t ROW_FORMAT_VERSION = 1;  // rebel.rs:990

uint64_t rules_table_hash();                                   // rebel.rs:996-1030
void pack_row(const State& s, const Ctx& ctx, uint8_t* out);  // rebel.rs:1236-1268

void pack_gpu_row(const State& s, const Ctx& ctx, uint8_t* out);
void expand_gpu_row(const uint8_t* row, const uint8_t* ids /*NTYPE*/, float* out /*PUBFEAT*/);
void write_public_features(const State& s, const Ctx& ctx, float* out);
void normalize_weights(const float* w, size_t n, float* out);

}  // namespace wc
