// TEST INFRASTRUCTURE — CPU oracle of the training batch: a restatement of
// the reference's replay-row expansion (engine/src/rebel.rs:1144-1234
// write_public_features_raw, 1353-1393 expand_row), the row mirror
// (train/mirror.py:60-85 mirror_rows), the per-seat public sizes
// (train/train.py:70-79 public_sizes) and the batch assembly
// (train/train.py:249-270 make_batch), checking the device operator
// wc_replay_expand. Also the row pairs (a state's row, its mirrored state's
// row) of engine/src/py.rs:1067-1097 mirror_row_pairs, from seeded playouts,
// for the mirror's check against the engine (train/mirror.py:176-196). Never
// linked by the product library.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <vector>

#include "../war-chest-bot-9000-_b200/csrc/host/roots.h"

namespace {

using namespace wc;

// rebel.rs:1144-1234, written out on its own from the raw fields.
void features_raw(const uint8_t* owner, const uint8_t* slot, const uint8_t* height, const uint8_t* marker,
                  const uint8_t* piles, const uint8_t* ids, const uint8_t* markers_hand, const uint8_t* hand,
                  const uint8_t* fd, const uint8_t* bag, uint8_t initiative, bool moved, uint8_t to_act,
                  uint16_t plies, float* out) {
    std::fill(out, out + PUBFEAT, 0.0f);
    const Board& bd = board();
    int i = 0;
    for (int h = 0; h < N_HEXES; ++h, i += HEX_CH) {
        if (owner[h] != NONE) {
            out[i + owner[h]] = 1.0f;
            out[i + 2] = (float)height[h] / 5.0f;
            if (slot[h] != NONE) out[i + HEX_FACTS + owner[h] * NSLOT + slot[h]] = 1.0f;
        }
        if (marker[h] != NONE) out[i + 3 + marker[h]] = 1.0f;
        out[i + 5] = bd.is_location[h] ? 1.0f : 0.0f;
    }
    for (int t = 0; t < NTYPE; ++t, i += PILE_COUNTS)
        for (int k = 0; k < PILE_COUNTS; ++k) out[i + k] = (float)piles[t * PILE_COUNTS + k] / 5.0f;
    for (int t = 0; t < NTYPE; ++t, i += CARD_FEATS) write_card_features(ids[t], out + i);
    for (int p = 0; p < 2; ++p, i += PLAYER_SCALARS) {
        out[i] = (float)markers_hand[p] / 6.0f;
        out[i + 1] = (float)(uint8_t)(6 - markers_hand[p]) / 6.0f;
        out[i + 2] = (float)hand[p] / 3.0f;
        out[i + 3] = (float)fd[p] / MAX_COINS;
        out[i + 4] = (float)bag[p] / MAX_COINS;
        out[i + 5] = initiative == p ? 1.0f : 0.0f;
    }
    out[i] = (float)plies / (float)MAX_MAIN_PLAYS;
    out[i + 1] = moved ? 1.0f : 0.0f;
    out[i + 2] = to_act == 0 ? 1.0f : 0.0f;
}

// rebel.rs:1353-1393
void expand_row(const uint8_t* row, const uint8_t* hand, const uint8_t* fd, const uint8_t* bag, float* out) {
    uint8_t markers_hand[2] = {0, 0};
    for (int h = 0; h < N_HEXES; ++h)
        if (row[ROW_HEX_MARKER + h] != NONE) ++markers_hand[row[ROW_HEX_MARKER + h]];
    for (int p = 0; p < 2; ++p) markers_hand[p] = (uint8_t)(6 - markers_hand[p]);
    uint8_t initiative = row[ROW_INITIATIVE];
    if (initiative > 1) initiative = 0;
    const uint16_t plies = (uint16_t)(row[ROW_PLIES] | (row[ROW_PLIES + 1] << 8));
    features_raw(row + ROW_HEX_OWNER, row + ROW_HEX_SLOT, row + ROW_HEX_HEIGHT, row + ROW_HEX_MARKER, row + ROW_PILES,
                 row + ROW_IDS, markers_hand, hand, fd, bag, initiative, row[ROW_INIT_MOVED] != 0, row[ROW_TO_ACT],
                 plies, out);
}

uint8_t flip_seat(uint8_t v) { return v == 0 ? 1 : (v == 1 ? 0 : v); }

// train/mirror.py:60-85
void mirror_row(const uint8_t* row, uint8_t* out) {
    std::memcpy(out, row, ROW_BYTES);
    for (int lo : {ROW_HEX_OWNER, ROW_HEX_SLOT, ROW_HEX_HEIGHT, ROW_HEX_MARKER})
        for (int h = 0; h < N_HEXES; ++h) out[lo + h] = row[lo + mirror_hex(h)];
    for (int h = 0; h < N_HEXES; ++h) {
        out[ROW_HEX_OWNER + h] = flip_seat(out[ROW_HEX_OWNER + h]);
        out[ROW_HEX_MARKER + h] = flip_seat(out[ROW_HEX_MARKER + h]);
    }
    auto swap = [&](int lo, int width) {
        for (int k = 0; k < width; ++k) std::swap(out[lo + k], out[lo + width + k]);
    };
    swap(ROW_IDS, NSLOT);
    swap(ROW_PILES, NSLOT * PILE_COUNTS);
    out[ROW_INITIATIVE] = flip_seat(out[ROW_INITIATIVE]);
    out[ROW_TO_ACT] = flip_seat(out[ROW_TO_ACT]);
}

}  // namespace

extern "C" {

int oracle_replay_mirror_rows(const uint8_t* rows, size_t n, uint8_t* out) {
    for (size_t r = 0; r < n; ++r) mirror_row(rows + r * ROW_BYTES, out + r * ROW_BYTES);
    return 0;
}

// One row's expansion with the given per-seat sizes (expand_batch's rows).
int oracle_replay_expand_row(const uint8_t* row, const uint8_t* hand, const uint8_t* fd, const uint8_t* bag,
                             float* out) {
    expand_row(row, hand, fd, bag, out);
    return 0;
}

// train/train.py:249-270 (x and phi; the other outputs pass through).
int oracle_replay_make_batch(const uint8_t* rows, size_t n, const uint8_t* cc, const int64_t* seg, size_t m,
                             float* x, float* phi) {
    std::vector<uint8_t> mrow(ROW_BYTES);
    for (size_t r = 0; r < n; ++r) {
        uint8_t sz[3][2];  // public_sizes: hand, fd, bag per seat
        for (int q = 0; q < 2; ++q) {
            const int64_t key = 2 * (int64_t)r + q;
            const size_t start = (size_t)(std::lower_bound(seg, seg + m, key) - seg);
            if (start >= m) return 1;  // np.searchsorted past the end: the index would raise
            for (int z = 0; z < 3; ++z) {
                unsigned sum = 0;
                for (int k = 0; k < NSLOT; ++k) sum += cc[start * CCOUNTS + z * NSLOT + k];
                sz[z][q] = (uint8_t)sum;
            }
        }
        expand_row(rows + r * ROW_BYTES, sz[0], sz[1], sz[2], x + (2 * r) * PUBFEAT);
        mirror_row(rows + r * ROW_BYTES, mrow.data());
        const uint8_t h2[2] = {sz[0][1], sz[0][0]}, f2[2] = {sz[1][1], sz[1][0]}, b2[2] = {sz[2][1], sz[2][0]};
        expand_row(mrow.data(), h2, f2, b2, x + (2 * r + 1) * PUBFEAT);
    }
    for (size_t i = 0; i < m * CCOUNTS; ++i) phi[i] = (float)cc[i] / CNORM;
    return 0;
}

// engine/src/py.rs:1067-1097 mirror_row_pairs: rows of normal coin-play states from
// `games` seeded uniform playouts, each followed by the row of the state the
// engine's rotation (State::mirror) gives. Returns the pairs written.
size_t oracle_replay_mirror_pairs(uint32_t games, uint64_t seed, uint8_t* out, size_t cap_pairs) {
    size_t n = 0;
    for (uint32_t g = 0; g < games && n < cap_pairs; ++g) {
        Rng rng(seed * 1000003ull + g);
        State s = make_game(rng, true);
        for (int ply = 0; ply < 400 && !s.is_terminal() && n < cap_pairs; ++ply) {
            if (s.is_chance()) {
                resolve_chance(s, s.to_act(), rng);
                continue;
            }
            if (s.pending.kind == C_MAINPLAY && s.conts.empty() && ply % 3 == 0) {
                const State m = s.mirror();
                pack_row(s, Ctx::make(s), out + (2 * n) * ROW_BYTES);
                pack_row(m, Ctx::make(m), out + (2 * n + 1) * ROW_BYTES);
                ++n;
            }
            const std::vector<Action> acts = s.legal_actions();
            if (acts.empty()) break;
            s.apply_inplace(acts[rng.below((uint32_t)acts.size())]);
        }
    }
    return n;
}

// The live encoder's view of a state (write_public_features, rebel.rs:1079,
// with the engine's own hand / face-down / bag counts), the reference for
// expand_row of the state's packed row: features PUBFEAT floats, sizes
// hand[2], fd[2], bag[2].
int oracle_replay_live(const uint8_t* state, size_t len, float* features, uint8_t* sizes) {
    State s;
    size_t at = 0;
    if (!read_state(state, len, &at, &s)) return 1;
    const Ctx ctx = Ctx::make(s);
    write_public_features(s, ctx, features);
    for (int p = 0; p < 2; ++p) {
        uint8_t fd = 0;
        for (int u = 0; u < N_UNITS; ++u) fd += s.zones[p][Z_FACEDOWN][u];
        sizes[p] = s.hand_size((uint8_t)p);
        sizes[2 + p] = fd;
        sizes[4 + p] = s.bag_size((uint8_t)p);
    }
    return 0;
}

}  // extern "C"
