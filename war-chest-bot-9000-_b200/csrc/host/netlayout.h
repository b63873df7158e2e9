// Offsets of every array in the v5 value-network blob: the contract between
// the trainer's flat() export and the engine (engine/src/net.rs:190-324,
// train/value_net.py:231). Three flat arrays: weights `w` (row-major
// [in, out] matrices and embeddings), biases `b` (plus the trailing value
// bias) and LayerNorm `(gamma, beta)` pairs `ln`, in blob order.
#pragma once
#include <cstddef>
#include <cstdint>

namespace wc {

constexpr int NET_TYPE = 64, NET_C = 96, NET_BLOCKS = 8, NET_D = 256, NET_POOL = 64, NET_CFGH = 128,
              NET_JW = 128, NET_JBLOCKS = 3;
constexpr int NET_JOIN_IN = 2 * NET_POOL + 1;
constexpr uint32_t NET_MODEL_TAG = 5;  // net.rs:41, the only dims NetLayout accepts

struct NetSpan {
    uint32_t w, b, i, o;  // b == UINT32_MAX: no bias
};

struct NetLayout {
    NetSpan card[2], pile;
    uint32_t seat;
    NetSpan hex_stem, tok_stem;
    uint32_t pos;
    NetSpan glob_stem;
    NetSpan mix[NET_BLOCKS], pool[NET_BLOCKS], out[NET_BLOCKS];
    NetSpan board_out, cfg1, cfg_f, cfg_g, cfg_m, join_p, join_b, join_w[NET_JBLOCKS], join_out;
    uint32_t value_bias;
    uint32_t norm_g[2 * NET_BLOCKS + 7], norm_b[2 * NET_BLOCKS + 7], norm_w[2 * NET_BLOCKS + 7];
    uint32_t w_len, b_len, ln_len;

    // LayerNorm indices in application order (net.rs:433-440).
#ifdef __CUDACC__
    __host__ __device__
#endif
    static constexpr int ln_block(int i, int half) { return 2 * i + half; }
    static constexpr int LN_TRUNK = 2 * NET_BLOCKS, LN_CFG = LN_TRUNK + 1, LN_JOIN = LN_CFG + 1,
                         LN_JOUT = LN_JOIN + NET_JBLOCKS, LN_H = LN_JOUT + 1, N_NORMS = LN_H + 1;

    static NetLayout make() {
        NetLayout L{};
        uint32_t cw = 0, cb = 0, cl = 0;
        auto lin = [&](uint32_t i, uint32_t o, bool bias) {
            NetSpan s{cw, bias ? cb : 0xFFFFFFFFu, i, o};
            cw += i * o;
            if (bias) cb += o;
            return s;
        };
        auto embed = [&](uint32_t n) { uint32_t at = cw; cw += n; return at; };
        const uint32_t CARD_FEATS = 25, PILE_COUNTS = 4, HEX_FACTS = 6, LOOSE = 15, N_HEXES = 37;
        L.card[0] = lin(CARD_FEATS, NET_TYPE, true);
        L.card[1] = lin(NET_TYPE, NET_TYPE, true);
        L.pile = lin(PILE_COUNTS, NET_TYPE, false);
        L.seat = embed(2 * NET_TYPE);
        L.hex_stem = lin(HEX_FACTS, NET_C, true);
        L.tok_stem = lin(NET_TYPE, NET_C, false);
        L.pos = embed(N_HEXES * NET_C);
        L.glob_stem = lin(LOOSE, NET_C, false);
        for (int i = 0; i < NET_BLOCKS; ++i) {
            L.mix[i] = lin(2 * NET_C, NET_C, true);
            L.pool[i] = lin(2 * NET_C, NET_C, true);
            L.out[i] = lin(NET_C, NET_C, true);
        }
        L.board_out = lin(2 * NET_C + LOOSE, NET_D, true);
        L.cfg1 = lin(3 + NET_TYPE, NET_CFGH, true);
        L.cfg_f = lin(NET_CFGH, NET_D, true);
        L.cfg_g = lin(NET_CFGH, NET_POOL, true);
        L.cfg_m = lin(NET_TYPE, 3 * NET_POOL, false);
        L.join_p = lin(NET_D, NET_JW, false);
        L.join_b = lin(NET_JOIN_IN, NET_JW, true);
        for (int i = 0; i < NET_JBLOCKS; ++i) L.join_w[i] = lin(NET_JW, NET_JW, true);
        L.join_out = lin(NET_JW, NET_D, true);
        L.value_bias = cb;
        cb += 1;
        int k = 0;
        auto norm = [&](uint32_t width) {
            L.norm_g[k] = cl;
            L.norm_b[k] = cl + width;
            L.norm_w[k] = width;
            cl += 2 * width;
            ++k;
        };
        for (int i = 0; i < NET_BLOCKS; ++i) { norm(NET_C); norm(NET_C); }
        norm(NET_C);
        norm(NET_CFGH);
        for (int i = 0; i < NET_JBLOCKS; ++i) norm(NET_JW);
        norm(NET_JW);
        norm(NET_D);
        L.w_len = cw;
        L.b_len = cb;
        L.ln_len = cl;
        return L;
    }
};

}  // namespace wc
