// TEST INFRASTRUCTURE — CPU oracle of the v5 value network (net.rs).
#include "net_cpu.h"

#include <cmath>
#include <limits>

#include "../war-chest-bot-9000-_b200/csrc/host/detmath.h"
#include "../war-chest-bot-9000-_b200/csrc/host/pbs.h"

namespace oracle {

using wc::CARD_FEATS;
using wc::CFEAT;
using wc::HEX_CH;
using wc::HEX_FACTS;
using wc::LOOSE;
using wc::N_HEXES;
using wc::NSLOT;
using wc::NTYPE;
using wc::OFF_LOOSE;
using wc::OFF_PILES;
using wc::PILE_COUNTS;
using wc::PUBFEAT;

// net.rs:230-324: hand out offsets in blob order.
Layout::Layout() {
    size_t cw = 0, cb = 0, cl = 0;
    auto lin = [&](size_t i, size_t o, bool bias) {
        Span s{cw, bias ? cb : (size_t)-1, i, o, bias};
        cw += i * o;
        if (bias) cb += o;
        return s;
    };
    auto embed = [&](size_t n) { size_t at = cw; cw += n; return at; };
    card[0] = lin(CARD_FEATS, TYPE, true);
    card[1] = lin(TYPE, TYPE, true);
    pile = lin(PILE_COUNTS, TYPE, false);
    seat = embed(2 * TYPE);
    hex_stem = lin(HEX_FACTS, C, true);
    tok_stem = lin(TYPE, C, false);
    pos = embed(N_HEXES * C);
    glob_stem = lin(LOOSE, C, false);
    for (int i = 0; i < BLOCKS; ++i) {
        mix[i] = lin(2 * C, C, true);
        pool[i] = lin(2 * C, C, true);
        out[i] = lin(C, C, true);
    }
    board_out = lin(2 * C + LOOSE, D, true);
    cfg1 = lin(3 + TYPE, CFGH, true);
    cfg_f = lin(CFGH, D, true);
    cfg_g = lin(CFGH, POOL, true);
    cfg_m = lin(TYPE, 3 * POOL, false);
    join_p = lin(D, JW, false);
    join_b = lin(JOIN_IN, JW, true);
    for (int i = 0; i < JBLOCKS; ++i) join_w[i] = lin(JW, JW, true);
    join_out = lin(JW, D, true);
    value_bias = cb;
    cb += 1;
    for (int i = 0; i < BLOCKS; ++i) { norm_width.push_back(C); norm_width.push_back(C); }
    norm_width.push_back(C);
    norm_width.push_back(CFGH);
    for (int i = 0; i < JBLOCKS; ++i) norm_width.push_back(JW);
    norm_width.push_back(JW);
    norm_width.push_back(D);
    for (size_t wd : norm_width) {
        norm_g.push_back(cl);
        norm_b.push_back(cl + wd);
        cl += 2 * wd;
    }
    w_len = cw;
    b_len = cb;
    ln_len = cl;
}

constexpr int LN_TRUNK = 2 * BLOCKS, LN_CFG = LN_TRUNK + 1, LN_JOIN = LN_CFG + 1, LN_JOUT = LN_JOIN + JBLOCKS,
              LN_H = LN_JOUT + 1;

// GELU, tanh form (net.rs:126-129). tanh is the deterministic Cephes-method
// tanh shared with the kernels (within 1 ulp of a correctly rounded tanh; the
// reference's platform tanhf is within 2), so the fp32 device network can be
// checked bit for bit.
float gelu(float x) { return wc::det_gelu(x); }

// net.rs:67-123, the non-Apple loop.
void gemm(size_t m, size_t n, size_t k, const float* a, size_t lda, const float* b, size_t ldb, float beta,
          float* c, size_t ldc) {
    if (m == 0 || n == 0) return;
    for (size_t i = 0; i < m; ++i) {
        float* row = c + i * ldc;
        if (beta == 0.0f) {
            for (size_t j = 0; j < n; ++j) row[j] = 0.0f;
        } else if (beta != 1.0f) {
            for (size_t j = 0; j < n; ++j) row[j] *= beta;
        }
        for (size_t p = 0; p < k; ++p) {
            float av = a[i * lda + p];
            if (av == 0.0f) continue;
            const float* brow = b + p * ldb;
            for (size_t j = 0; j < n; ++j) row[j] += av * brow[j];
        }
    }
}

namespace {

struct Lin {
    const float* w;
    const float* b;
    size_t i, o;
    void run(const float* in, size_t rows, std::vector<float>& out) const {
        if (out.size() < rows * o) out.resize(rows * o);
        gemm(rows, o, i, in, i, w, o, 0.0f, out.data(), o);
        bias(out.data(), rows);
    }
    void add(const float* in, size_t rows, float* out) const { gemm(rows, o, i, in, i, w, o, 1.0f, out, o); }
    void bias(float* out, size_t rows) const {
        if (!b) return;
        for (size_t r = 0; r < rows; ++r)
            for (size_t j = 0; j < o; ++j) out[r * o + j] += b[j];
    }
};

Lin mk(const Net& n, const Span& s) { return Lin{n.w.data() + s.w, s.has_b ? n.b.data() + s.b : nullptr, s.i, s.o}; }

void norm_rows(const Net& n, int which, float* x, size_t rows, bool act) {
    size_t width = n.L.norm_width[which];
    const float* g = n.ln.data() + n.L.norm_g[which];
    const float* bt = n.ln.data() + n.L.norm_b[which];
    for (size_t r = 0; r < rows; ++r) {
        float* row = x + r * width;
        float s = 0.0f;
        for (size_t j = 0; j < width; ++j) s += row[j];
        float mean = s / (float)width;
        float v = 0.0f;
        for (size_t j = 0; j < width; ++j) v += (row[j] - mean) * (row[j] - mean);
        float var = v / (float)width;
        float inv = 1.0f / std::sqrt(var + 1e-5f);
        for (size_t j = 0; j < width; ++j) row[j] = (row[j] - mean) * inv * g[j] + bt[j];
        if (act)
            for (size_t j = 0; j < width; ++j) row[j] = gelu(row[j]);
    }
}

}  // namespace

// net.rs:544-555. card_feat holds both views' NTYPE card-fact rows.
void Net::cards(const float* card_feat, std::vector<float>& out) const {
    std::vector<float> hidden;
    mk(*this, L.card[0]).run(card_feat, 2 * NTYPE, hidden);
    for (size_t i = 0; i < (size_t)2 * NTYPE * TYPE; ++i) hidden[i] = gelu(hidden[i]);
    mk(*this, L.card[1]).run(hidden.data(), 2 * NTYPE, out);
}

// net.rs:558-724 (tokens, stem, trunk, board) for the physical rows.
void Net::board(const float* xpub, const float* cards, size_t rows, std::vector<float>& out) const {
    const wc::Board& bd = wc::board();
    // tokens
    std::vector<float> piles(rows * NTYPE * PILE_COUNTS);
    for (size_t r = 0; r < rows; ++r)
        for (int q = 0; q < NTYPE * PILE_COUNTS; ++q) piles[r * NTYPE * PILE_COUNTS + q] = xpub[r * PUBFEAT + OFF_PILES + q];
    std::vector<float> tokens(rows * NTYPE * TYPE, 0.0f);
    mk(*this, L.pile).add(piles.data(), rows * NTYPE, tokens.data());
    const float* seat = w.data() + L.seat;
    for (size_t r = 0; r < rows; ++r)
        for (int t = 0; t < NTYPE; ++t) {
            const float* card = cards + t * TYPE;  // view 0
            const float* st = seat + (t / NSLOT) * TYPE;
            float* dst = tokens.data() + (r * NTYPE + t) * TYPE;
            for (int j = 0; j < TYPE; ++j) dst[j] += card[j] + st[j];
        }
    // stem
    size_t cells = rows * N_HEXES;
    std::vector<float> facts(cells * HEX_FACTS), occ(cells * C, 0.0f), loose(rows * LOOSE), projected;
    mk(*this, L.tok_stem).run(tokens.data(), rows * NTYPE, projected);
    std::vector<float> type_pool(rows * C, 0.0f);
    for (size_t r = 0; r < rows; ++r) {
        for (int t = 0; t < NTYPE; ++t) {
            const float* token = projected.data() + (r * NTYPE + t) * C;
            for (int j = 0; j < C; ++j) type_pool[r * C + j] += gelu(token[j]) / (float)NTYPE;
        }
        const float* src = xpub + r * PUBFEAT;
        for (int j = 0; j < LOOSE; ++j) loose[r * LOOSE + j] = src[OFF_LOOSE + j];
        for (int h = 0; h < N_HEXES; ++h) {
            const float* hex = src + h * HEX_CH;
            for (int j = 0; j < HEX_FACTS; ++j) facts[(r * N_HEXES + h) * HEX_FACTS + j] = hex[j];
            for (int t = 0; t < NTYPE; ++t)
                if (hex[HEX_FACTS + t] != 0.0f) {
                    const float* s2 = projected.data() + (r * NTYPE + t) * C;
                    for (int j = 0; j < C; ++j) occ[(r * N_HEXES + h) * C + j] = s2[j];
                    break;
                }
        }
    }
    std::vector<float> x, glob;
    mk(*this, L.hex_stem).run(facts.data(), cells, x);
    mk(*this, L.glob_stem).run(loose.data(), rows, glob);
    const float* pos = w.data() + L.pos;
    for (size_t r = 0; r < rows; ++r)
        for (int h = 0; h < N_HEXES; ++h) {
            float* dst = x.data() + (r * N_HEXES + h) * C;
            const float* o = occ.data() + (r * N_HEXES + h) * C;
            for (int j = 0; j < C; ++j) dst[j] += o[j] + pos[h * C + j] + glob[r * C + j] + type_pool[r * C + j];
        }
    // trunk
    std::vector<float> a(cells * C), mixed(cells * 2 * C), pooled(rows * 2 * C), y, gb, z;
    for (int i = 0; i < BLOCKS; ++i) {
        for (size_t q = 0; q < cells * C; ++q) a[q] = x[q];
        norm_rows(*this, 2 * i, a.data(), cells, true);
        for (size_t cell = 0; cell < cells; ++cell) {
            size_t h = cell % N_HEXES;
            float* self_part = mixed.data() + cell * 2 * C;
            float* neigh = self_part + C;
            for (int j = 0; j < C; ++j) { self_part[j] = a[cell * C + j]; neigh[j] = 0.0f; }
            for (int d = 0; d < 6; ++d) {
                uint8_t nb = bd.neighbors[h][d];
                if (nb == wc::NONE) continue;
                const float* s2 = a.data() + (cell - h + nb) * C;
                for (int j = 0; j < C; ++j) neigh[j] += s2[j];
            }
        }
        mk(*this, L.mix[i]).run(mixed.data(), cells, y);
        for (size_t r = 0; r < rows; ++r) {
            float* mean = pooled.data() + r * 2 * C;
            float* mx = mean + C;
            for (int j = 0; j < C; ++j) { mean[j] = 0.0f; mx[j] = -std::numeric_limits<float>::infinity(); }
            for (int h = 0; h < N_HEXES; ++h) {
                const float* s2 = a.data() + (r * N_HEXES + h) * C;
                for (int j = 0; j < C; ++j) {
                    mean[j] += s2[j] / (float)N_HEXES;
                    mx[j] = std::fmax(mx[j], s2[j]);
                }
            }
        }
        mk(*this, L.pool[i]).run(pooled.data(), rows, gb);
        for (size_t cell = 0; cell < cells; ++cell)
            for (int j = 0; j < C; ++j) y[cell * C + j] += gb[(cell / N_HEXES) * C + j];
        norm_rows(*this, 2 * i + 1, y.data(), cells, true);
        mk(*this, L.out[i]).run(y.data(), cells, z);
        for (size_t q = 0; q < cells * C; ++q) x[q] += z[q];
    }
    norm_rows(*this, LN_TRUNK, x.data(), cells, true);
    // board readout
    size_t width = 2 * C + LOOSE;
    std::vector<float> input(rows * width);
    for (size_t r = 0; r < rows; ++r) {
        float* dst = input.data() + r * width;
        for (int j = 0; j < C; ++j) { dst[j] = 0.0f; dst[C + j] = -std::numeric_limits<float>::infinity(); }
        for (int h = 0; h < N_HEXES; ++h) {
            const float* s2 = x.data() + (r * N_HEXES + h) * C;
            for (int j = 0; j < C; ++j) {
                dst[j] += s2[j] / (float)N_HEXES;
                dst[C + j] = std::fmax(dst[C + j], s2[j]);
            }
        }
        for (int j = 0; j < LOOSE; ++j) dst[2 * C + j] = xpub[r * PUBFEAT + OFF_LOOSE + j];
    }
    mk(*this, L.board_out).run(input.data(), rows, out);
}

void Net::join_cache(const float* p, size_t rows, std::vector<float>& out) const {
    mk(*this, L.join_p).run(p, rows, out);
}

// net.rs:735-797.
void Net::configs(const float* phi, const uint8_t* owner, size_t n, const float* cards, std::vector<float>& f,
                  std::vector<float>& g) const {
    // A subgame with no network rows interns no configs and builds no card
    // table (net.rs:778: the card views are counted from the table, so an
    // empty one runs no product): nothing to encode, and `cards` is unset.
    if (n == 0) {
        f.clear();
        g.clear();
        return;
    }
    size_t width = 3 + TYPE;
    std::vector<float> slots(n * NSLOT * width);
    for (size_t c = 0; c < n; ++c) {
        size_t q = owner[c];
        for (int k = 0; k < NSLOT; ++k) {
            float* row = slots.data() + (c * NSLOT + k) * width;
            row[0] = phi[c * CFEAT + k];
            row[1] = phi[c * CFEAT + NSLOT + k];
            row[2] = phi[c * CFEAT + 2 * NSLOT + k];
            for (int j = 0; j < TYPE; ++j) row[3 + j] = cards[(q * NTYPE + k) * TYPE + j];
        }
    }
    std::vector<float> hidden;
    mk(*this, L.cfg1).run(slots.data(), n * NSLOT, hidden);
    for (size_t i = 0; i < n * NSLOT * CFGH; ++i) hidden[i] = gelu(hidden[i]);
    std::vector<float> u(n * CFGH, 0.0f);
    for (size_t c = 0; c < n; ++c)
        for (int k = 0; k < NSLOT; ++k)
            for (int j = 0; j < CFGH; ++j) u[c * CFGH + j] += hidden[(c * NSLOT + k) * CFGH + j];
    norm_rows(*this, LN_CFG, u.data(), n, true);
    mk(*this, L.cfg_f).run(u.data(), n, f);
    mk(*this, L.cfg_g).run(u.data(), n, g);
    std::vector<float> bag;
    mk(*this, L.cfg_m).run(cards, 2 * NTYPE, bag);
    size_t stride = 3 * POOL;
    for (size_t c = 0; c < n; ++c) {
        size_t q = owner[c];
        float* dst = g.data() + c * POOL;
        for (int k = 0; k < NSLOT; ++k) {
            const float* v = bag.data() + (q * NTYPE + k) * stride;
            for (int zone = 0; zone < 3; ++zone) {
                float count = phi[c * CFEAT + zone * NSLOT + k];
                if (count == 0.0f) continue;
                for (int j = 0; j < POOL; ++j) dst[j] += count * v[zone * POOL + j];
            }
        }
    }
}

// net.rs:801-841.
void Net::join(const float* p, const float* jp, const float* pooled, size_t rows, int player,
               std::vector<float>& h) const {
    std::vector<float> z(rows * JW), input(rows * JOIN_IN);
    for (size_t r = 0; r < rows; ++r) {
        size_t q = 2 * r + player, o = 2 * r + 1 - player;
        float* dst = input.data() + r * JOIN_IN;
        for (int j = 0; j < POOL; ++j) { dst[j] = pooled[q * POOL + j]; dst[POOL + j] = pooled[o * POOL + j]; }
        dst[2 * POOL] = player == 0 ? -1.0f : 1.0f;
        for (int j = 0; j < JW; ++j) z[r * JW + j] = jp[r * JW + j];
    }
    Lin jb = mk(*this, L.join_b);
    jb.add(input.data(), rows, z.data());
    jb.bias(z.data(), rows);
    std::vector<float> t(rows * JW), d;
    for (int i = 0; i < JBLOCKS; ++i) {
        t = z;
        norm_rows(*this, LN_JOIN + i, t.data(), rows, true);
        mk(*this, L.join_w[i]).run(t.data(), rows, d);
        for (size_t q = 0; q < rows * JW; ++q) z[q] += d[q];
    }
    norm_rows(*this, LN_JOUT, z.data(), rows, true);
    h.assign(p, p + rows * D);
    Lin jo = mk(*this, L.join_out);
    jo.add(z.data(), rows, h.data());
    jo.bias(h.data(), rows);
    norm_rows(*this, LN_H, h.data(), rows, false);
}

float Net::value(const float* h, const float* f_row) const {
    float v = b[L.value_bias];
    for (int j = 0; j < D; ++j) v += f_row[j] * h[j];
    return v;
}

}  // namespace oracle
