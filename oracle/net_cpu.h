// TEST INFRASTRUCTURE — the CPU oracle. Only tests/, __graft_entry__.smoke()
// and bench.py's CPU-baseline leg use anything under oracle/; the product
// never links it.
//
// The fixed v5 value network on the CPU, restating engine/src/net.rs of the
// reference: the flat blob layout (net.rs:190-324), the naive row-major GEMM
// with sequential k accumulation (net.rs:102-122), tanh-form GELU
// (net.rs:126-129), LayerNorm eps 1e-5 (net.rs:380-405) and the solver's
// pieces cards/board/join_cache/configs/join/values (net.rs:544-853).
#pragma once
#include <cstddef>
#include <cstdint>
#include <vector>

namespace oracle {

constexpr int TYPE = 64, C = 96, BLOCKS = 8, D = 256, POOL = 64, CFGH = 128, JW = 128, JBLOCKS = 3;
constexpr int JOIN_IN = 2 * POOL + 1;

struct Span { size_t w, b, i, o; bool has_b; };

struct Layout {
    Span card[2], pile;
    size_t seat;
    Span hex_stem, tok_stem;
    size_t pos;
    Span glob_stem;
    Span mix[BLOCKS], pool[BLOCKS], out[BLOCKS];
    Span board_out, cfg1, cfg_f, cfg_g, cfg_m, join_p, join_b, join_w[JBLOCKS], join_out;
    size_t value_bias;
    std::vector<size_t> norm_g, norm_b, norm_width;
    size_t w_len, b_len, ln_len;
    Layout();
};

struct Net {
    Layout L;
    std::vector<float> w, b, ln;
    bool empty = true;

    void cards(const float* card_feat /*2 views x NTYPE x CARD_FEATS*/, std::vector<float>& out) const;
    // Board vectors P[rows, D] from expanded public rows xpub[rows, PUBFEAT]
    // (the unmirrored seat-0 encodings) with the view-0 card tokens.
    void board(const float* xpub, const float* cards, size_t rows, std::vector<float>& out) const;
    void join_cache(const float* p, size_t rows, std::vector<float>& out) const;
    void configs(const float* phi, const uint8_t* owner, size_t n, const float* cards, std::vector<float>& f,
                 std::vector<float>& g) const;
    void join(const float* p, const float* jp, const float* pooled, size_t rows, int player,
              std::vector<float>& h) const;
    float value(const float* h, const float* f_row) const;
};

float gelu(float x);
void gemm(size_t m, size_t n, size_t k, const float* a, size_t lda, const float* b, size_t ldb, float beta,
          float* c, size_t ldc);

}  // namespace oracle
