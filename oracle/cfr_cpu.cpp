// TEST INFRASTRUCTURE — CPU oracle of the subgame solver (search.rs).
#include "cfr_cpu.h"

#include <algorithm>
#include <cmath>
#include <limits>
#include <stdexcept>

namespace oracle {

using wc::NK_CHANCE;
using wc::NK_LEAF;
using wc::NO_TRANS;
using wc::NSLOT;
using wc::NTYPE;
using wc::PUBFEAT;

const float* Solver::reach_of(uint32_t i, int p) const {
    return reach.data() + roff[i] + (p == 1 ? t.nc(i, 0) : 0);
}
float* Solver::reach_of(uint32_t i, int p) { return reach.data() + roff[i] + (p == 1 ? t.nc(i, 0) : 0); }

// search.rs:801-875.
Solver::Solver(const wc::Tree& tree, const Net* n) : t(tree), net(n) {
    snap_list = wc::snapshot_iters(t.cfg.iters);
    size_t nn = t.nodes.size(), nc = t.ncells();
    regret.assign(nc, 0.0f);
    cur.assign(nc, 0.0f);
    sum.assign(nc, 0.0f);
    size_t r = 0, v = 0;
    for (uint32_t i = 0; i < nn; ++i) {
        roff.push_back((uint32_t)r);
        voff.push_back((uint32_t)v);
        size_t c0 = t.nc(i, 0), c1 = t.nc(i, 1);
        r += c0 + c1;
        v += std::max(c0, c1);
        const wc::NodeRec& nd = t.nodes[i];
        uint32_t so = t.soff[i], cells = t.soff[i + 1] - so;
        if (cells > 0) {
            size_t ncp = t.nc(i, nd.player);
            for (size_t c = 0; c < ncp; ++c) {
                uint32_t lo = t.legal_off[nd.row_off + c], hi = t.legal_off[nd.row_off + c + 1];
                float k = (float)(hi - lo);
                for (uint32_t cell = lo; cell < hi; ++cell) cur[so + cell] = 1.0f / k;
            }
        }
    }
    voff.push_back((uint32_t)v);
    reach.assign(r, 0.0f);
    vals.assign(v, 0.0f);
    precompute_reaches();
    for (uint32_t i = 0; i < nn; ++i) {
        const wc::NodeRec& nd = t.nodes[i];
        uint32_t so = t.soff[i];
        if (nd.kind != wc::NK_DECISION || t.soff[i + 1] == so) continue;
        int p = nd.player;
        for (size_t c = 0; c < t.nc(i, p); ++c) {
            float rr = reach_of(i, p)[c];
            for (uint32_t cell = t.legal_off[nd.row_off + c]; cell < t.legal_off[nd.row_off + c + 1]; ++cell)
                sum[so + cell] += rr * cur[so + cell];
        }
    }
    // snapshot_initial (search.rs:882-888)
    snap_t = 1;
    if (t.cfg.snapshots || t.cfg.iters == 0) snaps.push_back(cur);
}

void Solver::precompute_reaches() {
    propagate(cur, t.root_belief[0].p.data(), t.root_belief[1].p.data());
}

// search.rs:1273-1351.
void Solver::propagate(const std::vector<float>& strat, const float* root0, const float* root1) {
    std::fill(reach.begin(), reach.end(), 0.0f);
    size_t n0 = t.nc(0, 0), n1 = t.nc(0, 1);
    std::copy(root0, root0 + n0, reach.begin() + roff[0]);
    std::copy(root1, root1 + n1, reach.begin() + roff[0] + n0);
    for (uint32_t i = 0; i < t.nodes.size(); ++i) {
        const wc::NodeRec& n = t.nodes[i];
        if (n.kind == NK_LEAF) continue;
        int me = n.player, op = 1 - me;
        const float* src_me = reach_of(i, me);
        const float* src_op = reach_of(i, op);
        size_t nme = t.nc(i, me), nop = t.nc(i, op);
        if (n.kind == NK_CHANCE) {
            uint32_t c = t.child[n.child_off];
            float* dst_me = reach_of(c, me);
            float* dst_op = reach_of(c, op);
            std::copy(src_op, src_op + nop, dst_op);
            for (size_t ci = 0; ci < nme; ++ci) {
                float w = src_me[ci];
                if (w == 0.0f) continue;
                for (uint32_t k = t.draw_start[n.draw_off + ci]; k < t.draw_start[n.draw_off + ci + 1]; ++k)
                    dst_me[t.draw_to[k]] += w * t.draw_p[k];
            }
            continue;
        }
        const float* cs = strat.data() + t.soff[i];
        for (uint32_t ch = 0; ch < n.nch; ++ch) {
            uint32_t c = t.child[n.child_off + ch];
            float* dst_me = reach_of(c, me);
            float* dst_op = reach_of(c, op);
            std::copy(src_op, src_op + nop, dst_op);
            uint32_t s0 = t.obs_start[n.obs_off + ch], s1 = t.obs_start[n.obs_off + ch + 1];
            for (uint32_t j = s0; j < s1; ++j) {
                uint32_t a = t.obs_act[n.act_off + j];
                for (uint32_t x = t.action_off[n.aoff_off + a]; x < t.action_off[n.aoff_off + a + 1]; ++x) {
                    uint32_t cell = t.action_cell[t.soff[i] + x];
                    uint32_t tr = t.legal_trans[t.soff[i] + cell];
                    if (tr == NO_TRANS) continue;
                    uint32_t ci = t.cell_row[t.soff[i] + cell];
                    dst_me[tr] += src_me[ci] * cs[cell];
                }
            }
        }
    }
}

// search.rs:1654-1803.
void Solver::backprop(int traverser, const std::vector<float>* strat, Back mode) {
    const float EPS = 1e-6f;
    float da = 0, db = 0, dg = 0;
    const wc::CfrRule& k = t.cfg.cfr;
    if (mode == Back::Regret) {
        float m = (float)steps[traverser] + 1.0f;
        da = wc::cfr_factor(m, k.alpha);
        db = wc::cfr_factor(m, k.beta);
        dg = std::pow(m / (m + 1.0f), k.gamma);
    }
    for (int64_t ii = (int64_t)t.nodes.size() - 1; ii >= 0; --ii) {
        uint32_t i = (uint32_t)ii;
        const wc::NodeRec& n = t.nodes[i];
        if (n.kind == NK_LEAF) continue;
        int me = n.player;
        size_t nc = t.nc(i, traverser);
        if (n.kind == NK_CHANCE) {
            uint32_t ch = t.child[n.child_off];
            float* dst = vals.data() + voff[i];
            const float* src = vals.data() + voff[ch];
            if (me == traverser) {
                for (size_t c = 0; c < nc; ++c) {
                    float v = 0.0f;
                    for (uint32_t q = t.draw_start[n.draw_off + c]; q < t.draw_start[n.draw_off + c + 1]; ++q)
                        v += t.draw_p[q] * src[t.draw_to[q]];
                    dst[c] = v;
                }
            } else {
                std::copy(src, src + nc, dst);
            }
            continue;
        }
        float* vi = vals.data() + voff[i];
        bool br = mode == Back::BestResponse && me == traverser;
        std::fill(vi, vi + nc, br ? -std::numeric_limits<float>::infinity() : 0.0f);
        uint32_t so = t.soff[i];
        if (me == traverser) {
            for (uint32_t a = 0; a < n.na; ++a) {
                for (uint32_t x = t.action_off[n.aoff_off + a]; x < t.action_off[n.aoff_off + a + 1]; ++x) {
                    uint32_t cell = t.action_cell[so + x];
                    uint32_t tr = t.legal_trans[so + cell];
                    if (tr == NO_TRANS) continue;
                    uint32_t chn = t.legal_child[so + cell];
                    uint32_t c = t.cell_row[so + cell];
                    float av = vals[voff[chn] + tr];
                    if (mode == Back::Regret) vi[c] += av * cur[so + cell];
                    else if (mode == Back::Value) vi[c] += av * (*strat)[so + cell];
                    else vi[c] = std::fmax(vi[c], av);
                }
            }
            if (mode == Back::Regret) {
                for (size_t c = 0; c < nc; ++c) {
                    float base = vi[c];
                    uint32_t lo = t.legal_off[n.row_off + c], hi = t.legal_off[n.row_off + c + 1];
                    float s = 0.0f;
                    for (uint32_t cell = lo; cell < hi; ++cell) {
                        float delta = 0.0f;
                        uint32_t tr = t.legal_trans[so + cell];
                        if (tr != NO_TRANS) delta += vals[voff[t.legal_child[so + cell]] + tr];
                        delta -= base;
                        uint32_t at = so + cell;
                        float old = regret[at];
                        float r = old * (old > 0.0f ? da : db) + delta;
                        regret[at] = r;
                        float v = std::fmax(r + k.predict * delta, EPS);
                        cur[at] = v;
                        s += v;
                    }
                    if (s > 0.0f) {
                        float inv = 1.0f / s;
                        for (uint32_t cell = lo; cell < hi; ++cell) cur[so + cell] *= inv;
                    }
                }
                for (uint32_t cell = so; cell < t.soff[i + 1]; ++cell) sum[cell] *= dg;
            } else if (mode == Back::BestResponse) {
                for (size_t c = 0; c < nc; ++c)
                    if (vi[c] == -std::numeric_limits<float>::infinity()) vi[c] = 0.0f;
            }
        } else {
            for (uint32_t ch = 0; ch < n.nch; ++ch) {
                const float* cv = vals.data() + voff[t.child[n.child_off + ch]];
                for (size_t c = 0; c < nc; ++c) vi[c] += cv[c];
            }
        }
    }
}

// search.rs:1464-1499 (the network pieces that do not move between iterations).
void Solver::ensure_leaf_batch() {
    if (batch_ready) return;
    batch_ready = true;
    if (!net_ready()) return;
    size_t rows = t.leaf_rows.size();
    xb.assign(2 * rows * POOL, 0.0f);
    std::vector<float> card_feat(2 * NTYPE * wc::CARD_FEATS);
    for (int view = 0; view < 2; ++view)
        for (int ty = 0; ty < NTYPE; ++ty)
            wc::write_card_features(t.ids[view][ty], card_feat.data() + (view * NTYPE + ty) * wc::CARD_FEATS);
    if (rows > 0) net->cards(card_feat.data(), cards);
    std::vector<float> xpub(rows * PUBFEAT);
    for (size_t r = 0; r < rows; ++r)
        wc::expand_gpu_row(t.gpu_rows.data() + r * wc::GPU_ROW_BYTES, t.ids[0], xpub.data() + r * PUBFEAT);
    net->board(xpub.data(), cards.data(), rows, pb);
    net->join_cache(pb.data(), rows, jp);
    net->configs(t.cphi.data(), t.cplayer.data(), t.ncfg, cards.data(), cf, cg);
}

// search.rs:1512-1547.
void Solver::belief_blocks(int only) {
    std::vector<float> w;
    for (size_t r = 0; r < t.leaf_rows.size(); ++r) {
        uint32_t i = t.leaf_rows[r];
        for (int p = 0; p < 2; ++p) {
            if (only >= 0 && only != p) continue;
            size_t n = t.nc(i, p);
            w.resize(n);
            wc::normalize_weights(reach_of(i, p), n, w.data());
            size_t q = 2 * r + p;
            const uint32_t* idx = t.leaf_cidx.data() + t.leaf_coff[q];
            float* out = xb.data() + q * POOL;
            for (int j = 0; j < POOL; ++j) out[j] = 0.0f;
            for (size_t c = 0; c < n; ++c) {
                const float* row = cg.data() + (size_t)idx[c] * POOL;
                for (int j = 0; j < POOL; ++j) out[j] += w[c] * row[j];
            }
        }
    }
}

void Solver::pbs_head(int traverser) {
    if (!net_ready()) return;
    net->join(pb.data(), jp.data(), xb.data(), t.leaf_rows.size(), traverser, h);
}

// search.rs:1587-1636.
void Solver::readout(int p) {
    int opp = 1 - p;
    for (uint32_t i : t.term_leaves) {
        const float* ro = reach_of(i, opp);
        float opp_reach = 0.0f;
        for (size_t c = 0; c < t.nc(i, opp); ++c) opp_reach += ro[c];
        float u = p == t.nodes[i].player ? t.nodes[i].util : -t.nodes[i].util;
        float* v = vals.data() + voff[i];
        for (size_t c = 0; c < t.nc(i, p); ++c) v[c] = u * opp_reach;
    }
    for (size_t r = 0; r < t.leaf_rows.size(); ++r) {
        uint32_t i = t.leaf_rows[r];
        const float* ro = reach_of(i, opp);
        float opp_reach = 0.0f;
        for (size_t c = 0; c < t.nc(i, opp); ++c) opp_reach += ro[c];
        size_t n = t.nc(i, p);
        float* v = vals.data() + voff[i];
        if (!net_ready()) {
            for (size_t c = 0; c < n; ++c) v[c] = 0.0f;
            continue;
        }
        const uint32_t* idx = t.leaf_cidx.data() + t.leaf_coff[2 * r + p];
        for (size_t c = 0; c < n; ++c) v[c] = net->value(h.data() + r * D, cf.data() + (size_t)idx[c] * D);
        for (size_t c = 0; c < n; ++c) v[c] *= opp_reach;
    }
}

void Solver::leaf_values(int traverser) {
    ensure_leaf_batch();
    int redo = last_traverser;
    last_traverser = traverser;
    if (net_ready()) belief_blocks(redo);
    pbs_head(traverser);
    readout(traverser);
}

void Solver::avg_block(int traverser) {
    avg_touched[traverser] = true;
    for (uint32_t i = 0; i < t.nodes.size(); ++i) {
        const wc::NodeRec& n = t.nodes[i];
        if (n.kind != wc::NK_DECISION || n.player != traverser) continue;
        uint32_t so = t.soff[i];
        for (size_t c = 0; c < t.nc(i, traverser); ++c) {
            float r = reach_of(i, traverser)[c];
            for (uint32_t cell = t.legal_off[n.row_off + c]; cell < t.legal_off[n.row_off + c + 1]; ++cell)
                sum[so + cell] += r * cur[so + cell];
        }
    }
}

// search.rs:899-938.
void Solver::snapshot() {
    int tt = snap_t++;
    bool keep = t.cfg.snapshots ? std::find(snap_list.begin(), snap_list.end(), tt) != snap_list.end()
                                : tt == t.cfg.iters;
    if (!keep) return;
    std::vector<float> snap = cur;
    for (uint32_t i = 0; i < t.nodes.size(); ++i) {
        const wc::NodeRec& n = t.nodes[i];
        if (n.kind != wc::NK_DECISION || !avg_touched[n.player]) continue;
        uint32_t so = t.soff[i];
        for (size_t c = 0; c < t.nc(i, n.player); ++c) {
            uint32_t lo = t.legal_off[n.row_off + c], hi = t.legal_off[n.row_off + c + 1];
            float s = 0.0f;
            for (uint32_t cell = lo; cell < hi; ++cell) s += sum[so + cell];
            float k = (float)std::max<uint32_t>(hi - lo, 1);
            for (uint32_t cell = lo; cell < hi; ++cell) snap[so + cell] = s > 0.0f ? sum[so + cell] / s : 1.0f / k;
        }
    }
    snaps.push_back(std::move(snap));
}

void Solver::step(int traverser) {
    leaf_values(traverser);
    backprop(traverser, nullptr, Back::Regret);
    precompute_reaches();
    avg_block(traverser);
    snapshot();
    steps[traverser] += 1;
}

void Solver::multistep(int iters) {
    for (int i = 0; i < iters; ++i) step(i % 2);
}

// search.rs:1851-1871.
std::vector<std::vector<float>> Solver::value_under(const std::vector<std::vector<float>>& roots) {
    std::vector<float> reference = snaps.back();
    std::vector<std::vector<float>> out;
    size_t n0 = t.nc(0, 0);
    for (const std::vector<float>& root : roots) {
        propagate(reference, root.data(), root.data() + n0);
        ensure_leaf_batch();
        last_traverser = -1;
        if (net_ready()) belief_blocks(-1);
        std::vector<float> pair;
        for (int p = 0; p < 2; ++p) {
            pbs_head(p);
            readout(p);
            backprop(p, &reference, Back::Value);
            size_t n = t.nc(0, p);
            pair.insert(pair.end(), vals.begin() + voff[0], vals.begin() + voff[0] + n);
        }
        out.push_back(std::move(pair));
    }
    precompute_reaches();
    last_traverser = -1;
    return out;
}

// search.rs:1884-1906.
void Solver::nash_conv(float* nash, float* zero_sum) {
    std::vector<float> reference = snaps.back();
    propagate(reference, t.root_belief[0].p.data(), t.root_belief[1].p.data());
    ensure_leaf_batch();
    last_traverser = -1;
    if (net_ready()) belief_blocks(-1);
    float nsh = 0.0f, zs = 0.0f;
    for (int p = 0; p < 2; ++p) {
        pbs_head(p);
        readout(p);
        const float* root = t.root_belief[p].p.data();
        size_t nc = t.nc(0, p);
        auto expect = [&]() {
            float s = 0.0f;
            for (size_t c = 0; c < nc; ++c) s += root[c] * vals[voff[0] + c];
            return s;
        };
        backprop(p, &reference, Back::Value);
        float v = expect();
        backprop(p, &reference, Back::BestResponse);
        nsh += expect() - v;
        zs += v;
    }
    precompute_reaches();
    last_traverser = -1;
    *nash = nsh;
    *zero_sum = zs;
}

// search.rs:1937-1956.
std::vector<std::vector<float>> Solver::carried_beliefs(uint32_t leaf) {
    std::vector<std::vector<float>> out;
    size_t n = snaps.empty() ? 0 : snaps.size() - 1;
    for (size_t i = 0; i < n; ++i) {
        std::vector<float> snap = snaps[i];
        propagate(snap, t.root_belief[0].p.data(), t.root_belief[1].p.data());
        std::vector<float> pair;
        for (int p = 0; p < 2; ++p) {
            size_t m = t.nc(leaf, p);
            std::vector<float> w(m);
            wc::normalize_weights(reach_of(leaf, p), m, w.data());
            pair.insert(pair.end(), w.begin(), w.end());
        }
        out.push_back(std::move(pair));
    }
    return out;
}

}  // namespace oracle
