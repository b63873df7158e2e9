// Tree -> level-sorted job image.
#include "job.h"

#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <unordered_map>

namespace wc {

size_t JobImage::table_bytes() const {
    size_t b = 0;
    b += 4 * (cell_ref.size() + cell_vidx.size() + row_off.size() + vg_start.size() + vge_idx.size() +
              vge_w.size() + rg_start.size() + rge_src.size() + rge_w.size() + drawp.size() + lr_ridx.size() +
              lr_nc.size() + lr_vidx.size() + leaf_coff.size() + leaf_cidx.size() + tl_ridx.size() +
              tl_nc.size() + tl_vidx.size() + tl_util0.size() + cphi.size() + card_feat.size() + cfg_col.size() +
              root_belief.size() + carried.size() + row_rep.size() + row_gpu.size());
    b += row_player.size() + gpu_rows.size() + cplayer.size();
    return b;
}

std::unique_ptr<JobImage> flatten(const Tree& t, const std::vector<float>& carried, uint32_t ncarried) {
    if (t.capped) throw std::invalid_argument("a capped tree cannot be solved");
    auto j = std::make_unique<JobImage>();
    JobImage& J = *j;
    J.cfg = t.cfg;
    const uint32_t N = (uint32_t)t.nodes.size();
    J.nodes = N;
    J.ncells = (uint32_t)t.ncells();
    J.ndraw = (uint32_t)t.draw_to.size();
    J.nlevels = (uint32_t)t.max_depth() + 1;
    J.ncfg = (uint32_t)t.ncfg;
    J.root_nc[0] = (uint32_t)t.nc(0, 0);
    J.root_nc[1] = (uint32_t)t.nc(0, 1);
    for (int it : snapshot_iters(t.cfg.iters)) J.snap_iters.push_back((uint32_t)it);
    const uint32_t L = J.nlevels;
    auto nc = [&](uint32_t node, int p) { return (uint32_t)t.nc(node, p); };

    // parents and level groups
    std::vector<uint32_t> parent(N, 0xFFFFFFFFu), child_index(N, 0);
    for (uint32_t i = 0; i < N; ++i) {
        const NodeRec& n = t.nodes[i];
        if (n.kind == NK_LEAF) continue;
        for (uint32_t ch = 0; ch < n.nch; ++ch) {
            uint32_t c = t.child[n.child_off + ch];
            parent[c] = i;
            child_index[c] = ch;
        }
    }
    std::vector<std::vector<uint32_t>> dec[2], chance(L), leaves(L), all(L);
    dec[0].resize(L);
    dec[1].resize(L);
    for (uint32_t i = 0; i < N; ++i) {
        const NodeRec& n = t.nodes[i];
        all[n.depth].push_back(i);
        if (n.kind == NK_DECISION) dec[n.player][n.depth].push_back(i);
        else if (n.kind == NK_CHANCE) chance[n.depth].push_back(i);
        else leaves[n.depth].push_back(i);
    }

    // ---- cells and rows, sorted by (level, player, node, row)
    std::vector<uint32_t> sorted_of(J.ncells, 0);
    J.cell_ref.reserve(J.ncells);
    J.rows_rng.assign(2 * L, LevelRange());
    J.row_off.push_back(0);
    for (uint32_t lv = 0; lv < L; ++lv)
        for (int p = 0; p < 2; ++p) {
            LevelRange& rr = J.rows_rng[lv * 2 + p];
            rr.first = (uint32_t)J.row_player.size();
            for (uint32_t i : dec[p][lv]) {
                const NodeRec& n = t.nodes[i];
                uint32_t so = t.soff[i];
                for (uint32_t c = 0; c < nc(i, p); ++c) {
                    for (uint32_t cell = t.legal_off[n.row_off + c]; cell < t.legal_off[n.row_off + c + 1]; ++cell) {
                        sorted_of[so + cell] = (uint32_t)J.cell_ref.size();
                        J.cell_ref.push_back(so + cell);
                    }
                    J.row_off.push_back((uint32_t)J.cell_ref.size());
                    J.row_player.push_back((uint8_t)p);
                }
            }
            rr.count = (uint32_t)J.row_player.size() - rr.first;
        }
    J.ndec_rows = (uint32_t)J.row_player.size();
    if (J.cell_ref.size() != J.ncells) throw std::logic_error("cell sort lost cells");

    // ---- value arenas per traverser
    std::vector<uint32_t> vblk[2];
    J.vg_rng.assign(2 * L, LevelRange());
    for (int p = 0; p < 2; ++p) {
        vblk[p].assign(N, 0);
        uint32_t cur = 0;
        for (uint32_t lv = 0; lv < L; ++lv) {
            J.rows_rng[lv * 2 + p].out_first = cur;
            for (uint32_t i : dec[p][lv]) { vblk[p][i] = cur; cur += nc(i, p); }
            J.vg_rng[lv * 2 + p].out_first = cur;
            for (uint32_t i : dec[1 - p][lv]) { vblk[p][i] = cur; cur += nc(i, p); }
            for (uint32_t i : chance[lv]) { vblk[p][i] = cur; cur += nc(i, p); }
            for (uint32_t i : leaves[lv]) { vblk[p][i] = cur; cur += nc(i, p); }
        }
        J.val_len[p] = cur;
    }
    J.root_vblk[0] = vblk[0][0];
    J.root_vblk[1] = vblk[1][0];

    // ---- reach blocks: root, then per (level, mover); idle player aliased
    std::vector<uint32_t> rblk[2];
    rblk[0].assign(N, 0);
    rblk[1].assign(N, 0);
    J.rg_rng.assign(2 * L, LevelRange());
    uint32_t rcur = 0;
    rblk[0][0] = rcur; rcur += nc(0, 0);
    rblk[1][0] = rcur; rcur += nc(0, 1);
    J.root_rblk[0] = rblk[0][0];
    J.root_rblk[1] = rblk[1][0];
    for (uint32_t lv = 1; lv < L; ++lv)
        for (int q = 0; q < 2; ++q) {
            J.rg_rng[lv * 2 + q].out_first = rcur;
            for (uint32_t c : all[lv]) {
                uint32_t pa = parent[c];
                if (t.nodes[pa].player != q) continue;
                rblk[q][c] = rcur;
                rcur += nc(c, q);
                rblk[1 - q][c] = rblk[1 - q][pa];
            }
        }
    J.reach_len = rcur;

    const uint32_t ONE = J.ncells + J.ndraw;

    // ---- reach gathers, per (level, mover), in the oracle's order: a child's
    // entries are collected in the reference's visiting order, then grouped
    // by output config with a stable counting sort (each output keeps its
    // entries in visiting order)
    // every cell and every draw entry lands in at most one list, and every
    // non-root (node, mover) config heads one
    J.rge_src.reserve(J.ncells + J.ndraw);
    J.rge_w.reserve(J.ncells + J.ndraw);
    J.rg_start.reserve(J.reach_len + 1);
    J.rg_start.push_back(0);
    struct Ent {
        uint32_t out, src, w;
    };
    std::vector<Ent> ents, sorted;
    std::vector<uint32_t> at;
    for (uint32_t lv = 1; lv < L; ++lv)
        for (int q = 0; q < 2; ++q) {
            LevelRange& rg = J.rg_rng[lv * 2 + q];
            rg.first = (uint32_t)J.rg_start.size() - 1;
            for (uint32_t c : all[lv]) {
                uint32_t pa = parent[c];
                const NodeRec& pn = t.nodes[pa];
                if (pn.player != q) continue;
                uint32_t nout = nc(c, q);
                ents.clear();
                uint32_t src0 = rblk[q][pa];
                if (pn.kind == NK_CHANCE) {
                    for (uint32_t ci = 0; ci < nc(pa, q); ++ci)
                        for (uint32_t k = t.draw_start[pn.draw_off + ci]; k < t.draw_start[pn.draw_off + ci + 1]; ++k)
                            ents.push_back({t.draw_to[k], src0 + ci, J.ncells + k});
                } else {
                    uint32_t ch = child_index[c];
                    uint32_t so = t.soff[pa];
                    for (uint32_t x = t.obs_start[pn.obs_off + ch]; x < t.obs_start[pn.obs_off + ch + 1]; ++x) {
                        uint32_t a = t.obs_act[pn.act_off + x];
                        for (uint32_t y = t.action_off[pn.aoff_off + a]; y < t.action_off[pn.aoff_off + a + 1]; ++y) {
                            uint32_t cell = t.action_cell[so + y];
                            uint32_t tr = t.legal_trans[so + cell];
                            if (tr == NO_TRANS) continue;
                            ents.push_back({tr, src0 + t.cell_row[so + cell], sorted_of[so + cell]});
                        }
                    }
                }
                at.assign(nout + 1, 0);
                for (const Ent& e : ents) {
                    if (e.out >= nout) throw std::logic_error("a reach entry outside its child's configs");
                    ++at[e.out + 1];
                }
                for (uint32_t o = 0; o < nout; ++o) at[o + 1] += at[o];
                const size_t base = J.rge_src.size();
                for (uint32_t o = 0; o < nout; ++o) J.rg_start.push_back((uint32_t)(base + at[o + 1]));
                sorted.resize(ents.size());
                for (const Ent& e : ents) sorted[at[e.out]++] = e;
                J.rge_src.resize(base + sorted.size());
                J.rge_w.resize(base + sorted.size());
                for (size_t i = 0; i < sorted.size(); ++i) {
                    J.rge_src[base + i] = sorted[i].src;
                    J.rge_w[base + i] = sorted[i].w;
                }
            }
            rg.count = (uint32_t)J.rg_start.size() - 1 - rg.first;
        }

    // ---- value gathers, per (level, traverser)
    {
        size_t entries = 0, outs = 0;  // sized once: the loops below only append
        for (int p = 0; p < 2; ++p)
            for (uint32_t i = 0; i < N; ++i) {
                const NodeRec& n = t.nodes[i];
                if (n.kind == NK_DECISION && n.player != p) {
                    entries += (size_t)nc(i, p) * n.nch;
                    outs += nc(i, p);
                } else if (n.kind == NK_CHANCE) {
                    entries += n.player == p ? t.draw_start[n.draw_off + nc(i, p)] - t.draw_start[n.draw_off] : nc(i, p);
                    outs += nc(i, p);
                }
            }
        J.vge_idx.reserve(entries);
        J.vge_w.reserve(entries);
        J.vg_start.reserve(outs + 1);
    }
    J.vg_start.push_back(0);
    for (uint32_t lv = 0; lv < L; ++lv)
        for (int p = 0; p < 2; ++p) {
            LevelRange& vg = J.vg_rng[lv * 2 + p];
            vg.first = (uint32_t)J.vg_start.size() - 1;
            for (uint32_t i : dec[1 - p][lv]) {
                const NodeRec& n = t.nodes[i];
                for (uint32_t c = 0; c < nc(i, p); ++c) {
                    for (uint32_t ch = 0; ch < n.nch; ++ch) {
                        J.vge_idx.push_back(vblk[p][t.child[n.child_off + ch]] + c);
                        J.vge_w.push_back(ONE);
                    }
                    J.vg_start.push_back((uint32_t)J.vge_idx.size());
                }
            }
            for (uint32_t i : chance[lv]) {
                const NodeRec& n = t.nodes[i];
                uint32_t chn = t.child[n.child_off];
                for (uint32_t c = 0; c < nc(i, p); ++c) {
                    if (n.player == p) {
                        for (uint32_t k = t.draw_start[n.draw_off + c]; k < t.draw_start[n.draw_off + c + 1]; ++k) {
                            J.vge_idx.push_back(vblk[p][chn] + t.draw_to[k]);
                            J.vge_w.push_back(J.ncells + k);
                        }
                    } else {
                        J.vge_idx.push_back(vblk[p][chn] + c);
                        J.vge_w.push_back(ONE);
                    }
                    J.vg_start.push_back((uint32_t)J.vge_idx.size());
                }
            }
            vg.count = (uint32_t)J.vg_start.size() - 1 - vg.first;
        }

    // ---- successor value index of every cell
    J.cell_vidx.assign(J.ncells, 0);
    for (uint32_t i = 0; i < N; ++i) {
        const NodeRec& n = t.nodes[i];
        if (n.kind != NK_DECISION) continue;
        uint32_t so = t.soff[i];
        for (uint32_t cell = 0; cell < t.soff[i + 1] - so; ++cell) {
            uint32_t tr = t.legal_trans[so + cell];
            if (tr == NO_TRANS) throw std::logic_error("legal cell without a successor config");
            J.cell_vidx[sorted_of[so + cell]] = vblk[n.player][t.legal_child[so + cell]] + tr;
        }
    }

    J.drawp.assign(t.draw_p.begin(), t.draw_p.end());
    J.drawp.push_back(1.0f);

    // ---- leaves
    J.nrows_net = (uint32_t)t.leaf_rows.size();
    for (uint32_t i : t.leaf_rows) {
        for (int q = 0; q < 2; ++q) {
            J.lr_ridx.push_back(rblk[q][i]);
            J.lr_nc.push_back(nc(i, q));
            J.lr_vidx.push_back(vblk[q][i]);
        }
        J.exit_nodes.push_back(i);
    }
    J.leaf_coff = t.leaf_coff;
    J.leaf_cidx = t.leaf_cidx;
    // Network rows whose public rows are byte-identical (the same public
    // position reached along different public paths) get the same board
    // pieces P and jp: the board trunk reads nothing else of a row. Each
    // row names the first row with its bytes (FNV-1a buckets, confirmed by
    // comparing the bytes; a bucket shared by different rows keeps the later
    // ones as their own representatives), and the job keeps each distinct
    // row's bytes once (row_gpu: the row's index among them).
    J.row_rep.resize(J.nrows_net);
    J.row_gpu.resize(J.nrows_net);
    {
        std::unordered_map<uint64_t, uint32_t> first;
        first.reserve(2 * J.nrows_net);
        for (uint32_t r = 0; r < J.nrows_net; ++r) {
            const uint8_t* row = t.gpu_rows.data() + (size_t)r * GPU_ROW_BYTES;
            uint64_t h = 1469598103934665603ull;
            for (size_t k = 0; k < GPU_ROW_BYTES; ++k) h = (h ^ row[k]) * 1099511628211ull;
            auto ins = first.emplace(h, r);
            const uint32_t q = ins.first->second;
            const bool same = !ins.second && std::memcmp(t.gpu_rows.data() + (size_t)q * GPU_ROW_BYTES, row, GPU_ROW_BYTES) == 0;
            J.row_rep[r] = same ? q : r;
            if (same) {
                J.row_gpu[r] = J.row_gpu[q];
            } else {
                J.row_gpu[r] = (uint32_t)(J.gpu_rows.size() / GPU_ROW_BYTES);
                J.gpu_rows.insert(J.gpu_rows.end(), row, row + GPU_ROW_BYTES);
            }
        }
    }
    J.cphi = t.cphi;
    J.cplayer = t.cplayer;
    for (uint8_t q : J.cplayer) J.cfg_col.push_back(J.ncfg_player[q]++);
    J.nterm = (uint32_t)t.term_leaves.size();
    for (uint32_t i : t.term_leaves) {
        for (int q = 0; q < 2; ++q) {
            J.tl_ridx.push_back(rblk[q][i]);
            J.tl_nc.push_back(nc(i, q));
            J.tl_vidx.push_back(vblk[q][i]);
        }
        const NodeRec& n = t.nodes[i];
        J.tl_util0.push_back(n.player == 0 ? n.util : -n.util);
        J.exit_nodes.push_back(i);
    }
    J.card_feat.assign(2 * NTYPE * CARD_FEATS, 0.0f);
    for (int view = 0; view < 2; ++view)
        for (int ty = 0; ty < NTYPE; ++ty)
            write_card_features(t.ids[view][ty], J.card_feat.data() + (view * NTYPE + ty) * CARD_FEATS);

    J.root_belief.assign(t.root_belief[0].p.begin(), t.root_belief[0].p.end());
    J.root_belief.insert(J.root_belief.end(), t.root_belief[1].p.begin(), t.root_belief[1].p.end());
    uint32_t w = J.root_nc[0] + J.root_nc[1];
    if (ncarried == 0) {
        J.carried = J.root_belief;
        J.ncarried = 1;
    } else {
        if (carried.size() != (size_t)ncarried * w) throw std::invalid_argument("carried roots do not match the root support");
        J.carried = carried;
        J.ncarried = ncarried;
    }
    return j;
}

}  // namespace wc
