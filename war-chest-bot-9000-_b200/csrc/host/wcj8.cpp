// WCJ8: the reference's job bytes (engine/src/serialize.rs). See wcj8.h.
#include "wcj8.h"

#include <cstring>
#include <stdexcept>

#include "pbs.h"

namespace wc {

namespace {

constexpr uint32_t NO_ROW = 0xFFFFFFFFu;

template <class T>
void append(std::vector<T>& dst, const std::vector<T>& src, size_t a, size_t b) {
    dst.insert(dst.end(), src.begin() + (ptrdiff_t)a, src.begin() + (ptrdiff_t)b);
}

struct Writer {
    std::vector<uint8_t> b;
    void u32(uint32_t v) {
        for (int k = 0; k < 4; ++k) b.push_back((uint8_t)(v >> (8 * k)));
    }
    void f32(float v) {
        uint32_t u;
        std::memcpy(&u, &v, 4);
        u32(u);
    }
    void u8s(const std::vector<uint8_t>& v) {
        u32((uint32_t)v.size());
        b.insert(b.end(), v.begin(), v.end());
    }
    void u32s(const std::vector<uint32_t>& v) {
        u32((uint32_t)v.size());
        for (uint32_t x : v) u32(x);
    }
    void f32s(const std::vector<float>& v) {
        u32((uint32_t)v.size());
        for (float x : v) f32(x);
    }
};

struct Reader {
    const uint8_t* b;
    size_t n, at = 0;
    std::string err;
    bool take(size_t k, const char* what) {
        if (!err.empty()) return false;
        if (k > n - at) {
            err = std::string("job truncated reading ") + what;
            return false;
        }
        return true;
    }
    uint32_t u32(const char* what) {
        if (!take(4, what)) return 0;
        uint32_t v = 0;
        for (int k = 0; k < 4; ++k) v |= (uint32_t)b[at + k] << (8 * k);
        at += 4;
        return v;
    }
    float f32(const char* what) {
        const uint32_t u = u32(what);
        float v;
        std::memcpy(&v, &u, 4);
        return v;
    }
    std::vector<uint8_t> u8s(const char* what) {
        const uint32_t k = u32(what);
        if (!take(k, what)) return {};
        std::vector<uint8_t> v(b + at, b + at + k);
        at += k;
        return v;
    }
    std::vector<uint32_t> u32s(const char* what) {
        const uint32_t k = u32(what);
        if (!take(4ull * k, what)) return {};
        std::vector<uint32_t> v(k);
        for (uint32_t i = 0; i < k; ++i) v[i] = u32(what);
        return v;
    }
    std::vector<float> f32s(const char* what) {
        const uint32_t k = u32(what);
        if (!take(4ull * k, what)) return {};
        std::vector<float> v(k);
        for (uint32_t i = 0; i < k; ++i) v[i] = f32(what);
        return v;
    }
};

}  // namespace

// serialize.rs:340-357 and 689-955.
Wcj8Job wcj8_from_tree(const Tree& t, const std::vector<float>& carried, uint32_t ncarried,
                       const std::vector<uint32_t>& net_dims) {
    if (t.capped) throw std::invalid_argument("a capped tree has no job");
    Wcj8Job j;
    j.depth = (uint32_t)t.cfg.depth;
    j.iters = (uint32_t)t.cfg.iters;
    j.snapshots = t.cfg.snapshots;
    j.alpha = t.cfg.cfr.alpha;
    j.beta = t.cfg.cfr.beta;
    j.gamma = t.cfg.cfr.gamma;
    j.predict = t.cfg.cfr.predict;
    for (int it : snapshot_iters(t.cfg.iters)) j.snap_iters.push_back((uint32_t)it);
    j.net_dims = net_dims;
    const uint32_t N = (uint32_t)t.nodes.size();
    j.nodes = N;
    j.ncfg = (uint32_t)t.ncfg;
    j.cphi.assign(t.cphi.begin(), t.cphi.begin() + (ptrdiff_t)(t.ncfg * CFEAT));
    j.cplayer = t.cplayer;
    auto nc = [&](uint32_t i, int p) { return (uint32_t)t.nc(i, p); };
    // config spans per node and player
    uint32_t cfg_at = 0;
    for (uint32_t i = 0; i < N; ++i) {
        j.cfg_off.push_back(cfg_at);
        cfg_at += nc(i, 0);
        j.cfg_off.push_back(cfg_at);
        cfg_at += nc(i, 1);
    }
    j.cfg_off.push_back(cfg_at);
    // node arrays, flat CSRs and the reverse (gather) transitions
    j.node_parent.assign(N, NO_ROW);
    j.rev_row_of.assign(N, NO_ROW);
    j.rvd_row_of.assign(N, NO_ROW);
    j.legal_row_of.assign(N, NO_ROW);
    j.legal_off.push_back(0);
    j.rev_start.push_back(0);
    j.rvd_start.push_back(0);
    uint32_t reach_at = 0;
    std::vector<std::vector<std::pair<uint32_t, uint32_t>>> gather;
    std::vector<std::vector<std::pair<uint32_t, float>>> gather_p;
    for (uint32_t i = 0; i < N; ++i) {
        const NodeRec& n = t.nodes[i];
        const uint32_t so = t.soff[i];
        j.node_child_start.push_back((uint32_t)j.node_child.size());
        for (uint32_t ch = 0; ch < n.nch; ++ch) {
            const uint32_t c = t.child[n.child_off + ch];
            j.node_child.push_back(c);
            j.node_parent[c] = i;
        }
        j.node_kind.push_back(n.kind);
        j.node_player.push_back(n.player);
        j.obs_off.push_back((uint32_t)j.obs_start.size());
        if (n.kind == NK_DECISION) {
            append(j.obs_start, t.obs_start, n.obs_off, n.obs_off + n.nch + 1);
            append(j.obs_act, t.obs_act, n.act_off, n.act_off + n.na);
            append(j.obs_child, t.obs_child, n.act_off, n.act_off + n.na);
        }
        j.draw_off.push_back((uint32_t)j.draw_to.size());
        j.draw_row_off.push_back((uint32_t)j.draw_row_start.size());
        if (n.kind == NK_CHANCE) {
            const int me = n.player;
            const uint32_t rows = nc(i, me), g0 = t.draw_start[n.draw_off];
            append(j.draw_to, t.draw_to, g0, t.draw_start[n.draw_off + rows]);
            append(j.draw_p, t.draw_p, g0, t.draw_start[n.draw_off + rows]);
            for (uint32_t r = 0; r <= rows; ++r) j.draw_row_start.push_back(t.draw_start[n.draw_off + r] - g0);
            // per child config: (parent config, probability), parent configs
            // ascending then draw outcomes in row order
            const uint32_t ch = t.child[n.child_off], m = nc(ch, me);
            gather_p.assign(m, {});
            for (uint32_t ci = 0; ci < rows; ++ci)
                for (uint32_t k = t.draw_start[n.draw_off + ci]; k < t.draw_start[n.draw_off + ci + 1]; ++k)
                    gather_p[t.draw_to[k]].emplace_back(ci, t.draw_p[k]);
            j.rvd_row_of[ch] = (uint32_t)j.rvd_start.size() - 1;
            for (const auto& tv : gather_p) {
                for (const auto& e : tv) {
                    j.rvd_src.push_back(e.first);
                    j.rvd_p.push_back(e.second);
                }
                j.rvd_start.push_back((uint32_t)j.rvd_src.size());
            }
        }
        j.reach_off.push_back(reach_at);
        reach_at += nc(i, 0) + nc(i, 1);
        j.soff.push_back(so);
        if (n.kind == NK_DECISION) {
            const int me = n.player;
            j.legal_row_of[i] = (uint32_t)j.legal_off.size() - 1;
            const uint32_t cell_base = (uint32_t)j.legal_action.size();
            for (uint32_t c = 1; c <= nc(i, me); ++c) j.legal_off.push_back(cell_base + t.legal_off[n.row_off + c]);
            append(j.legal_action, t.legal_action, so, t.soff[i + 1]);
            append(j.legal_child, t.legal_child, so, t.soff[i + 1]);
            append(j.legal_trans, t.legal_trans, so, t.soff[i + 1]);
            append(j.cell_row, t.cell_row, so, t.soff[i + 1]);
            // per public child, per child config: (parent config, strategy
            // cell), actions in observation order, each action's cells ascending
            for (uint32_t chi = 0; chi < n.nch; ++chi) {
                const uint32_t ch = t.child[n.child_off + chi], m = nc(ch, me);
                gather.assign(m, {});
                for (uint32_t x = t.obs_start[n.obs_off + chi]; x < t.obs_start[n.obs_off + chi + 1]; ++x) {
                    const uint32_t a = t.obs_act[n.act_off + x];
                    for (uint32_t y = t.action_off[n.aoff_off + a]; y < t.action_off[n.aoff_off + a + 1]; ++y) {
                        const uint32_t cell = t.action_cell[so + y], tr = t.legal_trans[so + cell];
                        if (tr == NO_TRANS) continue;
                        gather[tr].emplace_back(t.cell_row[so + cell], so + cell);
                    }
                }
                j.rev_row_of[ch] = (uint32_t)j.rev_start.size() - 1;
                for (const auto& tv : gather) {
                    for (const auto& e : tv) {
                        j.rev_src.push_back(e.first);
                        j.rev_cell.push_back(e.second);
                    }
                    j.rev_start.push_back((uint32_t)j.rev_src.size());
                }
            }
        }
    }
    j.node_child_start.push_back((uint32_t)j.node_child.size());
    j.obs_off.push_back((uint32_t)j.obs_start.size());
    j.draw_off.push_back((uint32_t)j.draw_to.size());
    j.draw_row_off.push_back((uint32_t)j.draw_row_start.size());
    j.reach_off.push_back(reach_at);
    j.soff.push_back(t.soff[N]);
    j.ncells = (uint32_t)t.ncells();
    // leaves
    j.leaf_rows = t.leaf_rows;
    j.term_leaves = t.term_leaves;
    for (uint32_t i : t.term_leaves) j.terminal_utility.push_back(t.nodes[i].util);
    j.rows = (uint32_t)t.leaf_rows.size();
    j.leaf_coff = t.leaf_coff;
    if (j.leaf_coff.size() == 2ull * j.rows) j.leaf_coff.push_back((uint32_t)t.leaf_cidx.size());
    j.leaf_cidx = t.leaf_cidx;
    uint32_t snap_at = 0;
    for (int pass = 0; pass < 2; ++pass)
        for (uint32_t i : pass == 0 ? t.leaf_rows : t.term_leaves)
            for (int p = 0; p < 2; ++p) {
                j.snap_coff.push_back(snap_at);
                snap_at += nc(i, p);
            }
    j.snap_coff.push_back(snap_at);
    j.leaf_raw.assign(t.gpu_rows.begin(), t.gpu_rows.begin() + (ptrdiff_t)((size_t)j.rows * GPU_ROW_BYTES));
    j.card_feat.assign((size_t)NTYPE * CARD_FEATS, 0.0f);
    for (int ty = 0; ty < NTYPE; ++ty) write_card_features(t.ids[0][ty], j.card_feat.data() + ty * CARD_FEATS);
    // BFS levels: the root, its children, theirs, ...
    j.level_start.push_back(0);
    std::vector<uint32_t> frontier{0}, next;
    while (!frontier.empty()) {
        next.clear();
        for (uint32_t i : frontier) {
            j.bfs_order.push_back(i);
            for (uint32_t k = j.node_child_start[i]; k < j.node_child_start[i + 1]; ++k) next.push_back(j.node_child[k]);
        }
        frontier.swap(next);
        j.level_start.push_back((uint32_t)j.bfs_order.size());
    }
    // beliefs
    j.root[0] = t.root_belief[0].p;
    j.root[1] = t.root_belief[1].p;
    const size_t w0 = t.nc(0, 0), w1 = t.nc(0, 1);
    if (carried.size() != (size_t)ncarried * (w0 + w1)) throw std::invalid_argument("carried roots do not fit the root");
    for (uint32_t r = 0; r < ncarried; ++r) {
        const float* c = carried.data() + r * (w0 + w1);
        j.carried[0].emplace_back(c, c + w0);
        j.carried[1].emplace_back(c + w0, c + w0 + w1);
    }
    return j;
}

// serialize.rs:1051-1125.
std::vector<uint8_t> wcj8_write(const Wcj8Job& j) {
    Writer w;
    w.u32(WCJ8_MAGIC);
    w.u32(WCJ8_VERSION);
    w.u32(j.depth);
    w.u32(j.iters);
    w.b.push_back(j.snapshots ? 1 : 0);
    w.f32(j.alpha);
    w.f32(j.beta);
    w.f32(j.gamma);
    w.f32(j.predict);
    w.u32s(j.snap_iters);
    w.u32s(j.net_dims);
    w.u32(j.nodes);
    w.u32(j.ncfg);
    w.u32(j.rows);
    w.u32(j.ncells);
    w.u8s(j.node_kind);
    w.u8s(j.node_player);
    for (const auto* v : {&j.node_child_start, &j.node_child, &j.obs_off, &j.obs_start, &j.obs_act, &j.obs_child,
                          &j.legal_row_of, &j.legal_off, &j.legal_action, &j.legal_child, &j.legal_trans, &j.cell_row,
                          &j.draw_off, &j.draw_to})
        w.u32s(*v);
    w.f32s(j.draw_p);
    for (const auto* v : {&j.draw_row_off, &j.draw_row_start, &j.cfg_off, &j.reach_off, &j.soff, &j.node_parent,
                          &j.rev_row_of, &j.rev_start, &j.rev_src, &j.rev_cell, &j.rvd_row_of, &j.rvd_start, &j.rvd_src})
        w.u32s(*v);
    w.f32s(j.rvd_p);
    w.u32s(j.leaf_rows);
    w.u32s(j.term_leaves);
    w.f32s(j.terminal_utility);
    w.u32s(j.leaf_coff);
    w.u32s(j.leaf_cidx);
    w.u32s(j.snap_coff);
    w.u8s(j.leaf_raw);
    w.f32s(j.card_feat);
    w.f32s(j.cphi);
    w.u8s(j.cplayer);
    w.u32s(j.bfs_order);
    w.u32s(j.level_start);
    w.f32s(j.root[0]);
    w.f32s(j.root[1]);
    w.u32((uint32_t)j.carried[0].size());
    for (size_t r = 0; r < j.carried[0].size(); ++r) {
        w.f32s(j.carried[0][r]);
        w.f32s(j.carried[1][r]);
    }
    return w.b;
}

// serialize.rs:1127-1240, with its count checks.
bool wcj8_read(const uint8_t* data, size_t n, Wcj8Job* out, std::string* err) {
    Reader r{data, n, 0, {}};
    Wcj8Job j;
    auto fail = [&](const std::string& m) {
        if (err) *err = m;
        return false;
    };
    if (!data) return fail("job: no bytes");
    if (r.u32("magic") != WCJ8_MAGIC) return fail(r.err.empty() ? "job: bad magic" : r.err);
    if (r.u32("version") != WCJ8_VERSION) return fail(r.err.empty() ? "job: unsupported version" : r.err);
    j.depth = r.u32("depth");
    j.iters = r.u32("iters");
    if (r.take(1, "snapshots")) j.snapshots = data[r.at++] != 0;
    j.alpha = r.f32("alpha");
    j.beta = r.f32("beta");
    j.gamma = r.f32("gamma");
    j.predict = r.f32("predict");
    j.snap_iters = r.u32s("snap_iters");
    j.net_dims = r.u32s("net_dims");
    j.nodes = r.u32("nodes");
    j.ncfg = r.u32("ncfg");
    j.rows = r.u32("rows");
    j.ncells = r.u32("ncells");
    j.node_kind = r.u8s("node_kind");
    j.node_player = r.u8s("node_player");
    j.node_child_start = r.u32s("node_child_start");
    j.node_child = r.u32s("node_child");
    j.obs_off = r.u32s("obs_off");
    j.obs_start = r.u32s("obs_start");
    j.obs_act = r.u32s("obs_act");
    j.obs_child = r.u32s("obs_child");
    j.legal_row_of = r.u32s("legal_row_of");
    j.legal_off = r.u32s("legal_off");
    j.legal_action = r.u32s("legal_action");
    j.legal_child = r.u32s("legal_child");
    j.legal_trans = r.u32s("legal_trans");
    j.cell_row = r.u32s("cell_row");
    j.draw_off = r.u32s("draw_off");
    j.draw_to = r.u32s("draw_to");
    j.draw_p = r.f32s("draw_p");
    j.draw_row_off = r.u32s("draw_row_off");
    j.draw_row_start = r.u32s("draw_row_start");
    j.cfg_off = r.u32s("cfg_off");
    j.reach_off = r.u32s("reach_off");
    j.soff = r.u32s("soff");
    j.node_parent = r.u32s("node_parent");
    j.rev_row_of = r.u32s("rev_row_of");
    j.rev_start = r.u32s("rev_start");
    j.rev_src = r.u32s("rev_src");
    j.rev_cell = r.u32s("rev_cell");
    j.rvd_row_of = r.u32s("rvd_row_of");
    j.rvd_start = r.u32s("rvd_start");
    j.rvd_src = r.u32s("rvd_src");
    j.rvd_p = r.f32s("rvd_p");
    j.leaf_rows = r.u32s("leaf_rows");
    j.term_leaves = r.u32s("term_leaves");
    j.terminal_utility = r.f32s("terminal_utility");
    j.leaf_coff = r.u32s("leaf_coff");
    j.leaf_cidx = r.u32s("leaf_cidx");
    j.snap_coff = r.u32s("snap_coff");
    j.leaf_raw = r.u8s("leaf_raw");
    j.card_feat = r.f32s("card_feat");
    j.cphi = r.f32s("cphi");
    j.cplayer = r.u8s("cplayer");
    j.bfs_order = r.u32s("bfs_order");
    j.level_start = r.u32s("level_start");
    if (!r.err.empty()) return fail(r.err);
    const size_t N = j.nodes;
    struct Want { size_t got, want; const char* what; };
    const Want checks[] = {
        {j.node_kind.size(), N, "node_kind"}, {j.node_player.size(), N, "node_player"},
        {j.legal_row_of.size(), N, "legal_row_of"}, {j.node_child_start.size(), N + 1, "node_child_start"},
        {j.obs_off.size(), N + 1, "obs_off"}, {j.draw_off.size(), N + 1, "draw_off"},
        {j.draw_row_off.size(), N + 1, "draw_row_off"}, {j.reach_off.size(), N + 1, "reach_off"},
        {j.soff.size(), N + 1, "soff"}, {j.cfg_off.size(), 2 * N + 1, "cfg_off"},
        {j.cphi.size(), (size_t)j.ncfg * CFEAT, "cphi"}, {j.cplayer.size(), j.ncfg, "cplayer"},
        {j.leaf_raw.size(), (size_t)j.rows * GPU_ROW_BYTES, "leaf_raw"},
        {j.card_feat.size(), (size_t)NTYPE * CARD_FEATS, "card_feat"},
        {j.leaf_coff.size(), 2ull * j.rows + 1, "leaf_coff"}, {j.node_parent.size(), N, "node_parent"},
        {j.rev_row_of.size(), N, "rev_row_of"}, {j.rvd_row_of.size(), N, "rvd_row_of"},
        {j.rev_cell.size(), j.rev_src.size(), "rev_cell"}, {j.rvd_p.size(), j.rvd_src.size(), "rvd_p"},
        {j.legal_action.size(), j.ncells, "legal_action"}, {j.legal_child.size(), j.ncells, "legal_child"},
        {j.legal_trans.size(), j.ncells, "legal_trans"}, {j.cell_row.size(), j.ncells, "cell_row"},
        {j.legal_off.empty() ? 0 : j.legal_off.back(), j.ncells, "legal_off"},
        {j.snap_coff.size(), 2 * (j.leaf_rows.size() + j.term_leaves.size()) + 1, "snap_coff"},
        {j.rows, j.leaf_rows.size(), "rows"},
    };
    for (const Want& c : checks)
        if (c.got != c.want)
            return fail(std::string("job ") + c.what + ": count " + std::to_string(c.got) + " != expected " +
                        std::to_string(c.want));
    if (j.level_start.empty()) return fail("job level_start: empty");
    j.root[0] = r.f32s("root0");
    j.root[1] = r.f32s("root1");
    const uint32_t nroots = r.u32("nroots");
    for (uint32_t k = 0; k < nroots && r.err.empty(); ++k) {
        j.carried[0].push_back(r.f32s("carried0"));
        j.carried[1].push_back(r.f32s("carried1"));
    }
    if (!r.err.empty()) return fail(r.err);
    if (r.at != n) return fail("job: trailing bytes");
    *out = std::move(j);
    return true;
}

std::unique_ptr<Tree> wcj8_tree(const Wcj8Job& j, std::vector<float>* carried, uint32_t* ncarried, std::string* err) {
    auto fail = [&](const std::string& m) -> std::unique_ptr<Tree> {
        if (err) *err = m;
        return nullptr;
    };
    const uint32_t N = j.nodes;
    if (N == 0) return fail("job: no nodes");
    auto t = std::make_unique<Tree>();
    t->cfg.depth = (int)j.depth;
    t->cfg.iters = (int)j.iters;
    t->cfg.snapshots = j.snapshots;
    t->cfg.cfr = {j.alpha, j.beta, j.gamma, j.predict};
    std::vector<uint32_t> want_snaps;
    for (int it : snapshot_iters((int)j.iters)) want_snaps.push_back((uint32_t)it);
    if (want_snaps != j.snap_iters) return fail("job: a snapshot list other than snapshot_iters(iters)");
    // levels from the BFS tiling
    std::vector<uint32_t> depth(N, 0);
    for (size_t lv = 0; lv + 1 < j.level_start.size(); ++lv)
        for (uint32_t k = j.level_start[lv]; k < j.level_start[lv + 1]; ++k) {
            if (k >= j.bfs_order.size() || j.bfs_order[k] >= N) return fail("job: bfs_order out of range");
            depth[j.bfs_order[k]] = (uint32_t)lv;
        }
    // supports: one per (node, player), sized by the config spans (a solve
    // reads their counts only)
    // spans bounded before anything is sized by them: 2^20 configs per (node,
    // player) and 2^28 in all, against about 2^26.6 for the largest job the
    // builder makes (200,000 nodes x 2 players x 256 configs)
    constexpr uint32_t SPAN_MAX = 1u << 20, TOTAL_MAX = 1u << 28;
    if (j.cfg_off.size() != 2 * (size_t)N + 1 || j.cfg_off[0] != 0 || j.cfg_off.back() > TOTAL_MAX)
        return fail("job: config spans out of range");
    for (size_t k = 0; k + 1 < j.cfg_off.size(); ++k) {
        if (j.cfg_off[k + 1] < j.cfg_off[k]) return fail("job: cfg_off decreases");
        if (j.cfg_off[k + 1] - j.cfg_off[k] > SPAN_MAX) return fail("job: a config span out of range");
    }
    t->supports.reserve(2 * N);
    for (size_t k = 0; k + 1 < j.cfg_off.size(); ++k) t->supports.emplace_back(j.cfg_off[k + 1] - j.cfg_off[k]);
    std::vector<uint8_t> is_term(N, 0);
    std::vector<float> util(N, 0.0f);
    for (size_t k = 0; k < j.term_leaves.size(); ++k) {
        if (j.term_leaves[k] >= N || k >= j.terminal_utility.size()) return fail("job: term_leaves out of range");
        is_term[j.term_leaves[k]] = 1;
        util[j.term_leaves[k]] = j.terminal_utility[k];
    }
    t->nodes.resize(N);
    t->soff = j.soff;
    size_t act_cursor = 0;
    for (uint32_t i = 0; i < N; ++i) {
        NodeRec& n = t->nodes[i];
        std::memset(&n, 0, sizeof n);
        n.kind = j.node_kind[i];
        n.player = j.node_player[i];
        if (n.kind > NK_LEAF || n.player > 1) return fail("job: node kind or player out of range");
        n.util = util[i];
        n.terminal = is_term[i];
        n.sup[0] = 2 * i;
        n.sup[1] = 2 * i + 1;
        n.depth = depth[i];
        n.child_off = (uint32_t)t->child.size();
        if (j.node_child_start[i + 1] < j.node_child_start[i] || j.node_child_start[i + 1] > j.node_child.size())
            return fail("job: node_child_start out of range");
        n.nch = j.node_child_start[i + 1] - j.node_child_start[i];
        append(t->child, j.node_child, j.node_child_start[i], j.node_child_start[i + 1]);
        n.act_off = (uint32_t)t->obs_act.size();
        n.obs_off = (uint32_t)t->obs_start.size();
        n.row_off = (uint32_t)t->legal_off.size();
        n.aoff_off = (uint32_t)t->action_off.size();
        n.draw_off = (uint32_t)t->draw_start.size();
        const uint32_t so = j.soff[i], se = j.soff[i + 1];
        if (n.kind == NK_DECISION) {
            const uint32_t o0 = j.obs_off[i], o1 = j.obs_off[i + 1];
            if (o1 <= o0 || o1 > j.obs_start.size() || o1 - o0 != n.nch + 1) return fail("job: obs_off out of range");
            // the decision nodes' actions are concatenated in node order;
            // this node's count is its last observation group's end
            const uint32_t na = j.obs_start[o1 - 1];
            const size_t act_base = act_cursor;
            act_cursor += na;
            if (act_cursor > j.obs_act.size() || act_cursor > j.obs_child.size()) return fail("job: obs_act out of range");
            n.na = na;
            append(t->obs_start, j.obs_start, o0, o1);
            append(t->obs_act, j.obs_act, act_base, act_base + na);
            append(t->obs_child, j.obs_child, act_base, act_base + na);
            const int me = n.player;
            const uint32_t nc = (uint32_t)t->supports[n.sup[me]].size(), row0 = j.legal_row_of[i];
            if (row0 == NO_ROW || (uint64_t)row0 + nc >= j.legal_off.size() || se < so || se > j.ncells)
                return fail("job: legal rows out of range");
            for (uint32_t c = 0; c <= nc; ++c) t->legal_off.push_back(j.legal_off[row0 + c] - so);
            append(t->legal_action, j.legal_action, so, se);
            append(t->legal_child, j.legal_child, so, se);
            append(t->legal_trans, j.legal_trans, so, se);
            append(t->cell_row, j.cell_row, so, se);
            // each action's cells, ascending (the builder's counting sort)
            std::vector<uint32_t> aoff(na + 1, 0);
            for (uint32_t c = so; c < se; ++c) {
                if (j.legal_action[c] >= na) return fail("job: legal_action out of range");
                aoff[j.legal_action[c] + 1] += 1;
            }
            for (uint32_t a = 0; a < na; ++a) aoff[a + 1] += aoff[a];
            std::vector<uint32_t> fill(aoff.begin(), aoff.end() - 1), cells(se - so);
            for (uint32_t c = so; c < se; ++c) cells[fill[j.legal_action[c]]++] = c - so;
            t->action_off.insert(t->action_off.end(), aoff.begin(), aoff.end());
            t->action_cell.insert(t->action_cell.end(), cells.begin(), cells.end());
        } else if (se != so) {
            return fail("job: cells at a node without a decision");
        }
        if (n.kind == NK_CHANCE) {
            const uint32_t r0 = j.draw_row_off[i], r1 = j.draw_row_off[i + 1], g0 = j.draw_off[i];
            const uint32_t rows = (uint32_t)t->supports[n.sup[n.player]].size();
            if (r1 < r0 || r1 - r0 != rows + 1 || r1 > j.draw_row_start.size() || n.nch != 1 || j.draw_row_start[r0] != 0)
                return fail("job: draw rows out of range");
            const uint32_t base = (uint32_t)t->draw_to.size();
            for (uint32_t k = r0; k < r1; ++k) t->draw_start.push_back(base + j.draw_row_start[k]);
            const uint32_t e0 = g0 + j.draw_row_start[r0], e1 = g0 + j.draw_row_start[r1 - 1];
            if (e1 < e0 || e1 > j.draw_to.size() || e1 > j.draw_p.size()) return fail("job: draws out of range");
            append(t->draw_to, j.draw_to, e0, e1);
            append(t->draw_p, j.draw_p, e0, e1);
        }
    }
    // every index the flattener follows must be in range: a malformed job is
    // an error here, never an out-of-range read there
    {
        auto nc = [&](uint32_t i, int q) { return (uint32_t)t->supports[t->nodes[i].sup[q]].size(); };
        if (t->soff[0] != 0) return fail("job: soff does not start at 0");
        for (uint32_t i = 0; i < N; ++i) {
            const NodeRec& n = t->nodes[i];
            if (j.soff[i + 1] < j.soff[i]) return fail("job: soff decreases");
            for (uint32_t k = 0; k < n.nch; ++k) {
                const uint32_t c = t->child[n.child_off + k];
                if (c >= N || c <= i || j.node_parent[c] != i) return fail("job: a child out of range");
            }
            if (n.kind == NK_LEAF && n.nch != 0) return fail("job: a leaf with children");
            if (n.kind == NK_DECISION) {
                const int me = n.player;
                const uint32_t so = j.soff[i], ncell = j.soff[i + 1] - so;
                for (uint32_t c = 0; c <= nc(i, me); ++c)
                    if (t->legal_off[n.row_off + c] > ncell || (c && t->legal_off[n.row_off + c] < t->legal_off[n.row_off + c - 1]))
                        return fail("job: legal rows out of range");
                for (uint32_t x = 0; x <= n.nch; ++x)
                    if (t->obs_start[n.obs_off + x] > n.na || (x && t->obs_start[n.obs_off + x] < t->obs_start[n.obs_off + x - 1]))
                        return fail("job: observation groups out of range");
                for (uint32_t a = 0; a < n.na; ++a)
                    if (t->obs_act[n.act_off + a] >= n.na || t->obs_child[n.act_off + a] >= n.nch)
                        return fail("job: an action out of range");
                for (uint32_t c = so; c < so + ncell; ++c) {
                    const uint32_t ch = j.legal_child[c], tr = j.legal_trans[c];
                    if (ch >= N || j.node_parent[ch] != i) return fail("job: a cell's child out of range");
                    if (tr != NO_TRANS && tr >= nc(ch, me)) return fail("job: a cell's transition out of range");
                    if (j.cell_row[c] >= nc(i, me)) return fail("job: a cell's row out of range");
                }
            } else if (n.kind == NK_CHANCE) {
                const uint32_t ch = t->child[n.child_off], m = nc(ch, n.player);
                for (uint32_t r = 0; r < nc(i, n.player); ++r)
                    if (t->draw_start[n.draw_off + r + 1] < t->draw_start[n.draw_off + r])
                        return fail("job: draw rows decrease");
                for (uint32_t k = t->draw_start[n.draw_off]; k < t->draw_start[n.draw_off + nc(i, n.player)]; ++k)
                    if (t->draw_to[k] >= m) return fail("job: a draw out of range");
                if (nc(ch, 1 - n.player) != nc(i, 1 - n.player)) return fail("job: a draw changed the idle player's configs");
            }
        }
        if (j.soff[N] != j.ncells) return fail("job: soff does not end at ncells");
        for (uint32_t i : j.leaf_rows)
            if (i >= N || t->nodes[i].kind != NK_LEAF || t->nodes[i].terminal) return fail("job: a network row out of range");
        for (uint32_t i : j.term_leaves)
            if (i >= N || t->nodes[i].kind != NK_LEAF) return fail("job: a terminal leaf out of range");
        if (j.leaf_coff.empty() || j.leaf_coff[0] != 0) return fail("job: leaf_coff does not start at 0");
        for (size_t k = 0; k + 1 < j.leaf_coff.size(); ++k) {
            if (j.leaf_coff[k + 1] < j.leaf_coff[k]) return fail("job: leaf_coff decreases");
            const uint32_t r = (uint32_t)(k / 2), q = (uint32_t)(k % 2);
            if (j.leaf_coff[k + 1] - j.leaf_coff[k] != nc(j.leaf_rows[r], (int)q)) return fail("job: a row's configs do not fit its node");
        }
        for (uint32_t c : j.leaf_cidx)
            if (c >= j.ncfg || j.cplayer[c] > 1) return fail("job: a leaf config out of range");
    }
    // leaves, configs, public rows
    t->leaf_rows = j.leaf_rows;
    t->term_leaves = j.term_leaves;
    t->leaf_coff = j.leaf_coff;
    t->leaf_cidx = j.leaf_cidx;
    t->cphi = j.cphi;
    t->cplayer = j.cplayer;
    t->gpu_rows = j.leaf_raw;
    t->ncfg = j.ncfg;
    // card ids: the unit whose printed facts each coin type's are (units
    // with identical facts are interchangeable for everything a solve reads);
    // the second seat view is the first with the seats exchanged
    for (int ty = 0; ty < NTYPE; ++ty) {
        int found = -1;
        float f[CARD_FEATS];
        for (int u = 0; u < N_UNITS && found < 0; ++u) {
            write_card_features((uint8_t)u, f);
            if (std::memcmp(f, j.card_feat.data() + ty * CARD_FEATS, sizeof f) == 0) found = u;
        }
        if (found < 0) return fail("job: card facts of no known unit");
        t->ids[0][ty] = (uint8_t)found;
    }
    for (int ty = 0; ty < NTYPE; ++ty) t->ids[1][ty] = t->ids[0][(ty + NSLOT) % NTYPE];
    // beliefs
    for (int p = 0; p < 2; ++p) {
        if (j.root[p].size() != t->supports[p].size()) return fail("job: root belief does not fit the root's configs");
        t->root_belief[p].cfg = t->supports[p];
        t->root_belief[p].p = j.root[p];
    }
    carried->clear();
    *ncarried = (uint32_t)j.carried[0].size();
    for (uint32_t r = 0; r < *ncarried; ++r) {
        if (j.carried[0][r].size() != j.root[0].size() || j.carried[1][r].size() != j.root[1].size())
            return fail("job: a carried root does not fit the root's configs");
        carried->insert(carried->end(), j.carried[0][r].begin(), j.carried[0][r].end());
        carried->insert(carried->end(), j.carried[1][r].begin(), j.carried[1][r].end());
    }
    return t;
}

}  // namespace wc
