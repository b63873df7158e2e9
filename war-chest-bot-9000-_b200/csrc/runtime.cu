// Device runtime: job blobs, batch upload, the solve schedule, download.
#include "runtime.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <stdexcept>

#include "cuda/kernels.h"

namespace wc {

static thread_local std::string g_err;
void set_error(const std::string& e) { g_err = e; }
const std::string& last_error() { return g_err; }

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// ------------------------------------------------------------------ blobs

JobBlob::~JobBlob() {
    if (host && pinned) cudaFreeHost(host);
    else std::free(host);
}

namespace {
size_t align16(size_t x) { return (x + 15) & ~(size_t)15; }
}  // namespace

std::unique_ptr<JobBlob> make_blob(std::unique_ptr<JobImage> img) {
    auto b = std::make_unique<JobBlob>();
    JobImage& J = *img;
    // carry offsets over exit nodes (network rows, then terminal leaves)
    std::vector<uint32_t> carry_off;
    carry_off.push_back(0);
    for (uint32_t r = 0; r < J.nrows_net; ++r) carry_off.push_back(carry_off.back() + J.lr_nc[2 * r] + J.lr_nc[2 * r + 1]);
    for (uint32_t k = 0; k < J.nterm; ++k) carry_off.push_back(carry_off.back() + J.tl_nc[2 * k] + J.tl_nc[2 * k + 1]);
    b->nexit = J.nrows_net + J.nterm;
    b->carry_width = carry_off.back();
    b->nsnaps_kept = J.cfg.snapshots ? (uint32_t)J.snap_iters.size() : 1;
    struct Src { const void* p; size_t bytes; };
    auto v = [](const auto& vec) { return Src{vec.data(), vec.size() * sizeof(vec[0])}; };
    Src src[JobBlob::N_ARR] = {
        v(J.cell_vidx), v(J.row_off), v(J.row_player), v(J.vg_start), v(J.vge_idx), v(J.vge_w), v(J.rg_start),
        v(J.rge_src), v(J.rge_w), v(J.drawp), v(J.cell_ref), v(J.lr_ridx), v(J.lr_nc), v(J.lr_vidx),
        v(J.leaf_coff), v(J.leaf_cidx), v(J.tl_ridx), v(J.tl_nc), v(J.tl_vidx), v(J.tl_util0), v(J.gpu_rows),
        v(J.cphi), v(J.cplayer), v(J.card_feat), v(J.root_belief), v(J.carried), v(carry_off)};
    size_t at = 0;
    for (int i = 0; i < JobBlob::N_ARR; ++i) {
        b->off[i] = at;
        at = align16(at + src[i].bytes);
    }
    b->bytes = at;
    // Pinned so uploads are plain DMA; pageable where no driver is present
    // (building and inspecting jobs needs no GPU).
    if (cudaHostAlloc((void**)&b->host, std::max<size_t>(at, 16), cudaHostAllocPortable) == cudaSuccess) {
        b->pinned = true;
    } else {
        cudaGetLastError();
        b->host = static_cast<uint8_t*>(std::aligned_alloc(64, (std::max<size_t>(at, 16) + 63) & ~(size_t)63));
        if (!b->host) throw std::bad_alloc();
        b->pinned = false;
    }
    for (int i = 0; i < JobBlob::N_ARR; ++i)
        if (src[i].bytes) std::memcpy(b->host + b->off[i], src[i].p, src[i].bytes);
    b->img = std::move(img);
    return b;
}

// ---------------------------------------------------------------- batches

Batch::~Batch() {
    if (dmem) cudaFree(dmem);
    for (cudaEvent_t e : events) cudaEventDestroy(e);
    for (cudaEvent_t e : marks)
        if (e) cudaEventDestroy(e);
}

void read_profile(Batch& b, double* ms) {
    for (int c = 0; c < N_TC; ++c) ms[c] = 0.0;
    check(cudaStreamSynchronize(b.dev->stream), "profile sync");
    for (size_t i = 0; i < b.events_used / 2; ++i) {
        float t = 0.0f;
        check(cudaEventElapsedTime(&t, b.events[2 * i], b.events[2 * i + 1]), "event time");
        ms[b.event_class[i]] += t;
    }
    float t = 0.0f;
    check(cudaEventElapsedTime(&t, b.marks[0], b.marks[2]), "event time");
    ms[TC_TOTAL] = t;
    check(cudaEventElapsedTime(&t, b.marks[1], b.marks[2]), "event time");
    ms[TC_PHASE2] = t;
}

namespace {

struct Alloc {
    size_t at = 0;
    size_t take(size_t bytes) {
        size_t o = at;
        at = (at + bytes + 255) & ~(size_t)255;
        return o;
    }
};

void add_items(std::vector<wcdev::WorkItem>& items, uint32_t job, uint32_t first, uint32_t count,
               uint32_t out_first) {
    for (uint32_t k = 0; k < count; k += wcdev::WI_TASKS) {
        uint32_t n = std::min<uint32_t>(wcdev::WI_TASKS, count - k);
        items.push_back({job, first + k, n, out_first + k});
    }
}

}  // namespace

std::unique_ptr<Batch> upload_batch(DeviceCtx& dev, const std::vector<const JobBlob*>& jobs) {
    auto bp = std::make_unique<Batch>();
    Batch& b = *bp;
    b.dev = &dev;
    b.jobs = jobs;
    check(cudaSetDevice(dev.device), "set device");
    const size_t nj = jobs.size();
    // ---- device memory plan: per job, table blob then state then outputs
    Alloc A;
    struct Plan {
        size_t tables, cur, regret, sum, snap, reach, reach2, vals0, vals1, cards, cardm, pb, jp, cf, cg, pooled,
            out_strategy, out_roots, out_carry;
    };
    std::vector<Plan> plan(nj);
    for (size_t j = 0; j < nj; ++j) {
        const JobBlob& jb = *jobs[j];
        const JobImage& J = *jb.img;
        Plan& P = plan[j];
        P.tables = A.take(jb.bytes);
        P.cur = A.take(4ull * J.ncells);
        P.regret = A.take(4ull * J.ncells);
        P.sum = A.take(4ull * J.ncells);
        P.snap = A.take(4ull * J.ncells);
        P.reach = A.take(4ull * J.reach_len);
        P.reach2 = J.cfg.snapshots ? A.take(4ull * J.reach_len) : 0;
        P.vals0 = A.take(4ull * J.val_len[0]);
        P.vals1 = A.take(4ull * J.val_len[1]);
        bool net = dev.have_net;
        P.cards = net ? A.take(4ull * 2 * 10 * NET_TYPE) : 0;
        P.cardm = net ? A.take(4ull * 2 * 10 * 3 * NET_POOL) : 0;
        P.pb = net ? A.take(4ull * J.nrows_net * NET_D) : 0;
        P.jp = net ? A.take(4ull * J.nrows_net * NET_JW) : 0;
        P.cf = net ? A.take(4ull * J.ncfg * NET_D) : 0;
        P.cg = net ? A.take(4ull * J.ncfg * NET_POOL) : 0;
        P.pooled = net ? A.take(4ull * J.nrows_net * 2 * NET_POOL) : 0;
        P.out_strategy = A.take(4ull * J.ncells);
        P.out_roots = A.take(4ull * J.ncarried * (J.root_nc[0] + J.root_nc[1]));
        P.out_carry = J.cfg.snapshots ? A.take(2ull * (jb.nsnaps_kept - 1) * jb.carry_width) : 0;
        b.table_bytes += jb.bytes;
    }
    // ---- work items
    uint32_t L = 0;
    for (auto* jb : jobs) L = std::max(L, jb->img->nlevels);
    b.nlevels = L;
    std::vector<wcdev::WorkItem>& items = b.items;
    auto range_of = [&](auto&& fill) {
        Batch::Range r;
        r.off = (uint32_t)items.size();
        fill();
        r.n = (uint32_t)items.size() - r.off;
        return r;
    };
    b.rows.assign(2 * L, {});
    b.vg.assign(2 * L, {});
    b.rg.assign(2 * L, {});
    for (uint32_t lv = 0; lv < L; ++lv)
        for (int p = 0; p < 2; ++p) {
            b.rows[lv * 2 + p] = range_of([&] {
                for (uint32_t j = 0; j < nj; ++j) {
                    const JobImage& J = *jobs[j]->img;
                    if (lv >= J.nlevels) continue;
                    const LevelRange& r = J.rows_rng[lv * 2 + p];
                    add_items(items, j, r.first, r.count, r.out_first);
                }
            });
            b.vg[lv * 2 + p] = range_of([&] {
                for (uint32_t j = 0; j < nj; ++j) {
                    const JobImage& J = *jobs[j]->img;
                    if (lv >= J.nlevels) continue;
                    const LevelRange& r = J.vg_rng[lv * 2 + p];
                    add_items(items, j, r.first, r.count, r.out_first);
                }
            });
            b.rg[lv * 2 + p] = range_of([&] {
                for (uint32_t j = 0; j < nj; ++j) {
                    const JobImage& J = *jobs[j]->img;
                    if (lv >= J.nlevels || lv == 0) continue;
                    const LevelRange& r = J.rg_rng[lv * 2 + p];
                    add_items(items, j, r.first, r.count, r.out_first);
                }
            });
        }
    b.rows_all = range_of([&] { for (uint32_t j = 0; j < nj; ++j) add_items(items, j, 0, jobs[j]->img->ndec_rows, 0); });
    b.cells_all = range_of([&] { for (uint32_t j = 0; j < nj; ++j) add_items(items, j, 0, jobs[j]->img->ncells, 0); });
    b.term_all = range_of([&] { for (uint32_t j = 0; j < nj; ++j) add_items(items, j, 0, jobs[j]->img->nterm, 0); });
    b.netrows_all = range_of([&] { for (uint32_t j = 0; j < nj; ++j) add_items(items, j, 0, jobs[j]->img->nrows_net, 0); });
    b.exits_all = range_of([&] { for (uint32_t j = 0; j < nj; ++j) add_items(items, j, 0, jobs[j]->nexit, 0); });
    std::vector<uint32_t> row_job, row_local, cfg_job, cfg_local;
    for (uint32_t j = 0; j < nj; ++j) {
        const JobImage& J = *jobs[j]->img;
        for (uint32_t r = 0; r < J.nrows_net; ++r) { row_job.push_back(j); row_local.push_back(r); }
        for (uint32_t c = 0; c < J.ncfg; ++c) { cfg_job.push_back(j); cfg_local.push_back(c); }
        b.max_carried = std::max(b.max_carried, J.ncarried);
        b.node_updates += (double)J.nodes * (double)J.cfg.iters;
        b.leaf_evals += (double)J.nrows_net * (double)J.cfg.iters;
    }
    b.total_rows = (uint32_t)row_job.size();
    b.total_cfgs = (uint32_t)cfg_job.size();
    size_t o_jobs = A.take(sizeof(wcdev::JobDev) * nj);
    size_t o_items = A.take(sizeof(wcdev::WorkItem) * items.size());
    size_t o_rj = A.take(4ull * row_job.size()), o_rl = A.take(4ull * row_local.size());
    size_t o_cj = A.take(4ull * cfg_job.size()), o_cl = A.take(4ull * cfg_local.size());
    b.dbytes = A.at;
    check(cudaMalloc((void**)&b.dmem, std::max<size_t>(b.dbytes, 256)), "batch device memory");
    uint8_t* D = b.dmem;
    // ---- descriptors
    b.hj.resize(nj);
    b.out_off.resize(3 * nj);
    for (size_t j = 0; j < nj; ++j) {
        const JobBlob& jb = *jobs[j];
        const JobImage& J = *jb.img;
        const Plan& P = plan[j];
        wcdev::JobDev& d = b.hj[j];
        std::memset(&d, 0, sizeof d);
        uint8_t* T = D + P.tables;
        auto t32 = [&](int a) { return reinterpret_cast<const uint32_t*>(T + jb.off[a]); };
        auto tf = [&](int a) { return reinterpret_cast<const float*>(T + jb.off[a]); };
        auto t8 = [&](int a) { return reinterpret_cast<const uint8_t*>(T + jb.off[a]); };
        d.cell_vidx = t32(JobBlob::CELL_VIDX);
        d.row_off = t32(JobBlob::ROW_OFF);
        d.row_player = t8(JobBlob::ROW_PLAYER);
        d.vg_start = t32(JobBlob::VG_START);
        d.vge_idx = t32(JobBlob::VGE_IDX);
        d.vge_w = t32(JobBlob::VGE_W);
        d.rg_start = t32(JobBlob::RG_START);
        d.rge_src = t32(JobBlob::RGE_SRC);
        d.rge_w = t32(JobBlob::RGE_W);
        d.drawp = tf(JobBlob::DRAWP);
        d.cell_ref = t32(JobBlob::CELL_REF);
        d.lr_ridx = t32(JobBlob::LR_RIDX);
        d.lr_nc = t32(JobBlob::LR_NC);
        d.lr_vidx = t32(JobBlob::LR_VIDX);
        d.leaf_coff = t32(JobBlob::LEAF_COFF);
        d.leaf_cidx = t32(JobBlob::LEAF_CIDX);
        d.tl_ridx = t32(JobBlob::TL_RIDX);
        d.tl_nc = t32(JobBlob::TL_NC);
        d.tl_vidx = t32(JobBlob::TL_VIDX);
        d.tl_util0 = tf(JobBlob::TL_UTIL0);
        d.gpu_rows = t8(JobBlob::GPU_ROWS);
        d.cphi = tf(JobBlob::CPHI);
        d.cplayer = t8(JobBlob::CPLAYER);
        d.card_feat = tf(JobBlob::CARD_FEAT);
        d.root_belief = tf(JobBlob::ROOT_BELIEF);
        d.carried = tf(JobBlob::CARRIED);
        d.carry_off = t32(JobBlob::CARRY_OFF);
        d.cur = reinterpret_cast<float*>(D + P.cur);
        d.regret = reinterpret_cast<float*>(D + P.regret);
        d.sum = reinterpret_cast<float*>(D + P.sum);
        d.snap = reinterpret_cast<float*>(D + P.snap);
        d.reach = reinterpret_cast<float*>(D + P.reach);
        d.reach2 = J.cfg.snapshots ? reinterpret_cast<float*>(D + P.reach2) : nullptr;
        d.vals[0] = reinterpret_cast<float*>(D + P.vals0);
        d.vals[1] = reinterpret_cast<float*>(D + P.vals1);
        if (dev.have_net) {
            d.cards = reinterpret_cast<float*>(D + P.cards);
            d.cardm = reinterpret_cast<float*>(D + P.cardm);
            d.pb = reinterpret_cast<float*>(D + P.pb);
            d.jp = reinterpret_cast<float*>(D + P.jp);
            d.cf = reinterpret_cast<float*>(D + P.cf);
            d.cg = reinterpret_cast<float*>(D + P.cg);
            d.pooled = reinterpret_cast<float*>(D + P.pooled);
        }
        d.out_strategy = reinterpret_cast<float*>(D + P.out_strategy);
        d.out_roots = reinterpret_cast<float*>(D + P.out_roots);
        d.out_carry = J.cfg.snapshots ? reinterpret_cast<uint16_t*>(D + P.out_carry) : nullptr;
        d.ncells = J.ncells;
        d.ndraw = J.ndraw;
        d.nrows_net = J.nrows_net;
        d.nterm = J.nterm;
        d.ncfg = J.ncfg;
        d.ncarried = J.ncarried;
        d.reach_len = J.reach_len;
        d.nexit = jb.nexit;
        d.carry_width = jb.carry_width;
        for (int q = 0; q < 2; ++q) {
            d.root_nc[q] = J.root_nc[q];
            d.root_rblk[q] = J.root_rblk[q];
            d.root_vblk[q] = J.root_vblk[q];
        }
        b.out_off[3 * j] = P.out_strategy;
        b.out_off[3 * j + 1] = P.out_roots;
        b.out_off[3 * j + 2] = P.out_carry;
    }
    b.d_jobs = reinterpret_cast<wcdev::JobDev*>(D + o_jobs);
    b.d_items = reinterpret_cast<wcdev::WorkItem*>(D + o_items);
    b.d_row_job = reinterpret_cast<uint32_t*>(D + o_rj);
    b.d_row_local = reinterpret_cast<uint32_t*>(D + o_rl);
    b.d_cfg_job = reinterpret_cast<uint32_t*>(D + o_cj);
    b.d_cfg_local = reinterpret_cast<uint32_t*>(D + o_cl);
    cudaStream_t s = dev.stream;
    for (size_t j = 0; j < nj; ++j)
        check(cudaMemcpyAsync(D + plan[j].tables, jobs[j]->host, jobs[j]->bytes, cudaMemcpyHostToDevice, s), "upload job tables");
    check(cudaMemcpyAsync(b.d_jobs, b.hj.data(), sizeof(wcdev::JobDev) * nj, cudaMemcpyHostToDevice, s), "upload descriptors");
    check(cudaMemcpyAsync(b.d_items, items.data(), sizeof(wcdev::WorkItem) * items.size(), cudaMemcpyHostToDevice, s), "upload items");
    if (!row_job.empty()) {
        check(cudaMemcpyAsync(b.d_row_job, row_job.data(), 4 * row_job.size(), cudaMemcpyHostToDevice, s), "upload rows");
        check(cudaMemcpyAsync(b.d_row_local, row_local.data(), 4 * row_local.size(), cudaMemcpyHostToDevice, s), "upload rows");
    }
    if (!cfg_job.empty()) {
        check(cudaMemcpyAsync(b.d_cfg_job, cfg_job.data(), 4 * cfg_job.size(), cudaMemcpyHostToDevice, s), "upload cfgs");
        check(cudaMemcpyAsync(b.d_cfg_local, cfg_local.data(), 4 * cfg_local.size(), cudaMemcpyHostToDevice, s), "upload cfgs");
    }
    check(cudaStreamSynchronize(s), "batch upload");
    return bp;
}

// ---------------------------------------------------------- the schedule

namespace {

float factor(float t, float p) {
    if (std::isinf(p)) return p > 0.0f ? 1.0f : 0.0f;
    float x = std::pow(t, p);
    return x / (x + 1.0f);
}

struct Sched {
    Batch& b;
    cudaStream_t s;
    const wcdev::JobDev* J;
    const wcdev::WorkItem* I;
    explicit Sched(Batch& bb) : b(bb), s(bb.dev->stream), J(bb.d_jobs), I(bb.d_items) { b.events_used = 0; b.event_class.clear(); }

    cudaEvent_t next_event() {
        if (b.events_used == b.events.size()) {
            cudaEvent_t e;
            check(cudaEventCreate(&e), "event");
            b.events.push_back(e);
        }
        return b.events[b.events_used++];
    }
    // Run `f`'s launches between two recorded events when profiling.
    template <class F>
    void timed(int cls, F&& f) {
        if (!b.profile) { f(); return; }
        check(cudaEventRecord(next_event(), s), "event");
        f();
        check(cudaEventRecord(next_event(), s), "event");
        b.event_class.push_back(cls);
    }
    const wcdev::WorkItem* it(const Batch::Range& r) const { return I + r.off; }

    // Full or single-mover reach propagation below the seeded root.
    void propagate(int strat_sel, int which_reach, int mover_mask, int sum_update, float dg) {
        for (uint32_t lv = 1; lv < b.nlevels; ++lv)
            for (int q = 0; q < 2; ++q) {
                if (!(mover_mask & (1 << q))) continue;
                const Batch::Range& r = b.rg[lv * 2 + q];
                timed(TC_REACH, [&] { wcdev::launch_rgather(J, it(r), r.n, strat_sel, which_reach, sum_update, dg, s); });
            }
    }

    void leaf_values(int p, int pool_mask) {
        timed(TC_LEAF, [&] { leaf_values_(p, pool_mask); });
    }
    void leaf_values_(int p, int pool_mask) {
        DeviceCtx& dv = *b.dev;
        if (dv.have_net) {
            if (pool_mask) wcdev::launch_pool(J, b.d_row_job, b.d_row_local, b.total_rows, pool_mask, s);
            wcdev::launch_join_readout(J, b.d_row_job, b.d_row_local, b.total_rows, p, dv.W, dv.B, dv.LN, s);
        } else {
            wcdev::launch_netrows_zero(J, it(b.netrows_all), b.netrows_all.n, p, s);
        }
        wcdev::launch_terminal(J, it(b.term_all), b.term_all.n, p, s);
    }

    void backprop(int p, int mode, int strat_sel, float da, float db, float predict) {
        for (int lv = (int)b.nlevels - 1; lv >= 0; --lv) {
            const Batch::Range& rr = b.rows[lv * 2 + p];
            const Batch::Range& vr = b.vg[lv * 2 + p];
            timed(TC_ROWS, [&] { wcdev::launch_rows(J, it(rr), rr.n, p, mode, strat_sel, da, db, predict, s); });
            timed(TC_VGATHER, [&] { wcdev::launch_vgather(J, it(vr), vr.n, p, s); });
        }
    }

    void carries(int snap_index) {
        wcdev::launch_seed_root(J, (uint32_t)b.jobs.size(), 1, -1, s);
        propagate(wcdev::STRAT_SNAP, 1, 3, 0, 1.0f);
        wcdev::launch_carry(J, it(b.exits_all), b.exits_all.n, snap_index, s);
    }
};

}  // namespace

void enqueue_solve(Batch& b) {
    if (b.jobs.empty()) return;
    DeviceCtx& dv = *b.dev;
    check(cudaSetDevice(dv.device), "set device");
    Sched S(b);
    auto mark = [&](int i) {
        if (!b.profile) return;
        if (!b.marks[i]) check(cudaEventCreate(&b.marks[i]), "event");
        check(cudaEventRecord(b.marks[i], S.s), "event");
    };
    mark(0);
    // all jobs in a batch share the solve configuration of the first
    const SolveCfg& cfg = b.jobs[0]->img->cfg;
    const std::vector<uint32_t>& snap_list = b.jobs[0]->img->snap_iters;
    const CfrRule& k = cfg.cfr;
    const uint32_t nj = (uint32_t)b.jobs.size();
    // per-solve network pieces (search.rs:1464-1499)
    if (dv.have_net) {
        S.timed(TC_NET_SOLVE, [&] {
            wcdev::launch_cards(S.J, nj, dv.W, dv.B, S.s);
            wcdev::launch_trunk(S.J, b.d_row_job, b.d_row_local, b.total_rows, dv.W, dv.B, dv.LN, S.s);
            wcdev::launch_configs(S.J, b.d_cfg_job, b.d_cfg_local, b.total_cfgs, dv.W, dv.B, dv.LN, S.s);
        });
    }
    // Solver::new: uniform strategy, reaches, reach-weighted sum seed, snapshot 0
    S.timed(TC_INIT, [&] {
        wcdev::launch_init_rows(S.J, S.it(b.rows_all), b.rows_all.n, S.s);
        wcdev::launch_seed_root(S.J, nj, 0, -1, S.s);
    });
    S.propagate(wcdev::STRAT_CUR, 0, 3, 1, 1.0f);
    int snap_index = 0;
    if (cfg.snapshots || cfg.iters == 0) {
        wcdev::launch_copy_cur_to_snap(S.J, S.it(b.rows_all), b.rows_all.n, S.s);
        if (cfg.snapshots && snap_list.size() > 1) S.carries(snap_index);
        ++snap_index;
    }
    int steps[2] = {0, 0};
    int touched[2] = {0, 0};
    int last = -1;
    for (int t = 0; t < cfg.iters; ++t) {
        int p = t % 2;
        S.leaf_values(p, last < 0 ? 3 : (1 << last));
        last = p;
        float m = (float)steps[p] + 1.0f;
        float da = factor(m, k.alpha), db = factor(m, k.beta), dg = std::pow(m / (m + 1.0f), k.gamma);
        S.backprop(p, wcdev::BACK_REGRET, wcdev::STRAT_CUR, da, db, k.predict);
        S.propagate(wcdev::STRAT_CUR, 0, 1 << p, 1, dg);
        touched[p] = 1;
        int done = t + 1;
        bool keep = cfg.snapshots ? std::find(snap_list.begin(), snap_list.end(), (uint32_t)done) != snap_list.end()
                                  : done == cfg.iters;
        if (keep) {
            S.timed(TC_SNAP, [&] {
                wcdev::launch_snapshot(S.J, S.it(b.rows_all), b.rows_all.n, touched[0], touched[1], S.s);
            });
            if (cfg.snapshots && done != cfg.iters) S.carries(snap_index);
            ++snap_index;
        }
        steps[p] += 1;
    }
    S.timed(TC_SNAP, [&] { wcdev::launch_unsort(S.J, S.it(b.cells_all), b.cells_all.n, S.s); });
    // Phase 2: one fixed-policy pass per carried root (search.rs:1851-1871)
    mark(1);
    for (uint32_t r = 0; r < b.max_carried; ++r) {
        wcdev::launch_seed_root(S.J, nj, 0, (int)r, S.s);
        S.propagate(wcdev::STRAT_SNAP, 0, 3, 0, 1.0f);
        for (int p = 0; p < 2; ++p) {
            S.leaf_values(p, p == 0 ? 3 : 0);
            S.backprop(p, wcdev::BACK_VALUE, wcdev::STRAT_SNAP, 0.0f, 0.0f, 0.0f);
            wcdev::launch_collect_root(S.J, nj, (int)r, p, S.s);
        }
    }
    mark(2);
    check(cudaGetLastError(), "solve launch");
}

void download(Batch& b, size_t job, float* strategy, float* roots, uint16_t* carries) {
    const JobBlob& jb = *b.jobs[job];
    const JobImage& J = *jb.img;
    cudaStream_t s = b.dev->stream;
    if (strategy)
        check(cudaMemcpyAsync(strategy, b.dmem + b.out_off[3 * job], 4ull * J.ncells, cudaMemcpyDeviceToHost, s), "download strategy");
    if (roots)
        check(cudaMemcpyAsync(roots, b.dmem + b.out_off[3 * job + 1], 4ull * J.ncarried * (J.root_nc[0] + J.root_nc[1]),
                              cudaMemcpyDeviceToHost, s), "download roots");
    if (carries && J.cfg.snapshots)
        check(cudaMemcpyAsync(carries, b.dmem + b.out_off[3 * job + 2], 2ull * (jb.nsnaps_kept - 1) * jb.carry_width,
                              cudaMemcpyDeviceToHost, s), "download carries");
    check(cudaStreamSynchronize(s), "download");
}

}  // namespace wc
