// The C ABI (include/wc_b200.h) over the host builder and the device runtime.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cmath>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <map>
#include <stdexcept>
#include <string>
#include <thread>

#include "../../include/wc_b200.h"
#include "cuda/kernels.h"
#include "host/job.h"
#include "host/walk.h"
#include "host/wcj8.h"
#include "runtime.h"

using namespace wc;

struct wc_job {
    std::unique_ptr<JobBlob> blob;
};

struct wc_game {
    std::unique_ptr<Game> g;
};

struct wc_batch {
    std::unique_ptr<Batch> b;
    wc_ctx* ctx = nullptr;
};

struct Ticket {
    wc_job* job = nullptr;
    bool done = false;
    int status = 0;
    std::string err;
    wc_result res{};
};

struct wc_ctx {
    std::vector<std::unique_ptr<DeviceCtx>> devs;
    // streaming service
    std::mutex mu;
    std::condition_variable cv_work, cv_done;
    std::deque<uint64_t> queue;
    std::map<uint64_t, Ticket> tickets;
    uint64_t next_ticket = 1;
    uint64_t queued_cells = 0;
    bool stop = false;
    std::vector<std::thread> workers;
};

namespace {

int fail(int code, const std::string& msg) {
    set_error(msg);
    return code;
}

template <class F>
int guarded(F&& f) {
    try {
        return f();
    } catch (const std::bad_alloc&) {
        return fail(WC_E_NOMEM, "out of host memory");
    } catch (const std::exception& e) {
        std::string m = e.what();
        if (m.find("out of memory") != std::string::npos) return fail(WC_E_NOMEM, m);
        return fail(WC_E_CUDA, m);
    }
}

int upload_weights(DeviceCtx& d, const wc_weights* w) {
    check(cudaSetDevice(d.device), "set device");
    if (!w || !w->w) {
        d.have_net = false;
        return WC_OK;
    }
    if (w->ndims != 1 || !w->dims || w->dims[0] != NET_MODEL_TAG)
        return fail(WC_E_ARG, "unsupported model format; expected dims [5]");
    if (w->nw != d.L.w_len || w->nb != d.L.b_len || w->nln != d.L.ln_len)
        return fail(WC_E_ARG, "weight sizes do not match the v5 layout");
    if (!d.W) {
        check(cudaMalloc((void**)&d.W, 4ull * d.L.w_len), "weights");
        check(cudaMalloc((void**)&d.B, 4ull * d.L.b_len), "biases");
        check(cudaMalloc((void**)&d.LN, 4ull * d.L.ln_len), "norms");
    }
    check(cudaMemcpy(d.W, w->w, 4ull * d.L.w_len, cudaMemcpyHostToDevice), "upload weights");
    check(cudaMemcpy(d.B, w->b, 4ull * d.L.b_len, cudaMemcpyHostToDevice), "upload biases");
    check(cudaMemcpy(d.LN, w->ln, 4ull * d.L.ln_len, cudaMemcpyHostToDevice), "upload norms");
    build_fast_pack(d, w->w, w->b, w->ln);
    d.have_net = true;
    return WC_OK;
}

void fill_result(Batch& b, size_t j, uint64_t version, wc_result* r, cudaStream_t stream = nullptr) {
    const JobBlob& jb = *b.jobs[j];
    const JobImage& J = *jb.img;
    std::memset(r, 0, sizeof *r);
    r->ncells = J.ncells;
    r->strategy = (float*)std::malloc(4ull * std::max<uint32_t>(J.ncells, 1));
    r->nroots = J.ncarried;
    r->root_width = J.root_nc[0] + J.root_nc[1];
    r->root_values = (float*)std::malloc(4ull * std::max<uint64_t>(r->nroots * r->root_width, 1));
    if (J.cfg.snapshots) {
        r->carry_snapshots = jb.nsnaps_kept - 1;
        r->carry_width = jb.carry_width;
        r->carries = (uint16_t*)std::malloc(2ull * std::max<uint64_t>(r->carry_snapshots * r->carry_width, 1));
    }
    r->weight_version = version;
    download(b, j, r->strategy, r->root_values, r->carries, stream);
}

bool same_schedule(const SolveCfg& a, const SolveCfg& b) {
    auto feq = [](float x, float y) { return x == y || (std::isnan(x) && std::isnan(y)); };
    return a.iters == b.iters && a.snapshots == b.snapshots && feq(a.cfr.alpha, b.cfr.alpha) &&
           feq(a.cfr.beta, b.cfr.beta) && feq(a.cfr.gamma, b.cfr.gamma) && feq(a.cfr.predict, b.cfr.predict);
}

// The reference's per-job reservation (engine/src/serialize.rs:166-203,
// WorkVector::reserved_bytes): mutable bytes plus the table bytes rounded up
// to a power of two. At 4 GiB the reference gives the job an isolated lane
// wave (requires_exclusive_route, reported as oversize_route), at 6 GiB the
// whole card (requires_card_exclusive_route); here both run in a wave of
// their own and report the same flags.
struct JobRoute {
    size_t bytes = 0;
    bool oversize = false, card_exclusive = false;
};

JobRoute route_of(const DeviceCtx& d, const JobBlob& jb) {
    JobRoute r;
    r.bytes = job_device_bytes(d, jb);
    const size_t mut = r.bytes > jb.bytes ? r.bytes - jb.bytes : 0;
    size_t tab = 1;
    while (tab < jb.bytes) tab <<= 1;
    const size_t reserved = mut + tab;
    r.oversize = reserved >= (4ull << 30);
    r.card_exclusive = reserved >= (6ull << 30);
    return r;
}

// Bytes one wave may take: WC_WAVE_BYTES, else 44% of the device memory free
// at first use (two waves are resident at once: one uploading, one solving).
size_t wave_budget(DeviceCtx& d) {
    if (!d.wave_budget) {
        if (const char* e = std::getenv("WC_WAVE_BYTES")) d.wave_budget = (size_t)std::strtoull(e, nullptr, 10);
        if (!d.wave_budget) {
            size_t fr = 0, tot = 0;
            check(cudaMemGetInfo(&fr, &tot), "device memory info");
            d.wave_budget = (size_t)((double)fr * 0.44);
        }
    }
    return d.wave_budget;
}

void ensure_arena(DeviceCtx& d, int a, size_t bytes) {
    if (d.arena_bytes[a] >= bytes) return;
    if (d.arena[a]) check(cudaFree(d.arena[a]), "free wave arena");
    d.arena[a] = nullptr;
    d.arena_bytes[a] = 0;
    check(cudaMalloc((void**)&d.arena[a], bytes), "wave arena (out of memory)");
    d.arena_bytes[a] = bytes;
}

// Solve jobs[idx] on one device in memory-bounded waves, filling out[idx].
// The jobs are split into waves of at most wave_budget bytes (at least two
// when the batch is larger than 4 GiB, so the next wave's tables upload on
// the copy stream while this wave solves); a job the reference would route
// alone gets a wave of its own. Two arenas of the device context hold the
// waves in turn and are kept across calls.
void solve_on(DeviceCtx& d, wc_job* const* jobs, const std::vector<size_t>& idx, wc_result* out) {
    if (idx.empty()) return;
    std::lock_guard<std::mutex> lk(d.mu);
    check(cudaSetDevice(d.device), "set device");
    if (!d.copy_stream) check(cudaStreamCreateWithFlags(&d.copy_stream, cudaStreamNonBlocking), "copy stream");
    const size_t budget = wave_budget(d);
    std::vector<JobRoute> rt(idx.size());
    size_t ordinary = 0;
    for (size_t i = 0; i < idx.size(); ++i) {
        rt[i] = route_of(d, *jobs[idx[i]]->blob);
        if (!rt[i].oversize) ordinary += rt[i].bytes;
    }
    std::vector<std::vector<size_t>> waves;  // positions into idx
    size_t nw = std::max<size_t>((ordinary + budget - 1) / std::max<size_t>(budget, 1),
                                 ordinary > (4ull << 30) ? 2 : 1);
    {
        const size_t target = (ordinary + nw - 1) / nw;
        std::vector<size_t> cur;
        size_t acc = 0;
        for (size_t i = 0; i < idx.size(); ++i) {
            if (rt[i].oversize) continue;
            if (!cur.empty() && acc + rt[i].bytes > target && waves.size() + 1 < nw) {
                waves.push_back(std::move(cur));
                cur.clear();
                acc = 0;
            }
            cur.push_back(i);
            acc += rt[i].bytes;
        }
        if (!cur.empty()) waves.push_back(std::move(cur));
        for (size_t i = 0; i < idx.size(); ++i)
            if (rt[i].oversize) waves.push_back({i});
    }
    const size_t W = waves.size();
    std::vector<std::unique_ptr<Batch>> B(W);
    std::vector<cudaEvent_t> up(W, nullptr), done(W, nullptr);
    auto finish = [&](size_t k) {
        check(cudaEventSynchronize(done[k]), "wave solve");
        check_batch_error(*B[k], d.copy_stream);
        for (size_t q = 0; q < waves[k].size(); ++q) {
            const size_t i = waves[k][q];
            wc_result* r = out + idx[i];
            fill_result(*B[k], q, d.version, r, d.copy_stream);
            r->oversize_route = rt[i].oversize ? 1 : 0;
            r->card_exclusive_route = rt[i].card_exclusive ? 1 : 0;
        }
        B[k].reset();
    };
    try {
        for (size_t k = 0; k < W; ++k) {
            const int a = (int)(k % 2);
            std::vector<const JobBlob*> v;
            size_t need = 0;
            for (size_t i : waves[k]) {
                v.push_back(jobs[idx[i]]->blob.get());
                need += rt[i].bytes;
            }
            ensure_arena(d, a, need);  // wave k - 2, its last user, has finished
            B[k] = upload_batch(d, v, d.arena[a], d.arena_bytes[a], d.copy_stream);
            check(cudaEventCreateWithFlags(&up[k], cudaEventDisableTiming), "event");
            check(cudaEventCreateWithFlags(&done[k], cudaEventDisableTiming), "event");
            check(cudaEventRecord(up[k], d.copy_stream), "event");
            check(cudaStreamWaitEvent(d.stream, up[k], 0), "wait upload");
            enqueue_solve(*B[k]);
            check(cudaEventRecord(done[k], d.stream), "event");
            if (k >= 1) finish(k - 1);
        }
        finish(W - 1);
    } catch (...) {
        cudaStreamSynchronize(d.stream);
        cudaStreamSynchronize(d.copy_stream);
        for (cudaEvent_t e : up)
            if (e) cudaEventDestroy(e);
        for (cudaEvent_t e : done)
            if (e) cudaEventDestroy(e);
        throw;
    }
    for (cudaEvent_t e : up) cudaEventDestroy(e);
    for (cudaEvent_t e : done) cudaEventDestroy(e);
}

// The reference router's cost of a job (engine/src/gpu/client.rs:282-291).
uint64_t job_cost(const JobBlob& jb) {
    const JobImage& J = *jb.img;
    const uint64_t iters = (uint64_t)std::max(J.cfg.iters, 1);
    return std::max<uint64_t>(1, (uint64_t)J.nrows_net * iters * 16 + (uint64_t)J.ncells * iters +
                                     (uint64_t)J.reach_len * iters + jb.bytes / 16);
}

void worker_loop(wc_ctx* ctx, DeviceCtx* d) {
    for (;;) {
        std::vector<uint64_t> ids;
        {
            std::unique_lock<std::mutex> lk(ctx->mu);
            ctx->cv_work.wait(lk, [&] { return ctx->stop || !ctx->queue.empty(); });
            if (ctx->stop) return;
            // one batch: every queued job that shares the first one's schedule
            const SolveCfg& c0 = ctx->tickets[ctx->queue.front()].job->blob->img->cfg;
            for (auto it = ctx->queue.begin(); it != ctx->queue.end();) {
                if (same_schedule(ctx->tickets[*it].job->blob->img->cfg, c0)) {
                    ids.push_back(*it);
                    it = ctx->queue.erase(it);
                } else {
                    ++it;
                }
            }
        }
        std::vector<wc_job*> jobs;
        {
            std::lock_guard<std::mutex> lk(ctx->mu);
            for (uint64_t id : ids) jobs.push_back(ctx->tickets[id].job);
        }
        std::vector<wc_result> res(jobs.size());
        std::string err;
        int status = WC_OK;
        try {
            std::vector<size_t> all(jobs.size());
            for (size_t i = 0; i < all.size(); ++i) all[i] = i;
            solve_on(*d, jobs.data(), all, res.data());
        } catch (const std::exception& e) {
            status = WC_E_CUDA;
            err = e.what();
        }
        {
            std::lock_guard<std::mutex> lk(ctx->mu);
            for (size_t i = 0; i < ids.size(); ++i) {
                Ticket& t = ctx->tickets[ids[i]];
                t.done = true;
                t.status = status;
                t.err = err;
                t.res = res[i];
                ctx->queued_cells -= std::min<uint64_t>(ctx->queued_cells, t.job->blob->img->ncells);
            }
        }
        ctx->cv_done.notify_all();
    }
}

}  // namespace

extern "C" {

int wc_last_error(char* buf, size_t n) {
    const std::string& e = last_error();
    if (buf && n) {
        size_t k = std::min(n - 1, e.size());
        std::memcpy(buf, e.data(), k);
        buf[k] = 0;
    }
    return (int)e.size();
}

void wc_net_layout(uint64_t* w_len, uint64_t* b_len, uint64_t* ln_len) {
    NetLayout L = NetLayout::make();
    if (w_len) *w_len = L.w_len;
    if (b_len) *b_len = L.b_len;
    if (ln_len) *ln_len = L.ln_len;
}

void wc_set_cap_marker_value(float v) { set_cap_marker_value(v); }

// kind 0: seeded He-normal (every Linear W ~ N(0, 2 / fan_in), the seat and
// position embeddings ~ N(0, 2 / width)); kind 1: the reference GPU tests'
// weights, uniform +-0.05 from Rng(seed) (engine/src/gpu/tests.rs:34-48).
// Biases and the value bias 0, LayerNorm gamma 1 and beta 0.
int wc_weights_fill(int kind, uint64_t seed, float* w, float* b, float* ln) {
    if (!w || !b || !ln || kind < 0 || kind > 1) return fail(WC_E_ARG, "bad weights_fill arguments");
    NetLayout L = NetLayout::make();
    for (uint32_t i = 0; i < L.b_len; ++i) b[i] = 0.0f;
    for (uint32_t i = 0; i < L.ln_len; ++i) ln[i] = 0.0f;
    for (int k = 0; k < NetLayout::N_NORMS; ++k)
        for (uint32_t i = 0; i < L.norm_w[k]; ++i) ln[L.norm_g[k] + i] = 1.0f;
    Rng rng(seed);
    if (kind == 1) {
        for (uint32_t i = 0; i < L.w_len; ++i)
            w[i] = ((float)rng.next_u64() / (float)UINT64_MAX - 0.5f) * 0.1f;
        return WC_OK;
    }
    std::vector<float> sd(L.w_len, 0.0f);
    auto span = [&](const NetSpan& s) {
        float v = std::sqrt(2.0f / (float)s.i);
        for (uint32_t q = 0; q < s.i * s.o; ++q) sd[s.w + q] = v;
    };
    auto embed = [&](uint32_t at, uint32_t n, uint32_t width) {
        float v = std::sqrt(2.0f / (float)width);
        for (uint32_t q = 0; q < n; ++q) sd[at + q] = v;
    };
    span(L.card[0]); span(L.card[1]); span(L.pile);
    embed(L.seat, 2 * NET_TYPE, NET_TYPE);
    span(L.hex_stem); span(L.tok_stem);
    embed(L.pos, 37 * NET_C, NET_C);
    span(L.glob_stem);
    for (int i = 0; i < NET_BLOCKS; ++i) { span(L.mix[i]); span(L.pool[i]); span(L.out[i]); }
    span(L.board_out); span(L.cfg1); span(L.cfg_f); span(L.cfg_g); span(L.cfg_m); span(L.join_p); span(L.join_b);
    for (int i = 0; i < NET_JBLOCKS; ++i) span(L.join_w[i]);
    span(L.join_out);
    const double two_pi = 6.283185307179586;
    for (uint32_t i = 0; i < L.w_len; ++i) {
        double u1 = 1.0 - rng.unit_f64(), u2 = rng.unit_f64();
        double z = std::sqrt(-2.0 * std::log(u1)) * std::cos(two_pi * u2);
        w[i] = sd[i] * (float)z;
    }
    return WC_OK;
}

int wc_init(int ndev, const int* devices, const wc_weights* w, int net_mode, wc_ctx** out) {
    if (ndev < 1 || !out) return fail(WC_E_ARG, "need at least one device");
    if (net_mode != WC_NET_BF16 && net_mode != WC_NET_EXACT && net_mode != WC_NET_F16)
        return fail(WC_E_ARG, "unknown network mode");
    return guarded([&] {
        auto ctx = std::make_unique<wc_ctx>();
        const Board& bd = board();
        uint8_t nb[37 * 6], isloc[37];
        for (int h = 0; h < 37; ++h) {
            for (int d = 0; d < 6; ++d) nb[h * 6 + d] = bd.neighbors[h][d];
            isloc[h] = bd.is_location[h] ? 1 : 0;
        }
        for (int i = 0; i < ndev; ++i) {
            auto d = std::make_unique<DeviceCtx>();
            d->device = devices ? devices[i] : i;
            d->precise = net_mode == WC_NET_EXACT;
            d->half = net_mode == WC_NET_F16;
            d->L = NetLayout::make();
            check(cudaSetDevice(d->device), "set device");
            check(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking), "stream");
            wcdev::net_set_constants(d->L, nb, isloc);
            wcdev::trunk_set_constants(d->L, nb, isloc);
            int rc = upload_weights(*d, w);
            if (rc) return rc;
            d->version = 1;
            ctx->devs.push_back(std::move(d));
        }
        wc_ctx* c = ctx.release();
        for (auto& d : c->devs) c->workers.emplace_back(worker_loop, c, d.get());
        *out = c;
        return (int)WC_OK;
    });
}

int wc_publish(wc_ctx* ctx, const wc_weights* w, uint64_t* version) {
    if (!ctx) return fail(WC_E_ARG, "null context");
    return guarded([&] {
        for (auto& d : ctx->devs) {
            std::lock_guard<std::mutex> lk(d->mu);
            int rc = upload_weights(*d, w);
            if (rc) return rc;
            d->version += 1;
            if (version) *version = d->version;
        }
        return (int)WC_OK;
    });
}

int wc_publish_device(wc_ctx* ctx, int dev_index, const float* w, const float* b, const float* ln,
                      uint64_t* version) {
    if (!ctx || dev_index < 0 || dev_index >= (int)ctx->devs.size() || !w || !b || !ln)
        return fail(WC_E_ARG, "bad device publish arguments");
    return guarded([&] {
        DeviceCtx& d = *ctx->devs[dev_index];
        std::lock_guard<std::mutex> lk(d.mu);
        check(cudaSetDevice(d.device), "set device");
        if (!d.W) {
            check(cudaMalloc((void**)&d.W, 4ull * d.L.w_len), "weights");
            check(cudaMalloc((void**)&d.B, 4ull * d.L.b_len), "biases");
            check(cudaMalloc((void**)&d.LN, 4ull * d.L.ln_len), "norms");
        }
        check(cudaMemcpy(d.W, w, 4ull * d.L.w_len, cudaMemcpyDeviceToDevice), "publish weights");
        check(cudaMemcpy(d.B, b, 4ull * d.L.b_len, cudaMemcpyDeviceToDevice), "publish biases");
        check(cudaMemcpy(d.LN, ln, 4ull * d.L.ln_len, cudaMemcpyDeviceToDevice), "publish norms");
        std::vector<float> hw(d.L.w_len), hb(d.L.b_len), hl(d.L.ln_len);
        check(cudaMemcpy(hw.data(), w, 4ull * d.L.w_len, cudaMemcpyDeviceToHost), "read weights");
        check(cudaMemcpy(hb.data(), b, 4ull * d.L.b_len, cudaMemcpyDeviceToHost), "read biases");
        check(cudaMemcpy(hl.data(), ln, 4ull * d.L.ln_len, cudaMemcpyDeviceToHost), "read norms");
        build_fast_pack(d, hw.data(), hb.data(), hl.data());
        d.have_net = true;
        d.version += 1;
        if (version) *version = d.version;
        return (int)WC_OK;
    });
}

void wc_shutdown(wc_ctx* ctx) {
    if (!ctx) return;
    {
        std::lock_guard<std::mutex> lk(ctx->mu);
        ctx->stop = true;
    }
    ctx->cv_work.notify_all();
    for (auto& t : ctx->workers) t.join();
    for (auto& kv : ctx->tickets)
        if (kv.second.done) wc_result_free(&kv.second.res);
    for (auto& d : ctx->devs) {
        cudaSetDevice(d->device);
        if (d->W) cudaFree(d->W);
        if (d->B) cudaFree(d->B);
        if (d->LN) cudaFree(d->LN);
        if (d->fast_mem) cudaFree(d->fast_mem);
        for (int a = 0; a < 2; ++a)
            if (d->arena[a]) cudaFree(d->arena[a]);
        if (d->copy_stream) cudaStreamDestroy(d->copy_stream);
        if (d->stream) cudaStreamDestroy(d->stream);
    }
    delete ctx;
}

int wc_root_generate(uint64_t seed, int plies, int random_draft, uint8_t* buf, size_t cap, size_t* len) {
    return guarded([&] {
        Root r;
        if (!make_root(seed, plies, random_draft != 0, &r)) return fail(WC_E_ARG, "the game ended before the root");
        std::vector<uint8_t> b = root_to_bytes(r);
        if (len) *len = b.size();
        if (!buf || b.size() > cap) return fail(WC_E_ARG, "root buffer too small");
        std::memcpy(buf, b.data(), b.size());
        return (int)WC_OK;
    });
}

namespace {

SolveCfg solve_cfg(const wc_solve_cfg* cfg) {
    SolveCfg sc;
    sc.depth = cfg->depth;
    sc.iters = cfg->iters;
    sc.snapshots = cfg->snapshots != 0;
    sc.cfr = {cfg->alpha, cfg->beta, cfg->gamma, cfg->predict};
    sc.node_cap = (size_t)cfg->node_cap;
    return sc;
}

// One job from one root (search.rs Solver::new + serialize.rs
// PackedJob::from_solver). Never throws: the status comes back, and *msg
// holds the error message of a failed build.
int build_one(const uint8_t* root, size_t len, const SolveCfg& sc, const float* carried, uint32_t ncarried,
              wc_job** out, std::string* msg) {
    *out = nullptr;
    auto err = [&](int code, const std::string& m) {
        *msg = m;
        return code;
    };
    try {
        Root r;
        if (!root || !root_from_bytes(root, len, &r)) return err(WC_E_ARG, "malformed root bytes");
        auto tree = build_tree(r.s, r.ctx, sc, r.bel);
        if (tree->capped) return err(WC_E_CAPPED, "the tree hit the node cap");
        size_t w = tree->nc(0, 0) + tree->nc(0, 1);
        std::vector<float> car;
        if (ncarried) car.assign(carried, carried + (size_t)ncarried * w);
        auto img = flatten(*tree, car, ncarried);
        auto j = std::make_unique<wc_job>();
        j->blob = make_blob(std::move(img));
        *out = j.release();
        return (int)WC_OK;
    } catch (const std::bad_alloc&) {
        return err(WC_E_NOMEM, "out of host memory");
    } catch (const std::exception& e) {
        return err(WC_E_CUDA, e.what());
    }
}

}  // namespace

// ---- rules over the reference's State encoding (write_state, roots.rs:150-180)

namespace {
bool parse_state(const uint8_t* st, size_t len, State* s) {
    size_t at = 0;
    return st && read_state(st, len, &at, s) && at == len;
}
}  // namespace

// ---- continual re-solving (selfplay.rs:466-905)

int wc_game_new(uint64_t seed, int random_draft, const wc_solve_cfg* cfg, wc_game** out) {
    if (!cfg || !out) return fail(WC_E_ARG, "null argument");
    return guarded([&] {
        auto g = std::make_unique<wc_game>();
        g->g = std::make_unique<Game>(seed, random_draft != 0, solve_cfg(cfg));
        *out = g.release();
        return (int)WC_OK;
    });
}

int wc_game_from_root(const uint8_t* root, size_t len, uint64_t seed, const wc_solve_cfg* cfg, wc_game** out) {
    if (!root || !cfg || !out) return fail(WC_E_ARG, "null argument");
    return guarded([&] {
        Root r;
        if (!root_from_bytes(root, len, &r)) return fail(WC_E_ARG, "malformed root bytes");
        auto g = std::make_unique<wc_game>();
        g->g = std::make_unique<Game>(r, seed, solve_cfg(cfg));
        *out = g.release();
        return (int)WC_OK;
    });
}

int wc_game_set_max_solves(wc_game* g, uint32_t n) {
    if (!g) return fail(WC_E_ARG, "null game");
    g->g->set_max_solves(n);
    return WC_OK;
}

int wc_game_advance(wc_game* g, wc_job** job, int* step) {
    if (!g || !job || !step) return fail(WC_E_ARG, "null argument");
    *job = nullptr;
    return guarded([&] {
        const Game::Step st = g->g->advance();
        *step = st == Game::NEED_SOLVE ? WC_GAME_SOLVE : WC_GAME_ENDED;
        if (st == Game::NEED_SOLVE) {
            std::unique_ptr<Tree> tree = g->g->take_pending_tree();
            auto j = std::make_unique<wc_job>();
            j->blob = make_blob(flatten(*tree, g->g->pending_roots(), g->g->pending_nroots()));
            *job = j.release();
        }
        return (int)WC_OK;
    });
}

int wc_game_resume(wc_game* g, const wc_job* job, const wc_result* res) {
    if (!g || !job || !res) return fail(WC_E_ARG, "null argument");
    return guarded([&] {
        const JobBlob& jb = *job->blob;
        const JobImage& J = *jb.img;
        if (res->ncells != J.ncells) return fail(WC_E_ARG, "the result is not this job's");
        WalkResult w;
        w.strategy.assign(res->strategy, res->strategy + res->ncells);
        w.carry_snapshots = (uint32_t)res->carry_snapshots;
        w.carry_width = (uint32_t)res->carry_width;
        if (res->carries) w.carries.assign(res->carries, res->carries + res->carry_snapshots * res->carry_width);
        const uint32_t* co = jb.arr<uint32_t>(JobBlob::CARRY_OFF);
        w.carry_off.assign(co, co + jb.nexit + 1);
        w.exit_nodes = J.exit_nodes;
        g->g->resume(w);
        return (int)WC_OK;
    });
}

int wc_game_counters(const wc_game* g, int64_t* out) {
    if (!g || !out) return fail(WC_E_ARG, "null argument");
    g->g->counters(out);
    return WC_OK;
}

int wc_game_root(const wc_game* g, uint8_t* buf, size_t cap, size_t* len) {
    if (!g) return fail(WC_E_ARG, "null game");
    Root r;
    r.s = g->g->state();
    r.ctx = g->g->ctx();
    r.bel[0] = g->g->belief(0);
    r.bel[1] = g->g->belief(1);
    std::vector<uint8_t> b = root_to_bytes(r);
    if (len) *len = b.size();
    if (!buf || b.size() > cap) return fail(WC_E_ARG, "root buffer too small");
    std::memcpy(buf, b.data(), b.size());
    return WC_OK;
}

void wc_game_free(wc_game* g) { delete g; }

int wc_replay_pack_row(const uint8_t* state, size_t len, uint8_t* out) {
    return guarded([&] {
        static_assert(WC_ROW_BYTES == ROW_BYTES && WC_PUBFEAT == PUBFEAT, "replay layout");
        State s;
        size_t at = 0;
        if (!out) return fail(WC_E_ARG, "no output row");
        if (!state || !read_state(state, len, &at, &s)) return fail(WC_E_ARG, "malformed state bytes");
        pack_row(s, Ctx::make(s), out);
        return (int)WC_OK;
    });
}

int wc_replay_expand(const uint8_t* rows, size_t nrows, const uint8_t* cc, const int64_t* seg, size_t m, float* x,
                     float* phi, void* stream) {
    return guarded([&] {
        if (nrows > (1u << 30)) return fail(WC_E_ARG, "too many replay rows");
        if ((nrows && (!rows || !x)) || (m && (!cc || !seg || !phi)))
            return fail(WC_E_ARG, "null device pointer");
        if (nrows && !m) return fail(WC_E_ARG, "rows without configs");
        if (!wcdev::replay_tables_ready()) return fail(WC_E_CUDA, "replay tables: " + std::string(cudaGetErrorString(cudaGetLastError())));
        wcdev::launch_replay_expand(rows, (uint32_t)nrows, cc, seg, m, x, phi, static_cast<cudaStream_t>(stream));
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return fail(WC_E_CUDA, std::string("replay expand: ") + cudaGetErrorString(e));
        return (int)WC_OK;
    });
}

int wc_state_legal_actions(const uint8_t* state, size_t len, uint32_t* codes, size_t cap, size_t* n) {
    return guarded([&] {
        State s;
        if (!parse_state(state, len, &s)) return fail(WC_E_ARG, "malformed state bytes");
        std::vector<Action> acts = s.legal_actions();
        if (n) *n = acts.size();
        if (acts.size() > cap || (!codes && !acts.empty())) return fail(WC_E_ARG, "action buffer too small");
        for (size_t i = 0; i < acts.size(); ++i) codes[i] = acts[i].encode();
        return (int)WC_OK;
    });
}

int wc_state_apply(const uint8_t* state, size_t len, uint32_t code, int unchecked, uint8_t* out, size_t cap,
                   size_t* out_len) {
    return guarded([&] {
        State s;
        if (!parse_state(state, len, &s)) return fail(WC_E_ARG, "malformed state bytes");
        Action a;
        if (!Action::decode(code, &a)) return fail(WC_E_ARG, "undecodable action code");
        if (!unchecked) {
            bool legal = false;
            for (const Action& x : s.legal_actions()) legal = legal || x == a;
            if (!legal) return fail(WC_E_ARG, "action " + a.to_string() + " is not legal in this state");
        } else if (!action_well_formed(s, a)) {
            return fail(WC_E_ARG, "action " + a.to_string() + " names an empty hex, a missing unit or a field "
                                  "out of range");
        }
        s.apply_inplace(a);
        std::vector<uint8_t> b;
        write_state(b, s);
        if (out_len) *out_len = b.size();
        if (!out || b.size() > cap) return fail(WC_E_ARG, "state buffer too small");
        std::memcpy(out, b.data(), b.size());
        return (int)WC_OK;
    });
}

int wc_state_query(const uint8_t* state, size_t len, int32_t* out) {
    return guarded([&] {
        State s;
        if (!out || !parse_state(state, len, &s)) return fail(WC_E_ARG, "malformed state bytes");
        out[0] = s.to_act();
        out[1] = s.winner == NONE ? -1 : (int32_t)s.winner;
        out[2] = s.is_terminal() ? 1 : 0;
        out[3] = s.is_chance() ? 1 : 0;
        return (int)WC_OK;
    });
}

int wc_roots_file_split(const uint8_t* file, size_t len, uint64_t* offsets, uint64_t* lengths, size_t cap,
                        size_t* n) {
    return guarded([&] {
        std::vector<std::pair<size_t, size_t>> spans;
        if (!file || !roots_file_split(file, len, &spans))
            return fail(WC_E_ARG, "not a version-3 roots file, or a malformed root in it");
        if (n) *n = spans.size();
        if (spans.size() > cap || (!spans.empty() && (!offsets || !lengths)))
            return fail(WC_E_ARG, "span buffers too small");
        for (size_t i = 0; i < spans.size(); ++i) {
            offsets[i] = spans[i].first;
            lengths[i] = spans[i].second;
        }
        return (int)WC_OK;
    });
}

int wc_root_generate_wide(uint64_t seed, int plies, int random_draft, uint32_t ncfg, uint8_t* buf, size_t cap,
                          size_t* len) {
    return guarded([&] {
        Root r;
        if (!make_wide_root(seed, plies, random_draft != 0, ncfg, &r))
            return fail(WC_E_ARG, "the game ended before the root");
        std::vector<uint8_t> b = root_to_bytes(r);
        if (len) *len = b.size();
        if (!buf || b.size() > cap) return fail(WC_E_ARG, "root buffer too small");
        std::memcpy(buf, b.data(), b.size());
        return (int)WC_OK;
    });
}

int wc_job_build(const uint8_t* root, size_t len, const wc_solve_cfg* cfg, const float* carried, uint32_t ncarried,
                 wc_job** out) {
    if (!root || !cfg || !out) return fail(WC_E_ARG, "null argument");
    const SolveCfg sc = solve_cfg(cfg);
    if (sc.depth < 1 || sc.iters < 0) return fail(WC_E_ARG, "depth must be >= 1 and iters >= 0");
    std::string msg;
    const int rc = build_one(root, len, sc, carried, ncarried, out, &msg);
    return rc == WC_OK ? rc : fail(rc, msg);
}

int wc_wcj8_from_root(const uint8_t* root, size_t len, const wc_solve_cfg* cfg, const float* carried,
                      uint32_t ncarried, const uint32_t* net_dims, uint32_t ndims, uint8_t* buf, size_t cap,
                      size_t* out_len) {
    if (!root || !cfg || !out_len || (ndims && !net_dims) || (ncarried && !carried)) return fail(WC_E_ARG, "null argument");
    const SolveCfg sc = solve_cfg(cfg);
    if (sc.depth < 1 || sc.iters < 0) return fail(WC_E_ARG, "depth must be >= 1 and iters >= 0");
    return guarded([&] {
        Root r;
        if (!root_from_bytes(root, len, &r)) return fail(WC_E_ARG, "malformed root bytes");
        auto tree = build_tree(r.s, r.ctx, sc, r.bel);
        if (tree->capped) return fail(WC_E_CAPPED, "the tree hit the node cap");
        const size_t w = tree->nc(0, 0) + tree->nc(0, 1);
        std::vector<float> car(carried, carried + (size_t)ncarried * w);
        const std::vector<uint8_t> bytes =
            wcj8_write(wcj8_from_tree(*tree, car, ncarried, std::vector<uint32_t>(net_dims, net_dims + ndims)));
        *out_len = bytes.size();
        if (bytes.size() > cap || !buf) return fail(WC_E_ARG, "buffer too small for the job bytes");
        std::memcpy(buf, bytes.data(), bytes.size());
        return (int)WC_OK;
    });
}

int wc_job_from_wcj8(const uint8_t* bytes, size_t len, wc_job** out) {
    if (!bytes || !out) return fail(WC_E_ARG, "null argument");
    *out = nullptr;
    return guarded([&] {
        Wcj8Job j;
        std::string msg;
        if (!wcj8_read(bytes, len, &j, &msg)) return fail(WC_E_ARG, msg);
        std::vector<float> car;
        uint32_t ncar = 0;
        auto tree = wcj8_tree(j, &car, &ncar, &msg);
        if (!tree) return fail(WC_E_ARG, msg);
        auto job = std::make_unique<wc_job>();
        job->blob = make_blob(flatten(*tree, car, ncar));
        *out = job.release();
        return (int)WC_OK;
    });
}

int wc_job_build_batch(const uint8_t* const* roots, const size_t* lens, size_t n, const wc_solve_cfg* cfg,
                       const float* const* carried, const uint32_t* ncarried, int threads, wc_job** out,
                       int* status) {
    if (!cfg || (n && (!roots || !lens || !out || !status))) return fail(WC_E_ARG, "null argument");
    const SolveCfg sc = solve_cfg(cfg);
    if (sc.depth < 1 || sc.iters < 0) return fail(WC_E_ARG, "depth must be >= 1 and iters >= 0");
    for (size_t i = 0; i < n; ++i) {
        out[i] = nullptr;
        status[i] = WC_OK;
    }
    if (!n) return WC_OK;
    return guarded([&] {
        size_t nt = threads > 0 ? (size_t)threads : std::max<size_t>(1, std::thread::hardware_concurrency());
        nt = std::min(nt, n);
        // roots are taken one at a time from a shared counter: tree sizes are
        // heavy-tailed, so a fixed split would leave threads idle
        std::atomic<size_t> next{0};
        std::vector<std::string> msg(n);
        auto work = [&] {
            for (size_t i; (i = next.fetch_add(1)) < n;) {
                const uint32_t nc = carried && ncarried ? ncarried[i] : 0;
                if (nc && !carried[i]) {
                    status[i] = WC_E_ARG;
                    msg[i] = "carried beliefs missing";
                    continue;
                }
                status[i] = build_one(roots[i], lens[i], sc, nc ? carried[i] : nullptr, nc, &out[i], &msg[i]);
            }
        };
        std::vector<std::thread> pool;
        try {
            for (size_t k = 1; k < nt; ++k) pool.emplace_back(work);
        } catch (...) {
            // fewer threads than asked: the ones running (and this one) finish the work
        }
        work();
        for (auto& t : pool) t.join();
        for (size_t i = 0; i < n; ++i)
            if (status[i] != WC_OK && status[i] != WC_E_CAPPED)
                return fail(status[i], "root " + std::to_string(i) + ": " + msg[i]);
        return (int)WC_OK;
    });
}

int wc_job_digest(const wc_job* job, uint64_t* out) {
    if (!job || !out) return fail(WC_E_ARG, "null argument");
    const JobBlob& b = *job->blob;
    // FNV-1a over the blob's 64-bit words (its size is a multiple of 16)
    uint64_t h = 1469598103934665603ull;
    for (size_t i = 0; i + 8 <= b.bytes; i += 8) {
        uint64_t w;
        std::memcpy(&w, b.host + i, 8);
        h = (h ^ w) * 1099511628211ull;
    }
    *out = h ^ (uint64_t)b.bytes;
    return WC_OK;
}

int wc_job_info_get(const wc_job* job, wc_job_info* o) {
    if (!job || !o) return fail(WC_E_ARG, "null argument");
    const JobImage& J = *job->blob->img;
    o->nodes = J.nodes;
    o->cells = J.ncells;
    o->net_rows = J.nrows_net;
    o->terminal_leaves = J.nterm;
    o->configs = J.ncfg;
    o->levels = J.nlevels;
    o->root_nc0 = J.root_nc[0];
    o->root_nc1 = J.root_nc[1];
    o->ncarried = J.ncarried;
    o->carry_snapshots = J.cfg.snapshots ? job->blob->nsnaps_kept - 1 : 0;
    o->carry_width = job->blob->carry_width;
    o->table_bytes = job->blob->bytes;
    return WC_OK;
}

void wc_job_free(wc_job* job) { delete job; }

uint64_t wc_batch_launches(const wc_batch* b) { return b ? b->b->launches : 0; }

int wc_debug_set_wait_limit(wc_ctx* ctx, uint64_t ns) {
    if (!ctx) return fail(WC_E_ARG, "null context");
    return guarded([&] {
        for (auto& d : ctx->devs) {
            std::lock_guard<std::mutex> lk(d->mu);
            d->wait_ns = ns ? ns : DEFAULT_WAIT_NS;
            d->fast.wait_ns = d->wait_ns;
        }
        return (int)WC_OK;
    });
}

int wc_debug_umma_gemm(const uint16_t* a, const uint16_t* b, int k, int n, float* d) {
    int rc = wcdev::umma_selftest(a, b, k, n, d);
    if (rc) return fail(WC_E_CUDA, "tcgen05 self-test failed with code " + std::to_string(rc));
    return WC_OK;
}

int wc_debug_umma_gemm_static(const uint16_t* a, const uint16_t* b, int k, int n, float* d) {
    if (!a || !b || !d) return fail(WC_E_ARG, "null operand");
    switch (wcdev::umma_selftest_static(a, b, k, n, d)) {
        case 0: return WC_OK;
        case 1: return fail(WC_E_ARG, "k must be a positive multiple of 64; n a multiple of 16 in [16, 256]");
        case 4:
            return fail(WC_E_ARG, "k = " + std::to_string(k) +
                                      " exceeds 256, the largest problem the static scratch holds "
                                      "(128 x 256 and 256 x 256 bf16 operands, a 128 x 256 f32 result)");
        case 5: return fail(WC_E_CUDA, "cudaGetSymbolAddress of the static scratch failed");
        case 3: return fail(WC_E_CUDA, "tcgen05 self-test: the MMA completion wait timed out");
        default: return fail(WC_E_CUDA, "tcgen05 self-test: CUDA error");
    }
}

int wc_job_counts(const wc_job* job, uint64_t* out, int n) {
    if (!job || !out || n < 20) return fail(WC_E_ARG, "wc_job_counts needs 20 slots");
    const JobImage& J = *job->blob->img;
    const JobBlob& B = *job->blob;
    const uint32_t *row_off = B.arr<uint32_t>(JobBlob::ROW_OFF), *vg_start = B.arr<uint32_t>(JobBlob::VG_START),
                   *rg_start = B.arr<uint32_t>(JobBlob::RG_START), *rge_w = B.arr<uint32_t>(JobBlob::RGE_W),
                   *lr_nc = B.arr<uint32_t>(JobBlob::LR_NC), *tl_nc = B.arr<uint32_t>(JobBlob::TL_NC);
    for (int i = 0; i < 20; ++i) out[i] = 0;
    for (uint32_t lv = 0; lv < J.nlevels; ++lv)
        for (int p = 0; p < 2; ++p) {
            const LevelRange& rr = J.rows_rng[lv * 2 + p];
            out[0 + p] += row_off[rr.first + rr.count] - row_off[rr.first];
            out[2 + p] += rr.count;
            const LevelRange& vr = J.vg_rng[lv * 2 + p];
            out[4 + p] += vg_start[vr.first + vr.count] - vg_start[vr.first];
            out[6 + p] += vr.count;
            if (lv == 0) continue;
            const LevelRange& gr = J.rg_rng[lv * 2 + p];
            for (uint32_t e = rg_start[gr.first]; e < rg_start[gr.first + gr.count]; ++e) {
                if (rge_w[e] < J.ncells) out[8 + p] += 1;
                else out[10 + p] += 1;
            }
            out[12 + p] += gr.count;
        }
    for (uint32_t r = 0; r < J.nrows_net; ++r) { out[14] += lr_nc[2 * r]; out[15] += lr_nc[2 * r + 1]; }
    for (uint32_t k = 0; k < J.nterm; ++k) { out[16] += tl_nc[2 * k]; out[17] += tl_nc[2 * k + 1]; }
    out[18] = J.reach_len;
    out[19] = (uint64_t)J.val_len[0] + J.val_len[1];
    if (n > 20) {
        const uint32_t* rep = B.arr<uint32_t>(JobBlob::ROW_REP);
        out[20] = 0;
        for (uint32_t r = 0; r < J.nrows_net; ++r) out[20] += rep[r] == r;
    }
    return WC_OK;
}

int wc_job_root_belief(const wc_job* job, float* out) {
    if (!job || !out) return fail(WC_E_ARG, "null argument");
    const JobImage& J = *job->blob->img;
    std::memcpy(out, job->blob->arr<float>(JobBlob::ROOT_BELIEF), 4ull * (J.root_nc[0] + J.root_nc[1]));
    return WC_OK;
}

int wc_job_carry_offsets(const wc_job* job, uint32_t* out, uint32_t* exit_nodes) {
    if (!job) return fail(WC_E_ARG, "null argument");
    const JobBlob& jb = *job->blob;
    if (out) std::memcpy(out, jb.host + jb.off[JobBlob::CARRY_OFF], 4ull * (jb.nexit + 1));
    if (exit_nodes) std::memcpy(exit_nodes, jb.img->exit_nodes.data(), 4ull * jb.nexit);
    return WC_OK;
}

int wc_solve_batch(wc_ctx* ctx, wc_job* const* jobs, size_t n, wc_result* out) {
    if (!ctx || (!jobs && n) || (!out && n)) return fail(WC_E_ARG, "null argument");
    for (size_t i = 0; i < n; ++i)
        if (!jobs[i] || !same_schedule(jobs[i]->blob->img->cfg, jobs[0]->blob->img->cfg))
            return fail(WC_E_ARG, "every job of a batch needs the same iterations, snapshots and CFR rule");
    return guarded([&] {
        size_t nd = ctx->devs.size();
        // longest processing time first by the reference's job cost: each job
        // to the device with the least work so far (heavy-tailed trees)
        std::vector<size_t> order(n);
        for (size_t i = 0; i < n; ++i) order[i] = i;
        std::vector<uint64_t> cost(n);
        for (size_t i = 0; i < n; ++i) cost[i] = job_cost(*jobs[i]->blob);
        std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) { return cost[a] > cost[b]; });
        std::vector<std::vector<size_t>> mine(nd);
        std::vector<uint64_t> load(nd, 0);
        for (size_t i : order) {
            const size_t d = (size_t)(std::min_element(load.begin(), load.end()) - load.begin());
            mine[d].push_back(i);
            load[d] += cost[i];
        }
        for (auto& m : mine) std::sort(m.begin(), m.end());
        std::vector<std::thread> th;
        std::vector<std::string> errs(nd);
        for (size_t d = 0; d < nd; ++d) {
            if (mine[d].empty()) continue;
            th.emplace_back([&, d] {
                try {
                    solve_on(*ctx->devs[d], jobs, mine[d], out);
                } catch (const std::exception& e) {
                    errs[d] = e.what();
                }
            });
        }
        for (auto& t : th) t.join();
        for (auto& e : errs)
            if (!e.empty()) throw std::runtime_error(e);
        return (int)WC_OK;
    });
}

void wc_result_free(wc_result* r) {
    if (!r) return;
    std::free(r->strategy);
    std::free(r->root_values);
    std::free(r->carries);
    std::memset(r, 0, sizeof *r);
}

int wc_batch_upload(wc_ctx* ctx, int dev_index, wc_job* const* jobs, size_t n, wc_batch** out) {
    if (!ctx || dev_index < 0 || dev_index >= (int)ctx->devs.size() || !out) return fail(WC_E_ARG, "bad arguments");
    for (size_t i = 0; i < n; ++i)
        if (!jobs[i] || !same_schedule(jobs[i]->blob->img->cfg, jobs[0]->blob->img->cfg))
            return fail(WC_E_ARG, "every job of a batch needs the same iterations, snapshots and CFR rule");
    return guarded([&] {
        std::vector<const JobBlob*> v;
        for (size_t i = 0; i < n; ++i) v.push_back(jobs[i]->blob.get());
        auto b = std::make_unique<wc_batch>();
        b->ctx = ctx;
        b->b = upload_batch(*ctx->devs[dev_index], v);
        *out = b.release();
        return (int)WC_OK;
    });
}

int wc_batch_solve(wc_batch* b) {
    if (!b) return fail(WC_E_ARG, "null batch");
    return guarded([&] {
        std::lock_guard<std::mutex> lk(b->b->dev->mu);
        enqueue_solve(*b->b);
        check(cudaStreamSynchronize(b->b->dev->stream), "batch solve");
        check_batch_error(*b->b);
        return (int)WC_OK;
    });
}

int wc_batch_solve_profiled(wc_batch* b, double* class_ms, int nclass) {
    if (!b || !class_ms || nclass < N_TC) return fail(WC_E_ARG, "bad profile arguments");
    return guarded([&] {
        std::lock_guard<std::mutex> lk(b->b->dev->mu);
        b->b->profile = true;
        enqueue_solve(*b->b);
        read_profile(*b->b, class_ms);
        b->b->profile = false;
        check_batch_error(*b->b);
        return (int)WC_OK;
    });
}

int wc_batch_nash_conv(wc_batch* b, float* nash, float* zero_sum) {
    if (!b || !nash || !zero_sum) return fail(WC_E_ARG, "bad nash-conv arguments");
    return guarded([&] {
        std::lock_guard<std::mutex> lk(b->b->dev->mu);
        enqueue_nash_conv(*b->b);
        check(cudaStreamSynchronize(b->b->dev->stream), "nash conv");
        check_batch_error(*b->b);
        for (size_t j = 0; j < b->b->jobs.size(); ++j) {
            const JobBlob& jb = *b->b->jobs[j];
            const JobImage& J = *jb.img;
            const uint32_t n0 = J.root_nc[0], n1 = J.root_nc[1], w = n0 + n1;
            std::vector<float> v(2ull * w);
            download_conv(*b->b, j, v.data());
            const float* root = jb.arr<float>(JobBlob::ROOT_BELIEF);
            // search.rs:1895-1903, in its summation order
            float nsh = 0.0f, zs = 0.0f;
            for (int p = 0; p < 2; ++p) {
                const uint32_t off = p == 0 ? 0 : n0, n = p == 0 ? n0 : n1;
                float val = 0.0f, best = 0.0f;
                for (uint32_t c = 0; c < n; ++c) val += root[off + c] * v[off + c];
                for (uint32_t c = 0; c < n; ++c) best += root[off + c] * v[w + off + c];
                nsh += best - val;
                zs += val;
            }
            nash[j] = nsh;
            zero_sum[j] = zs;
        }
        return (int)WC_OK;
    });
}

int wc_batch_leaf_values(wc_batch* b, int p, double* class_ms) {
    if (!b || p < 0 || p > 1) return fail(WC_E_ARG, "bad leaf-values arguments");
    return guarded([&] {
        std::lock_guard<std::mutex> lk(b->b->dev->mu);
        b->b->profile = class_ms != nullptr;
        enqueue_leaf_values(*b->b, p);
        if (class_ms) {
            read_profile(*b->b, class_ms);
            b->b->profile = false;
        } else {
            check(cudaStreamSynchronize(b->b->dev->stream), "leaf values");
        }
        check_batch_error(*b->b);
        return (int)WC_OK;
    });
}

int wc_batch_download_leaf_values(wc_batch* b, size_t job, int p, float* out) {
    if (!b || job >= b->b->jobs.size() || p < 0 || p > 1 || !out) return fail(WC_E_ARG, "bad arguments");
    return guarded([&] {
        download_leaf_values(*b->b, job, p, out);
        return (int)WC_OK;
    });
}

int wc_batch_download_board_rows(wc_batch* b, size_t job, float* pb, float* jp) {
    if (!b || job >= b->b->jobs.size() || !b->b->dev->have_net) return fail(WC_E_ARG, "bad arguments");
    return guarded([&] {
        download_board_rows(*b->b, job, pb, jp);
        return (int)WC_OK;
    });
}

int wc_batch_download(wc_batch* b, size_t job, float* strategy, float* root_values, uint16_t* carries) {
    if (!b || job >= b->b->jobs.size()) return fail(WC_E_ARG, "bad batch or job index");
    return guarded([&] {
        download(*b->b, job, strategy, root_values, carries);
        return (int)WC_OK;
    });
}

void wc_batch_stats(const wc_batch* b, double* node_updates, double* leaf_evals, uint64_t* table_bytes,
                    uint64_t* device_bytes) {
    if (!b) return;
    if (node_updates) *node_updates = b->b->node_updates;
    if (leaf_evals) *leaf_evals = b->b->leaf_evals;
    if (table_bytes) *table_bytes = b->b->table_bytes;
    if (device_bytes) *device_bytes = b->b->dbytes;
}

void wc_batch_free(wc_batch* b) { delete b; }

int wc_submit(wc_ctx* ctx, wc_job* job, uint64_t* ticket) {
    if (!ctx || !job || !ticket) return fail(WC_E_ARG, "null argument");
    {
        std::lock_guard<std::mutex> lk(ctx->mu);
        uint64_t id = ctx->next_ticket++;
        ctx->tickets[id].job = job;
        ctx->queue.push_back(id);
        ctx->queued_cells += job->blob->img->ncells;
        *ticket = id;
    }
    ctx->cv_work.notify_one();
    return WC_OK;
}

int wc_wait(wc_ctx* ctx, uint64_t ticket, wc_result* out) {
    if (!ctx || !out) return fail(WC_E_ARG, "null argument");
    std::unique_lock<std::mutex> lk(ctx->mu);
    auto it = ctx->tickets.find(ticket);
    if (it == ctx->tickets.end()) return fail(WC_E_STATE, "unknown ticket");
    ctx->cv_done.wait(lk, [&] { return ctx->tickets[ticket].done; });
    Ticket t = ctx->tickets[ticket];
    ctx->tickets.erase(ticket);
    if (t.status) return fail(t.status, t.err);
    *out = t.res;
    return WC_OK;
}

uint64_t wc_queued_work(wc_ctx* ctx) {
    if (!ctx) return 0;
    std::lock_guard<std::mutex> lk(ctx->mu);
    return ctx->queued_cells;
}

}  // extern "C"
