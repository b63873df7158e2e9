// Device runtime: job blobs, batch upload, the solve schedule, download.
#include "runtime.h"

#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>

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
        v(J.cphi), v(J.cplayer), v(J.card_feat), v(J.root_belief), v(J.carried), v(carry_off), v(J.cfg_col),
        v(J.row_rep), v(J.row_gpu)};
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
    for (int i = 0; i < JobBlob::N_ARR; ++i) {
        if (src[i].bytes) std::memcpy(b->host + b->off[i], src[i].p, src[i].bytes);
        // the alignment gap after the array is zeroed: the blob's bytes are a
        // function of the job alone (wc_job_digest)
        const size_t end = b->off[i] + src[i].bytes, next = i + 1 < JobBlob::N_ARR ? b->off[i + 1] : b->bytes;
        if (next > end) std::memset(b->host + end, 0, next - end);
    }
    // the blob is now the only copy of the arrays (readers use JobBlob::arr):
    // a batch of thousands of jobs keeps half the host memory
    auto drop = [](auto& v) { std::decay_t<decltype(v)>().swap(v); };
    drop(J.cell_vidx), drop(J.row_off), drop(J.row_player), drop(J.vg_start), drop(J.vge_idx), drop(J.vge_w);
    drop(J.rg_start), drop(J.rge_src), drop(J.rge_w), drop(J.drawp), drop(J.cell_ref), drop(J.lr_ridx);
    drop(J.lr_nc), drop(J.lr_vidx), drop(J.leaf_coff), drop(J.leaf_cidx), drop(J.tl_ridx), drop(J.tl_nc);
    drop(J.tl_vidx), drop(J.tl_util0), drop(J.gpu_rows), drop(J.cphi), drop(J.cplayer), drop(J.card_feat);
    drop(J.root_belief), drop(J.carried), drop(J.cfg_col), drop(J.row_rep), drop(J.row_gpu);
    b->img = std::move(img);
    return b;
}

// ---------------------------------------------------------- fast weights

namespace {
uint16_t to_bf16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
uint16_t to_op16(float f, bool half) { return half ? __half_as_ushort(__float2half_rn(f)) : to_bf16(f); }
size_t sw128_offset(uint32_t R, uint32_t r, uint32_t k) {
    uint32_t atom = k >> 6, kk = k & 63;
    uint32_t chunk = (kk >> 3) ^ (r & 7);
    return (size_t)atom * R * 128u + r * 128u + chunk * 16u + (kk & 7) * 2u;
}
// B operand tile of a [in = K][out = N] weight (rows k0 .. k0 + K): element
// (n, k) = W[(k0 + k) * N + n], K-major and swizzled.
void put_tile(uint8_t* dst, const float* W, uint32_t K, uint32_t N, bool half, uint32_t ldw = 0) {
    if (!ldw) ldw = N;
    for (uint32_t n = 0; n < N; ++n)
        for (uint32_t k = 0; k < K; ++k) {
            uint16_t v = to_op16(W[(size_t)k * ldw + n], half);
            std::memcpy(dst + sw128_offset(N, n, k), &v, 2);
        }
}
}  // namespace

void build_fast_pack(DeviceCtx& d, const float* W, const float* B, const float* LN) {
    const NetLayout& L = d.L;
    const size_t TJ = 128 * 128 * 2;
    // layout: 4 join tiles, out tile, trunk tiles, then f32 vectors
    const size_t MIX = 96 * 3 * 128, BLK = MIX + 96 * 2 * 128;
    size_t off_out = 4 * TJ, off_trunk = off_out + 2 * TJ, off_f = off_trunk + NET_BLOCKS * BLK;
    std::vector<float> vec;
    auto push = [&](const float* src, size_t n) {  // each vector 16-byte aligned (vector loads)
        while (vec.size() % 4) vec.push_back(0.0f);
        size_t at = vec.size();
        vec.insert(vec.end(), src, src + n);
        return at;
    };
    std::vector<float> beff0(NET_JW), beff1(NET_JW);
    for (int j = 0; j < NET_JW; ++j) {
        float seat_w = W[L.join_b.w + 128 * NET_JW + j];
        beff0[j] = B[L.join_b.b + j] - seat_w;
        beff1[j] = B[L.join_b.b + j] + seat_w;
    }
    size_t o_beff0 = push(beff0.data(), NET_JW), o_beff1 = push(beff1.data(), NET_JW);
    size_t o_bj[3];
    for (int i = 0; i < 3; ++i) o_bj[i] = push(B + L.join_w[i].b, NET_JW);
    size_t o_bout = push(B + L.join_out.b, NET_D);
    // the stem's token projection is linear in the pile counts:
    // (piles W_pile + cards + seat) W_tok = piles (W_pile W_tok) + (cards + seat) W_tok
    std::vector<float> pile_tok(4 * NET_C);
    for (int k = 0; k < 4; ++k)
        for (int c = 0; c < NET_C; ++c) {
            double acc = 0.0;
            for (int j = 0; j < NET_TYPE; ++j)
                acc += (double)W[L.pile.w + k * NET_TYPE + j] * (double)W[L.tok_stem.w + j * NET_C + c];
            pile_tok[k * NET_C + c] = (float)acc;
        }
    size_t o_ptok = push(pile_tok.data(), pile_tok.size());
    // per trunk block: y = mix + b_mix + (pooled W_pool + b_pool), so the two biases travel as one
    std::vector<float> tpb(NET_BLOCKS * NET_C), tob(NET_BLOCKS * NET_C);
    for (int i = 0; i < NET_BLOCKS; ++i)
        for (int c = 0; c < NET_C; ++c) {
            tpb[i * NET_C + c] = B[L.pool[i].b + c] + B[L.mix[i].b + c];
            tob[i * NET_C + c] = B[L.out[i].b + c];
        }
    size_t o_tpb = push(tpb.data(), tpb.size()), o_tob = push(tob.data(), tob.size());
    // the trunk stem: x = facts W_hex + (pos[hex] + b_hex) + ...; aligned copies for vector loads
    std::vector<float> spb(37 * NET_C);
    for (int h = 0; h < 37; ++h)
        for (int c = 0; c < NET_C; ++c) spb[h * NET_C + c] = W[L.pos + h * NET_C + c] + B[L.hex_stem.b + c];
    size_t o_sw = push(W + L.hex_stem.w, 6 * NET_C), o_spb = push(spb.data(), spb.size());
    size_t o_g[5], o_b[5];
    for (int i = 0; i < 5; ++i) {
        int norm = NetLayout::LN_JOIN + i;
        o_g[i] = push(LN + L.norm_g[norm], L.norm_w[norm]);
        o_b[i] = push(LN + L.norm_b[norm], L.norm_w[norm]);
    }
    std::vector<uint8_t> blob(off_f + 4 * vec.size(), 0);
    const bool h = d.half;
    put_tile(blob.data(), W + L.join_b.w, 128, NET_JW, h);
    for (int i = 0; i < 3; ++i) put_tile(blob.data() + (1 + i) * TJ, W + L.join_w[i].w, NET_JW, NET_JW, h);
    put_tile(blob.data() + off_out, W + L.join_out.w, NET_JW, NET_D, h);
    for (int i = 0; i < NET_BLOCKS; ++i) {  // the trunk's tiles are f16 in both modes
        put_tile(blob.data() + off_trunk + i * BLK, W + L.mix[i].w, 2 * NET_C, NET_C, true);
        put_tile(blob.data() + off_trunk + i * BLK + MIX, W + L.out[i].w, NET_C, NET_C, true);
    }
    std::memcpy(blob.data() + off_f, vec.data(), 4 * vec.size());
    check(cudaSetDevice(d.device), "set device");
    if (d.fast_mem) cudaFree(d.fast_mem);
    check(cudaMalloc((void**)&d.fast_mem, blob.size()), "fast weights");
    check(cudaMemcpy(d.fast_mem, blob.data(), blob.size(), cudaMemcpyHostToDevice), "upload fast weights");
    const float* F = reinterpret_cast<const float*>(d.fast_mem + off_f);
    d.fast.join_tiles = d.fast_mem;
    d.fast.out_tile = d.fast_mem + off_out;
    d.fast.trunk_tiles = d.fast_mem + off_trunk;
    d.fast.beff[0] = F + o_beff0;
    d.fast.beff[1] = F + o_beff1;
    for (int i = 0; i < 3; ++i) d.fast.bj[i] = F + o_bj[i];
    d.fast.bout = F + o_bout;
    for (int i = 0; i < 5; ++i) {
        d.fast.ln_g[i] = F + o_g[i];
        d.fast.ln_b[i] = F + o_b[i];
    }
    d.fast.vbias = B[L.value_bias];
    d.fast.pile_tok = F + o_ptok;
    d.fast.trunk_pb = F + o_tpb;
    d.fast.trunk_ob = F + o_tob;
    d.fast.stem_w = F + o_sw;
    d.fast.stem_pb = F + o_spb;
    d.fast.half = h ? 1 : 0;
    d.fast.wait_ns = d.wait_ns;
}

// ---------------------------------------------------------------- batches

Batch::~Batch() {
    if (dmem && owns_dmem) cudaFree(dmem);
    for (cudaEvent_t e : events) cudaEventDestroy(e);
    for (cudaEvent_t e : marks)
        if (e) cudaEventDestroy(e);
}

void read_profile(Batch& b, double* ms) {
    for (int c = 0; c < N_TC; ++c) ms[c] = 0.0;
    check(cudaStreamSynchronize(b.dev->stream), "profile sync");
    for (size_t i = 0; i + 2 < b.event_class.size(); i += 3) {
        float t = 0.0f;
        check(cudaEventElapsedTime(&t, b.events[b.event_class[i + 1]], b.events[b.event_class[i + 2]]), "event time");
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

// Regret-matching rows: at most WI_TASKS rows and ROW_CELL_CAP cells per
// item (a longer single row gets an item of its own), so the kernel can stage
// an item's cells in shared memory.
void add_row_items(std::vector<wcdev::WorkItem>& items, uint32_t job, uint32_t first, uint32_t count,
                   uint32_t out_first, const uint32_t* row_off) {
    uint32_t k = 0;
    while (k < count) {
        uint32_t n = 1;
        while (n < (uint32_t)wcdev::WI_TASKS && k + n < count &&
               row_off[first + k + n + 1] - row_off[first + k] <= (uint32_t)wcdev::ROW_CELL_CAP)
            ++n;
        items.push_back({job, first + k, n, out_first + k});
        k += n;
    }
}

void add_items(std::vector<wcdev::WorkItem>& items, uint32_t job, uint32_t first, uint32_t count,
               uint32_t out_first) {
    for (uint32_t k = 0; k < count; k += wcdev::WI_TASKS) {
        uint32_t n = std::min<uint32_t>(wcdev::WI_TASKS, count - k);
        items.push_back({job, first + k, n, out_first + k});
    }
}

}  // namespace

std::unique_ptr<Batch> upload_batch(DeviceCtx& dev, const std::vector<const JobBlob*>& jobs, uint8_t* mem,
                                    size_t mem_bytes, cudaStream_t copy_stream) {
    auto bp = std::make_unique<Batch>();
    Batch& b = *bp;
    b.dev = &dev;
    b.jobs = jobs;
    check(cudaSetDevice(dev.device), "set device");
    const size_t nj = jobs.size();
    // ---- device memory plan: per job, table blob then state then outputs
    Alloc A;
    struct Plan {
        size_t tables, lcol, cur, regret, sum, snap, reach, reach2, vals0, vals1, cards, cardm, tokproj, pb, jp, cf, cg,
            pooled, out_strategy, out_roots, out_carry, out_conv;
    };
    std::vector<Plan> plan(nj);
    for (size_t j = 0; j < nj; ++j) {
        const JobBlob& jb = *jobs[j];
        const JobImage& J = *jb.img;
        Plan& P = plan[j];
        P.tables = A.take(jb.bytes);
        P.lcol = A.take(4ull * jb.arr<uint32_t>(JobBlob::LEAF_COFF)[2 * J.nrows_net]);
        P.cur = A.take(4ull * J.ncells);
        P.regret = A.take(4ull * J.ncells);
        P.sum = A.take(4ull * J.ncells);
        P.snap = A.take(4ull * J.ncells);
        P.reach = A.take(4ull * J.reach_len);
        P.reach2 = J.cfg.snapshots ? A.take(4ull * J.reach_len) : 0;
        P.vals0 = A.take(4ull * J.val_len[0]);
        P.vals1 = A.take(4ull * J.val_len[1]);
        bool net = dev.have_net, exact = net && dev.precise;
        P.cards = net ? A.take(4ull * 2 * 10 * NET_TYPE) : 0;
        P.cardm = net ? A.take(4ull * 2 * 10 * 3 * NET_POOL) : 0;
        P.tokproj = (net && !exact) ? A.take(4ull * 10 * NET_C) : 0;
        P.pb = exact ? A.take(4ull * J.nrows_net * NET_D) : 0;
        P.jp = exact ? A.take(4ull * J.nrows_net * NET_JW) : 0;
        P.cf = net ? A.take(4ull * J.ncfg * NET_D) : 0;
        P.cg = net ? A.take(4ull * J.ncfg * NET_POOL) : 0;
        P.pooled = exact ? A.take(4ull * J.nrows_net * 2 * NET_POOL) : 0;
        P.out_strategy = A.take(4ull * J.ncells);
        P.out_roots = A.take(4ull * J.ncarried * (J.root_nc[0] + J.root_nc[1]));
        P.out_carry = J.cfg.snapshots ? A.take(2ull * (jb.nsnaps_kept - 1) * jb.carry_width) : 0;
        P.out_conv = A.take(8ull * (J.root_nc[0] + J.root_nc[1]));
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
                    add_row_items(items, j, r.first, r.count, r.out_first, jobs[j]->arr<uint32_t>(JobBlob::ROW_OFF));
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
    std::vector<uint32_t> row_job, row_local, cfg_job, cfg_local, dup;
    const bool fast = dev.have_net && !dev.precise;
    for (uint32_t j = 0; j < nj; ++j) {
        const JobImage& J = *jobs[j]->img;
        // the tensor-core trunk runs on each distinct public row once; the
        // other rows take their representative's P and jp (k_board_dup)
        const uint32_t* rep = jobs[j]->arr<uint32_t>(JobBlob::ROW_REP);
        for (uint32_t r = 0; r < J.nrows_net; ++r) {
            if (fast && rep[r] != r) {
                dup.insert(dup.end(), {j, r, rep[r]});
                continue;
            }
            row_job.push_back(j);
            row_local.push_back(r);
        }
        for (uint32_t c = 0; c < J.ncfg; ++c) { cfg_job.push_back(j); cfg_local.push_back(c); }
        b.max_carried = std::max(b.max_carried, J.ncarried);
        b.node_updates += (double)J.nodes * (double)J.cfg.iters;
        b.leaf_evals += (double)J.nrows_net * (double)J.cfg.iters;
    }
    b.total_rows = (uint32_t)row_job.size();
    b.n_dup = (uint32_t)(dup.size() / 3);
    b.total_cfgs = (uint32_t)cfg_job.size();
    std::vector<size_t> o_f16(nj, 0);
    size_t o_gpool = 0, o_gjp = 0, o_gmass = 0, o_gpb = 0, o_gz = 0, o_tiles = 0, o_err = 0;
    struct HeadTile { uint32_t job, first, count, pad; };
    std::vector<HeadTile> head_tiles;
    std::vector<uint32_t> tile_base(nj, 0);
    std::vector<size_t> f16_bytes(nj, 0);
    if (fast) {
        // per-job tiles of 128 network rows; the pooled beliefs and the join
        // output live as per-tile operand images (128-byte swizzled, K-major)
        for (uint32_t j = 0; j < nj; ++j) {
            tile_base[j] = (uint32_t)head_tiles.size();
            for (uint32_t f = 0; f < jobs[j]->img->nrows_net; f += 128)
                head_tiles.push_back({j, f, std::min<uint32_t>(128, jobs[j]->img->nrows_net - f), 0});
        }
        const size_t NT = head_tiles.size();
        for (size_t j = 0; j < nj; ++j) {
            const JobImage& J = *jobs[j]->img;
            // f(c) as readout operand images: 128 configs x 256 per pass, per player
            // g(c) as pooling operand images: 64 x 128 configs per chunk, per player
            const size_t npass = (J.ncfg_player[0] + 127) / 128 + (J.ncfg_player[1] + 127) / 128;
            f16_bytes[j] = (65536ull + 16384ull) * npass;
            o_f16[j] = A.take(f16_bytes[j]);
        }
        size_t R = row_job.size() + b.n_dup;
        o_gpool = A.take(32768ull * NT);  // [tile][player 0 | player 1] 128 x 64 images
        o_gjp = A.take(2ull * R * NET_JW);
        o_gmass = A.take(8ull * R);
        o_gpb = A.take(65536ull * NT);    // [tile] 128 x 256 P image (row-swizzled 16-byte chunks)
        o_gz = A.take(32768ull * NT);     // [tile] 128 x 128 image
        o_tiles = A.take(sizeof(HeadTile) * head_tiles.size());
        o_err = A.take(16);
    }
    size_t o_jobs = A.take(sizeof(wcdev::JobDev) * nj);
    size_t o_items = A.take(sizeof(wcdev::WorkItem) * items.size());
    size_t o_rj = A.take(4ull * row_job.size()), o_rl = A.take(4ull * row_local.size());
    size_t o_cj = A.take(4ull * cfg_job.size()), o_cl = A.take(4ull * cfg_local.size());
    size_t o_dup = A.take(4ull * dup.size());
    b.dbytes = A.at;
    if (mem) {
        if (b.dbytes > mem_bytes) throw std::runtime_error("batch plan exceeds its arena");
        b.dmem = mem;
        b.owns_dmem = false;
    } else {
        check(cudaMalloc((void**)&b.dmem, std::max<size_t>(b.dbytes, 256)), "batch device memory");
    }
    uint8_t* D = b.dmem;
    // ---- descriptors
    b.hj.resize(nj);
    std::vector<uint32_t> row_base(nj, 0);
    for (size_t j = 1; j < nj; ++j) row_base[j] = row_base[j - 1] + jobs[j - 1]->img->nrows_net;
    b.out_off.resize(4 * nj);
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
        d.row_gpu = t32(JobBlob::ROW_GPU);
        d.cphi = tf(JobBlob::CPHI);
        d.cplayer = t8(JobBlob::CPLAYER);
        d.card_feat = tf(JobBlob::CARD_FEAT);
        d.root_belief = tf(JobBlob::ROOT_BELIEF);
        d.carried = tf(JobBlob::CARRIED);
        d.carry_off = t32(JobBlob::CARRY_OFF);
        d.cfg_col = t32(JobBlob::CFG_COL);
        d.leaf_col = reinterpret_cast<uint32_t*>(D + P.lcol);
        d.ncfg_player[0] = J.ncfg_player[0];
        d.ncfg_player[1] = J.ncfg_player[1];
        d.row_base = row_base[j];
        d.tile_base = tile_base[j];
        d.f16 = fast ? reinterpret_cast<uint16_t*>(D + o_f16[j]) : nullptr;
        d.g16 = fast ? reinterpret_cast<uint16_t*>(D + o_f16[j] + 65536ull * ((J.ncfg_player[0] + 127) / 128 +
                                                                             (J.ncfg_player[1] + 127) / 128))
                     : nullptr;
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
            d.tokproj = dev.precise ? nullptr : reinterpret_cast<float*>(D + P.tokproj);
            d.pb = dev.precise ? reinterpret_cast<float*>(D + P.pb) : nullptr;
            d.jp = dev.precise ? reinterpret_cast<float*>(D + P.jp) : nullptr;
            d.cf = reinterpret_cast<float*>(D + P.cf);
            d.cg = reinterpret_cast<float*>(D + P.cg);
            d.pooled = dev.precise ? reinterpret_cast<float*>(D + P.pooled) : nullptr;
        }
        d.out_strategy = reinterpret_cast<float*>(D + P.out_strategy);
        d.out_roots = reinterpret_cast<float*>(D + P.out_roots);
        d.out_carry = J.cfg.snapshots ? reinterpret_cast<uint16_t*>(D + P.out_carry) : nullptr;
        d.out_conv = reinterpret_cast<float*>(D + P.out_conv);
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
        b.out_off[4 * j] = P.out_strategy;
        b.out_off[4 * j + 1] = P.out_roots;
        b.out_off[4 * j + 2] = P.out_carry;
        b.out_off[4 * j + 3] = P.out_conv;
    }
    b.d_jobs = reinterpret_cast<wcdev::JobDev*>(D + o_jobs);
    b.d_items = reinterpret_cast<wcdev::WorkItem*>(D + o_items);
    b.d_row_job = reinterpret_cast<uint32_t*>(D + o_rj);
    b.d_row_local = reinterpret_cast<uint32_t*>(D + o_rl);
    b.d_cfg_job = reinterpret_cast<uint32_t*>(D + o_cj);
    b.d_cfg_local = reinterpret_cast<uint32_t*>(D + o_cl);
    b.d_dup = reinterpret_cast<uint32_t*>(D + o_dup);
    if (fast) {
        b.g_pool_img = reinterpret_cast<uint16_t*>(D + o_gpool);
        b.g_jp = reinterpret_cast<uint16_t*>(D + o_gjp);
        b.g_mass = reinterpret_cast<float*>(D + o_gmass);
        b.g_pb = reinterpret_cast<uint16_t*>(D + o_gpb);
        b.g_zout_img = reinterpret_cast<uint16_t*>(D + o_gz);
        b.d_head_tiles = D + o_tiles;
        b.n_head_tiles = (uint32_t)head_tiles.size();
        b.d_err = reinterpret_cast<int*>(D + o_err);
    }
    cudaStream_t s = copy_stream ? copy_stream : dev.stream;
    for (size_t j = 0; j < nj; ++j)
        check(cudaMemcpyAsync(D + plan[j].tables, jobs[j]->host, jobs[j]->bytes, cudaMemcpyHostToDevice, s), "upload job tables");
    check(cudaMemcpyAsync(b.d_jobs, b.hj.data(), sizeof(wcdev::JobDev) * nj, cudaMemcpyHostToDevice, s), "upload descriptors");
    check(cudaMemcpyAsync(b.d_items, items.data(), sizeof(wcdev::WorkItem) * items.size(), cudaMemcpyHostToDevice, s), "upload items");
    if (!row_job.empty()) {
        check(cudaMemcpyAsync(b.d_row_job, row_job.data(), 4 * row_job.size(), cudaMemcpyHostToDevice, s), "upload rows");
        check(cudaMemcpyAsync(b.d_row_local, row_local.data(), 4 * row_local.size(), cudaMemcpyHostToDevice, s), "upload rows");
    }
    if (!dup.empty())
        check(cudaMemcpyAsync(b.d_dup, dup.data(), 4 * dup.size(), cudaMemcpyHostToDevice, s), "upload duplicate rows");
    // the readout column of every leaf-config entry, from the uploaded tables
    wcdev::launch_leaf_col(b.d_jobs, (uint32_t)nj, s);
    check(cudaGetLastError(), "leaf columns");
    if (!cfg_job.empty()) {
        check(cudaMemcpyAsync(b.d_cfg_job, cfg_job.data(), 4 * cfg_job.size(), cudaMemcpyHostToDevice, s), "upload cfgs");
        check(cudaMemcpyAsync(b.d_cfg_local, cfg_local.data(), 4 * cfg_local.size(), cudaMemcpyHostToDevice, s), "upload cfgs");
    }
    if (fast) {
        if (!head_tiles.empty())
            check(cudaMemcpyAsync(b.d_head_tiles, head_tiles.data(), sizeof(HeadTile) * head_tiles.size(),
                                  cudaMemcpyHostToDevice, s), "upload head tiles");
        check(cudaMemsetAsync(b.d_err, 0, 16, s), "clear error flag");
        // padding rows and configs of the operand images stay zero
        check(cudaMemsetAsync(b.g_pool_img, 0, 32768ull * head_tiles.size(), s), "clear pooled images");
        for (size_t j = 0; j < nj; ++j)
            check(cudaMemsetAsync(D + o_f16[j], 0, f16_bytes[j], s), "clear readout images");
    }
    if (!copy_stream) check(cudaStreamSynchronize(s), "batch upload");
    return bp;
}

// The device bytes a job takes in a batch plan: its tables, state and
// outputs (as upload_batch lays them out), its share of the batch-wide
// tensor-core images (per 128-row tile and per network row) and of the work
// items, rounded up. Used to size waves before the exact plan is made.
size_t job_device_bytes(const DeviceCtx& dev, const JobBlob& jb) {
    const JobImage& J = *jb.img;
    auto r = [](size_t x) { return (x + 255) & ~(size_t)255; };
    size_t b = r(jb.bytes) + r(4ull * jb.arr<uint32_t>(JobBlob::LEAF_COFF)[2 * J.nrows_net]) + 4 * r(4ull * J.ncells) +
               r(4ull * J.reach_len) * (J.cfg.snapshots ? 2 : 1) +
               r(4ull * J.val_len[0]) + r(4ull * J.val_len[1]) + r(4ull * J.ncells) +
               r(4ull * J.ncarried * (J.root_nc[0] + J.root_nc[1])) + r(8ull * (J.root_nc[0] + J.root_nc[1]));
    if (J.cfg.snapshots) b += r(2ull * (jb.nsnaps_kept - 1) * jb.carry_width);
    const bool net = dev.have_net, exact = net && dev.precise;
    if (net) {
        b += r(4ull * 2 * 10 * NET_TYPE) + r(4ull * 2 * 10 * 3 * NET_POOL) + r(4ull * J.ncfg * NET_D) +
             r(4ull * J.ncfg * NET_POOL);
        if (exact) {
            b += r(4ull * J.nrows_net * NET_D) + r(4ull * J.nrows_net * NET_JW) + r(4ull * J.nrows_net * 2 * NET_POOL);
        } else {
            const size_t tiles = (J.nrows_net + 127) / 128;
            const size_t npass = (J.ncfg_player[0] + 127) / 128 + (J.ncfg_player[1] + 127) / 128;
            b += r(4ull * 10 * NET_C) + r((65536ull + 16384ull) * npass) + tiles * (32768ull + 65536ull + 32768ull + 16) +
                 J.nrows_net * (2ull * NET_JW + 8);
        }
    }
    // descriptors, work items (one per <= 256 tasks of a level range) and row / config indices
    b += sizeof(wcdev::JobDev) + 16ull * (J.ncells / 128 + 4 * J.nlevels + 8) + 8ull * (J.nrows_net + J.ncfg) +
         12ull * J.nrows_net;
    return b + b / 64 + 4096;
}

// ---------------------------------------------------------- the schedule

namespace {

float factor(float t, float p) {
    if (std::isinf(p)) return p > 0.0f ? 1.0f : 0.0f;
    float x = std::pow(t, p);
    return x / (x + 1.0f);
}

// WC_DEBUG_SYNC=1 in the environment: after every timed kernel class the
// stream is synchronised and checked, so a device fault is reported with the
// class that raised it (for diagnosis only; it serialises the solve).
bool debug_sync() {
    static const bool on = [] {
        const char* e = std::getenv("WC_DEBUG_SYNC");
        return e && e[0] == '1';
    }();
    return on;
}

const char* class_name(int cls) {
    static const char* names[N_TC] = {"per-solve network", "leaf evaluation", "regret-matching rows",
                                      "value gathers", "reach gathers", "snapshots", "phase 2", "init", "total",
                                      "k_pool_fast", "k_join_fast", "k_head_fast", "k_trunk_fast"};
    return cls >= 0 && cls < N_TC ? names[cls] : "kernel";
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
        if (debug_sync()) {  // WC_DEBUG_SYNC: each class's launches finish and are checked before the next
            f();
            check(cudaStreamSynchronize(s), class_name(cls));
            check(cudaGetLastError(), class_name(cls));
            return;
        }
        if (!b.profile) { f(); return; }
        const int e0 = (int)b.events_used;
        check(cudaEventRecord(next_event(), s), "event");
        f();
        const int e1 = (int)b.events_used;
        check(cudaEventRecord(next_event(), s), "event");
        b.event_class.push_back(cls);
        b.event_class.push_back(e0);
        b.event_class.push_back(e1);
    }
    const wcdev::WorkItem* it(const Batch::Range& r) const { return I + r.off; }

    // Full or single-mover reach propagation below the seeded root.
    void propagate(int strat_sel, int which_reach, int mover_mask, int sum_update, float dg) {
        for (uint32_t lv = 1; lv < b.nlevels; ++lv)
            for (int q = 0; q < 2; ++q) {
                if (!(mover_mask & (1 << q))) continue;
                const Batch::Range& r = b.rg[lv * 2 + q];
                timed(TC_REACH, [&] { b.count_launch(r.n), wcdev::launch_rgather(J, it(r), r.n, strat_sel, which_reach, sum_update, dg, s); });
            }
    }

    void leaf_values(int p, int pool_mask) {
        timed(TC_LEAF, [&] { leaf_values_(p, pool_mask); });
    }
    void leaf_values_(int p, int pool_mask) {
        DeviceCtx& dv = *b.dev;
        if (dv.have_net && !dv.precise) {
            timed(TC_POOL, [&] {
                b.count_launch((pool_mask ? b.n_head_tiles : 0)), wcdev::launch_pool_fast(J, b.d_head_tiles, b.n_head_tiles, pool_mask, b.g_pool_img, b.g_mass, dv.half,
                                        b.d_err, dv.fast.wait_ns, s);
            });
            timed(TC_JOIN, [&] {
                b.count_launch(b.n_head_tiles), wcdev::launch_join_fast(J, b.d_head_tiles, b.n_head_tiles, dv.fast, p, b.g_pool_img, b.g_jp,
                                        b.g_zout_img, b.d_err, s);
            });
            timed(TC_HEAD, [&] {
                b.count_launch(b.n_head_tiles), wcdev::launch_head_fast(J, b.d_head_tiles, b.n_head_tiles, dv.fast, p, b.g_zout_img, b.g_pb, b.g_mass,
                                        b.d_err, s);
            });
        } else if (dv.have_net) {
            if (pool_mask) b.count_launch((pool_mask ? b.total_rows : 0)), wcdev::launch_pool(J, b.d_row_job, b.d_row_local, b.total_rows, pool_mask, s);
            b.count_launch(b.total_rows), wcdev::launch_join_readout(J, b.d_row_job, b.d_row_local, b.total_rows, p, dv.W, dv.B, dv.LN, s);
        } else {
            b.count_launch(b.netrows_all.n), wcdev::launch_netrows_zero(J, it(b.netrows_all), b.netrows_all.n, p, s);
        }
        b.count_launch(b.term_all.n), wcdev::launch_terminal(J, it(b.term_all), b.term_all.n, p, s);
    }

    void backprop(int p, int mode, int strat_sel, float da, float db, float predict) {
        for (int lv = (int)b.nlevels - 1; lv >= 0; --lv) {
            const Batch::Range& rr = b.rows[lv * 2 + p];
            const Batch::Range& vr = b.vg[lv * 2 + p];
            timed(TC_ROWS, [&] { b.count_launch(rr.n), wcdev::launch_rows(J, it(rr), rr.n, p, mode, strat_sel, da, db, predict, s); });
            timed(TC_VGATHER, [&] { b.count_launch(vr.n), wcdev::launch_vgather(J, it(vr), vr.n, p, s); });
        }
    }

    void carries(int snap_index) {
        b.count_launch(b.jobs.size()), wcdev::launch_seed_root(J, (uint32_t)b.jobs.size(), 1, -1, s);
        propagate(wcdev::STRAT_SNAP, 1, 3, 0, 1.0f);
        b.count_launch(b.exits_all.n), wcdev::launch_carry(J, it(b.exits_all), b.exits_all.n, snap_index, s);
    }
};

}  // namespace

void enqueue_leaf_values(Batch& b, int p) {
    if (b.jobs.empty()) return;
    b.launches = 0;
    DeviceCtx& dv = *b.dev;
    check(cudaSetDevice(dv.device), "set device");
    Sched S(b);
    const uint32_t nj = (uint32_t)b.jobs.size();
    auto mark = [&](int i) {
        if (!b.profile) return;
        if (!b.marks[i]) check(cudaEventCreate(&b.marks[i]), "event");
        check(cudaEventRecord(b.marks[i], S.s), "event");
    };
    mark(0);
    if (dv.have_net) {
        S.timed(TC_NET_SOLVE, [&] {
            b.count_launch(nj), wcdev::launch_cards(S.J, nj, dv.W, dv.B, S.s);
            if (dv.precise) {
                b.count_launch(b.total_rows), wcdev::launch_trunk(S.J, b.d_row_job, b.d_row_local, b.total_rows, dv.W, dv.B, dv.LN, S.s);
            } else {
                S.timed(TC_TRUNK, [&] {
                    b.count_launch(nj), wcdev::launch_tokproj(S.J, nj, dv.W, S.s);
                    b.count_launch(b.total_rows), wcdev::launch_trunk_fast(S.J, b.d_row_job, b.d_row_local, b.total_rows, dv.fast.trunk_tiles, dv.W,
                                             dv.B, dv.LN, dv.fast, b.g_pb, b.g_jp, b.d_err, S.s);
                    b.count_launch(b.n_dup ? 1 : 0), wcdev::launch_board_dup(S.J, b.d_dup, b.n_dup, b.g_pb, b.g_jp, S.s);
                });
            }
            b.count_launch(b.total_cfgs), wcdev::launch_configs(S.J, b.d_cfg_job, b.d_cfg_local, b.total_cfgs, dv.W, dv.B, dv.LN, S.s);
            if (!dv.precise) b.count_launch(b.total_cfgs), wcdev::launch_pack_f16(S.J, b.d_cfg_job, b.d_cfg_local, b.total_cfgs, dv.half, S.s);
        });
    }
    S.timed(TC_INIT, [&] {
        b.count_launch(b.rows_all.n), wcdev::launch_init_rows(S.J, S.it(b.rows_all), b.rows_all.n, S.s);
        b.count_launch(b.jobs.size()), wcdev::launch_seed_root(S.J, nj, 0, -1, S.s);
    });
    S.propagate(wcdev::STRAT_CUR, 0, 3, 1, 1.0f);
    mark(1);
    S.leaf_values(p, 3);
    mark(2);
    check(cudaGetLastError(), "leaf values launch");
}

void download_leaf_values(Batch& b, size_t job, int p, float* out) {
    const JobImage& J = *b.jobs[job]->img;
    const uint32_t* lr_vidx = b.jobs[job]->arr<uint32_t>(JobBlob::LR_VIDX);
    const uint32_t* lr_nc = b.jobs[job]->arr<uint32_t>(JobBlob::LR_NC);
    const wcdev::JobDev& d = b.hj[job];
    cudaStream_t s = b.dev->stream;
    std::vector<float> vals(J.val_len[p]);
    check(cudaMemcpyAsync(vals.data(), d.vals[p], 4ull * J.val_len[p], cudaMemcpyDeviceToHost, s), "download values");
    check(cudaStreamSynchronize(s), "download values");
    size_t at = 0;
    for (uint32_t r = 0; r < J.nrows_net; ++r) {
        uint32_t v0 = lr_vidx[2 * r + p], n = lr_nc[2 * r + p];
        for (uint32_t c = 0; c < n; ++c) out[at++] = vals[v0 + c];
    }
}

void download_board_rows(Batch& b, size_t job, float* pb, float* jp) {
    const JobImage& J = *b.jobs[job]->img;
    const wcdev::JobDev& d = b.hj[job];
    cudaStream_t s = b.dev->stream;
    const size_t n = J.nrows_net;
    if (b.dev->precise) {
        if (pb) check(cudaMemcpyAsync(pb, d.pb, 4 * n * NET_D, cudaMemcpyDeviceToHost, s), "download P");
        if (jp) check(cudaMemcpyAsync(jp, d.jp, 4 * n * NET_JW, cudaMemcpyDeviceToHost, s), "download jp");
        check(cudaStreamSynchronize(s), "download rows");
        return;
    }
    const size_t ntile = (n + 127) / 128;
    std::vector<uint16_t> hpt(ntile * 32768), hp(n * NET_D), hj(n * NET_JW);
    check(cudaMemcpyAsync(hpt.data(), b.g_pb + (size_t)d.tile_base * 32768, 2 * hpt.size(), cudaMemcpyDeviceToHost, s),
          "download P");
    check(cudaMemcpyAsync(hj.data(), b.g_jp + (size_t)d.row_base * NET_JW, 2 * n * NET_JW, cudaMemcpyDeviceToHost, s), "download jp");
    check(cudaStreamSynchronize(s), "download rows");
    for (size_t r = 0; r < n; ++r) {  // undo the per-tile layout of P
        const size_t rt = r % 128, base = (r / 128) * 32768 + rt * 256;
        for (size_t c = 0; c < NET_D; ++c) hp[r * NET_D + c] = hpt[base + (((c >> 3) ^ (rt & 7)) << 3) + (c & 7)];
    }
    auto f = [](uint16_t v) { return __half2float(__ushort_as_half(v)); };  // P and jp are f16 in both modes
    if (pb) for (size_t i = 0; i < hp.size(); ++i) pb[i] = f(hp[i]);
    if (jp) for (size_t i = 0; i < hj.size(); ++i) jp[i] = f(hj[i]);
}

void enqueue_solve(Batch& b) {
    if (b.jobs.empty()) return;
    b.launches = 0;
    DeviceCtx& dv = *b.dev;
    check(cudaSetDevice(dv.device), "set device");
    // each solve reports its own tensor-core wait failures
    if (b.d_err) check(cudaMemsetAsync(b.d_err, 0, 16, dv.stream), "clear error flag");
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
            b.count_launch(nj), wcdev::launch_cards(S.J, nj, dv.W, dv.B, S.s);
            if (dv.precise) {
                b.count_launch(b.total_rows), wcdev::launch_trunk(S.J, b.d_row_job, b.d_row_local, b.total_rows, dv.W, dv.B, dv.LN, S.s);
            } else {
                S.timed(TC_TRUNK, [&] {
                    b.count_launch(nj), wcdev::launch_tokproj(S.J, nj, dv.W, S.s);
                    b.count_launch(b.total_rows), wcdev::launch_trunk_fast(S.J, b.d_row_job, b.d_row_local, b.total_rows, dv.fast.trunk_tiles, dv.W,
                                             dv.B, dv.LN, dv.fast, b.g_pb, b.g_jp, b.d_err, S.s);
                    b.count_launch(b.n_dup ? 1 : 0), wcdev::launch_board_dup(S.J, b.d_dup, b.n_dup, b.g_pb, b.g_jp, S.s);
                });
            }
            b.count_launch(b.total_cfgs), wcdev::launch_configs(S.J, b.d_cfg_job, b.d_cfg_local, b.total_cfgs, dv.W, dv.B, dv.LN, S.s);
            if (!dv.precise) b.count_launch(b.total_cfgs), wcdev::launch_pack_f16(S.J, b.d_cfg_job, b.d_cfg_local, b.total_cfgs, dv.half, S.s);
        });
    }
    // Solver::new: uniform strategy, reaches, reach-weighted sum seed, snapshot 0
    S.timed(TC_INIT, [&] {
        b.count_launch(b.rows_all.n), wcdev::launch_init_rows(S.J, S.it(b.rows_all), b.rows_all.n, S.s);
        b.count_launch(b.jobs.size()), wcdev::launch_seed_root(S.J, nj, 0, -1, S.s);
    });
    S.propagate(wcdev::STRAT_CUR, 0, 3, 1, 1.0f);
    int snap_index = 0;
    if (cfg.snapshots || cfg.iters == 0) {
        b.count_launch(b.rows_all.n), wcdev::launch_copy_cur_to_snap(S.J, S.it(b.rows_all), b.rows_all.n, S.s);
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
                b.count_launch(b.rows_all.n), wcdev::launch_snapshot(S.J, S.it(b.rows_all), b.rows_all.n, touched[0], touched[1], S.s);
            });
            if (cfg.snapshots && done != cfg.iters) S.carries(snap_index);
            ++snap_index;
        }
        steps[p] += 1;
    }
    S.timed(TC_SNAP, [&] { b.count_launch(b.cells_all.n), wcdev::launch_unsort(S.J, S.it(b.cells_all), b.cells_all.n, S.s); });
    // Phase 2: one fixed-policy pass per carried root (search.rs:1851-1871)
    mark(1);
    for (uint32_t r = 0; r < b.max_carried; ++r) {
        b.count_launch(b.jobs.size()), wcdev::launch_seed_root(S.J, nj, 0, (int)r, S.s);
        S.propagate(wcdev::STRAT_SNAP, 0, 3, 0, 1.0f);
        for (int p = 0; p < 2; ++p) {
            S.leaf_values(p, p == 0 ? 3 : 0);
            S.backprop(p, wcdev::BACK_VALUE, wcdev::STRAT_SNAP, 0.0f, 0.0f, 0.0f);
            b.count_launch(nj), wcdev::launch_collect_root(S.J, nj, (int)r, p, S.s);
        }
    }
    mark(2);
    check(cudaGetLastError(), "solve launch");
}

void enqueue_nash_conv(Batch& b) {
    if (b.jobs.empty()) return;
    b.launches = 0;
    DeviceCtx& dv = *b.dev;
    check(cudaSetDevice(dv.device), "set device");
    Sched S(b);
    const uint32_t nj = (uint32_t)b.jobs.size();
    // search.rs:1884-1907: reaches of the live root belief under the average,
    // both players' leaf beliefs pooled once, then per player a value pass
    // and a best-response pass over the same leaf values
    b.count_launch(nj), wcdev::launch_seed_root(S.J, nj, 0, -1, S.s);
    S.propagate(wcdev::STRAT_SNAP, 0, 3, 0, 1.0f);
    for (int p = 0; p < 2; ++p) {
        S.leaf_values(p, p == 0 ? 3 : 0);
        S.backprop(p, wcdev::BACK_VALUE, wcdev::STRAT_SNAP, 0.0f, 0.0f, 0.0f);
        b.count_launch(nj), wcdev::launch_collect_conv(S.J, nj, 0, p, S.s);
        S.backprop(p, wcdev::BACK_BEST, wcdev::STRAT_SNAP, 0.0f, 0.0f, 0.0f);
        b.count_launch(nj), wcdev::launch_collect_conv(S.J, nj, 1, p, S.s);
    }
    check(cudaGetLastError(), "nash conv launch");
}

void download_conv(Batch& b, size_t job, float* out) {
    const JobImage& J = *b.jobs[job]->img;
    cudaStream_t s = b.dev->stream;
    check(cudaMemcpyAsync(out, b.dmem + b.out_off[4 * job + 3], 8ull * (J.root_nc[0] + J.root_nc[1]),
                          cudaMemcpyDeviceToHost, s), "download conv");
    check(cudaStreamSynchronize(s), "download conv");
}

void check_batch_error(Batch& b, cudaStream_t stream) {
    if (!b.d_err) return;
    cudaStream_t s = stream ? stream : b.dev->stream;
    int e[4] = {0, 0, 0, 0};
    check(cudaMemcpyAsync(e, b.d_err, 16, cudaMemcpyDeviceToHost, s), "read error flag");
    check(cudaStreamSynchronize(s), "read error flag");
    if (e[0])
        throw std::runtime_error("a tensor-core wait exceeded its time limit (code " + std::to_string(e[0]) +
                                 (e[0] > 10 ? ", in-flight work did not drain: reset the device context" : "") + ")");
}

void download(Batch& b, size_t job, float* strategy, float* roots, uint16_t* carries, cudaStream_t stream) {
    const JobBlob& jb = *b.jobs[job];
    const JobImage& J = *jb.img;
    cudaStream_t s = stream ? stream : b.dev->stream;
    if (strategy)
        check(cudaMemcpyAsync(strategy, b.dmem + b.out_off[4 * job], 4ull * J.ncells, cudaMemcpyDeviceToHost, s), "download strategy");
    if (roots)
        check(cudaMemcpyAsync(roots, b.dmem + b.out_off[4 * job + 1], 4ull * J.ncarried * (J.root_nc[0] + J.root_nc[1]),
                              cudaMemcpyDeviceToHost, s), "download roots");
    if (carries && J.cfg.snapshots)
        check(cudaMemcpyAsync(carries, b.dmem + b.out_off[4 * job + 2], 2ull * (jb.nsnaps_kept - 1) * jb.carry_width,
                              cudaMemcpyDeviceToHost, s), "download carries");
    check(cudaStreamSynchronize(s), "download");
}

}  // namespace wc
