// Device runtime: per-device weight banks, job blobs, device batches and the
// solve schedule. This replaces the reference's GPU executor
// (engine/src/gpu/device.rs:596-754) and its wave packer (gpu/wave.rs).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "cuda/device.h"
#include "host/job.h"
#include "host/netlayout.h"

namespace wc {

// The tensor-core kernels' limit on each mbarrier wait (%globaltimer ns);
// the work waited on takes microseconds.
constexpr uint64_t DEFAULT_WAIT_NS = 2000000000ull;

struct DeviceCtx {
    int device = 0;
    cudaStream_t stream = nullptr;
    float* W = nullptr;
    float* B = nullptr;
    float* LN = nullptr;
    bool have_net = false;
    bool precise = true;  // fp32 network in the reference's operation order
    bool half = true;     // the tensor-core net's per-iteration chain operands: f16 (true) or bf16
    uint64_t wait_ns = DEFAULT_WAIT_NS;  // limit of each tensor-core mbarrier wait (ns)
    uint64_t version = 0;
    NetLayout L;
    // 16-bit tensor-core copy of the network (fast path)
    uint8_t* fast_mem = nullptr;
    wcdev::FastNetDev fast{};
    std::mutex mu;  // one batch at a time per device
    // Waves (solve_waves): two device arenas reused across calls, so a wave's
    // tables upload on copy_stream while the previous wave solves on
    // `stream`; wave_budget bounds a wave's device bytes (0: set from the
    // free memory on first use, or from WC_WAVE_BYTES).
    uint8_t* arena[2] = {nullptr, nullptr};
    size_t arena_bytes[2] = {0, 0};
    cudaStream_t copy_stream = nullptr;
    size_t wave_budget = 0;
};

// Build the fast-path weight pack from the fp32 blob (host arrays) and upload it.
void build_fast_pack(DeviceCtx& d, const float* W, const float* B, const float* LN);

// A job's flattened tables in one pinned host blob (device copies keep the
// same layout).
struct JobBlob {
    std::unique_ptr<JobImage> img;
    uint8_t* host = nullptr;
    bool pinned = false;
    size_t bytes = 0;
    enum Arr {
        CELL_VIDX, ROW_OFF, ROW_PLAYER, VG_START, VGE_IDX, VGE_W, RG_START, RGE_SRC, RGE_W, DRAWP, CELL_REF,
        LR_RIDX, LR_NC, LR_VIDX, LEAF_COFF, LEAF_CIDX, TL_RIDX, TL_NC, TL_VIDX, TL_UTIL0, GPU_ROWS, CPHI,
        CPLAYER, CARD_FEAT, ROOT_BELIEF, CARRIED, CARRY_OFF, CFG_COL, ROW_REP, ROW_GPU, N_ARR
    };
    size_t off[N_ARR] = {};
    // A packed array. The blob is the only copy: make_blob releases the
    // image's vectors once they are packed, and keeps its scalars, level
    // ranges, exit nodes and snapshot list.
    template <class T>
    const T* arr(Arr a) const {
        return reinterpret_cast<const T*>(host + off[a]);
    }
    uint32_t nexit = 0, carry_width = 0, nsnaps_kept = 0;
    ~JobBlob();
};

std::unique_ptr<JobBlob> make_blob(std::unique_ptr<JobImage> img);

struct Batch {
    DeviceCtx* dev = nullptr;
    std::vector<const JobBlob*> jobs;
    uint8_t* dmem = nullptr;
    size_t dbytes = 0;
    bool owns_dmem = true;  // false when placed in a device arena of the context
    std::vector<wcdev::JobDev> hj;
    wcdev::JobDev* d_jobs = nullptr;
    struct Range { uint32_t off = 0, n = 0; };
    std::vector<wcdev::WorkItem> items;  // host copy
    wcdev::WorkItem* d_items = nullptr;
    uint32_t nlevels = 0;
    std::vector<Range> rows, vg, rg;  // [level * 2 + player]
    Range rows_all, cells_all, term_all, netrows_all, exits_all;
    uint32_t* d_row_job = nullptr;
    uint32_t* d_row_local = nullptr;
    uint32_t* d_cfg_job = nullptr;
    uint32_t* d_cfg_local = nullptr;
    uint32_t total_rows = 0, total_cfgs = 0, max_carried = 0;
    // tensor-core path: the row lists above hold each job's distinct public
    // rows only; d_dup holds (job, row, representative row) of the others
    uint32_t* d_dup = nullptr;
    uint32_t n_dup = 0;
    // fast network path: global per-row bf16 activations and per-job tiles
    uint16_t* g_pool_img = nullptr; // [tile][player][128 x POOL operand image]
    uint16_t* g_jp = nullptr;     // [rows][JW]
    uint16_t* g_pb = nullptr;     // [rows][D]
    uint16_t* g_zout_img = nullptr; // [tile][128 x JW operand image]: the join output
    float* g_mass = nullptr;      // [rows][2]: each player's reach mass at the row (pooling's normaliser)
    void* d_head_tiles = nullptr;
    uint32_t n_head_tiles = 0;
    int* d_err = nullptr;
    std::vector<size_t> out_off;  // per job: strategy, roots, carry, conv offsets in dmem
    double node_updates = 0.0;    // sum over jobs of nodes * iters
    double leaf_evals = 0.0;      // network-row joins per solve
    size_t table_bytes = 0;
    // Optional per-class device timing of a solve (CUDA events on the
    // runtime's stream): class ids are the TimeClass values.
    bool profile = false;
    std::vector<cudaEvent_t> events;
    std::vector<int> event_class;  // per timed region: class, start event, end event
    uint64_t launches = 0;         // kernel launches of the last enqueued solve or leaf evaluation
    void count_launch(uint64_t n) {
        if (n) ++launches;  // the launchers launch nothing for an empty range
    }
    size_t events_used = 0;
    cudaEvent_t marks[3] = {nullptr, nullptr, nullptr};  // solve start, Phase 2 start, solve end
    ~Batch();
};

// Set the error string of the calling thread.
void set_error(const std::string& e);
const std::string& last_error();

enum TimeClass {
    TC_NET_SOLVE = 0, TC_LEAF = 1, TC_ROWS = 2, TC_VGATHER = 3, TC_REACH = 4, TC_SNAP = 5, TC_PHASE2 = 6,
    TC_INIT = 7, TC_TOTAL = 8,
    // parts of TC_LEAF / TC_NET_SOLVE on the tensor-core path (not in the total twice)
    TC_POOL = 9, TC_JOIN = 10, TC_HEAD = 11, TC_TRUNK = 12, N_TC = 13
};
// After a profiled solve has finished: summed milliseconds per class.
void read_profile(Batch& b, double* ms /* N_TC */);

// Plan a batch and copy its tables to the device. Without `mem` the batch
// allocates its own device memory and the copies finish before the return;
// with `mem` (mem_bytes long, e.g. a wave arena) it is placed there, and with
// `copy_stream` the copies are only enqueued on that stream.
std::unique_ptr<Batch> upload_batch(DeviceCtx& dev, const std::vector<const JobBlob*>& jobs, uint8_t* mem = nullptr,
                                    size_t mem_bytes = 0, cudaStream_t copy_stream = nullptr);
// An upper bound of the device bytes a job takes in a batch (wave sizing).
size_t job_device_bytes(const DeviceCtx& dev, const JobBlob& jb);
// Run the whole solve on the device (asynchronous on dev.stream).
void enqueue_solve(Batch& b);
// Leaf evaluation alone: the per-solve network, the initial (uniform)
// reaches, then every network row's values for traverser p.
void enqueue_leaf_values(Batch& b, int p);
// Values of one job's network rows for traverser p, rows in reference
// leaf_rows order, each row's configs in support order.
void download_leaf_values(Batch& b, size_t job, int p, float* out);
// The per-solve board vectors P[rows][256] and join projections jp[rows][128]
// of one job as the network path stores them (the bf16 path stores them minus
// their row means).
void download_board_rows(Batch& b, size_t job, float* pb, float* jp);
// Copy one job's results to host buffers (synchronous). Any pointer may be null.
void download(Batch& b, size_t job, float* strategy, float* roots, uint16_t* carries, cudaStream_t stream = nullptr);

// After a solve: exploitability passes of every job's live root under its
// average strategy (Solver::nash_conv, search.rs:1884-1907); download_conv
// reads one job's 2 * (nc0 + nc1) root values: under the average, then the
// best responses, each [player 0 | player 1].
void enqueue_nash_conv(Batch& b);
void download_conv(Batch& b, size_t job, float* out);

void check(cudaError_t e, const char* what);
// Throw if a kernel recorded a bounded-wait timeout during the last solve.
void check_batch_error(Batch& b, cudaStream_t stream = nullptr);

}  // namespace wc
