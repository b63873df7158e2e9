/* War Chest batched CFR solver on B200 — the C ABI.
 *
 * This is the boundary a host engine binds (the reference engine would bind
 * it from Rust with an `extern "C"` block over these declarations). It replaces
 * the reference's GPU solve service:
 *
 *   reference (fplonka/war-chest-bot-9000-)              this ABI
 *   gpu::service::spawn      engine/src/gpu/service.rs:55-82   wc_init
 *   GpuClient::set_weights   engine/src/gpu/client.rs:259-275  wc_publish
 *   PackedJob::from_solver   engine/src/serialize.rs:340-360   wc_job_build
 *   GpuClient::submit        engine/src/gpu/client.rs:212-228  wc_submit / wc_solve_batch
 *   SolveHandle::wait        engine/src/gpu/client.rs:306-313  wc_wait
 *   SolveResult              engine/src/gpu/client.rs:115-122  wc_result
 *   selfplay root states     engine/src/selfplay.rs:59-81,588-905  wc_root_generate
 *
 * Conventions: every call returns 0 on success or a nonzero WC_E_* class;
 * the message is in a thread-local buffer read by wc_last_error. Inputs are
 * copied; results are owned by the library and released by wc_result_free.
 * Submit/wait are thread-safe. Results are bit-reproducible for a fixed
 * batch composition and device.
 */
#ifndef WC_B200_H
#define WC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    WC_OK = 0,
    WC_E_ARG = 1,     /* bad argument or malformed input */
    WC_E_CUDA = 2,    /* CUDA error (message has the detail) */
    WC_E_CAPPED = 3,  /* the tree hit the node cap; the caller falls back */
    WC_E_STATE = 4,   /* call out of order (unknown ticket, no weights, ...) */
    WC_E_NOMEM = 5    /* the batch does not fit on the device */
};

/* search::Cfg (engine/src/search.rs:50-95) and the Cfr rule (:133-138). */
typedef struct wc_solve_cfg {
    int32_t depth;      /* public-tree depth in coin plays */
    int32_t iters;      /* CFR iterations (alternating traversers) */
    int32_t snapshots;  /* keep log-spaced average snapshots and carries */
    int32_t reserved;
    float alpha, beta, gamma, predict; /* discounting rule; CFR+ = (inf, -inf, 2, 0) */
    uint64_t node_cap;  /* 0 = unlimited */
} wc_solve_cfg;

/* Weight blob of the v5 value network (engine/src/net.rs:507-528): dims must
 * be {5}; w, b, ln are the three flat f32 arrays. A NULL w means "no network"
 * (every non-terminal leaf is valued 0, like the reference's empty Nets). */
typedef struct wc_weights {
    uint32_t ndims;
    const uint32_t* dims;
    const float* w;
    uint64_t nw;
    const float* b;
    uint64_t nb;
    const float* ln;
    uint64_t nln;
} wc_weights;

typedef struct wc_ctx wc_ctx;
typedef struct wc_job wc_job;
typedef struct wc_batch wc_batch;

typedef struct wc_job_info {
    uint64_t nodes, cells, net_rows, terminal_leaves, configs, levels;
    uint64_t root_nc0, root_nc1, ncarried, carry_snapshots, carry_width, table_bytes;
} wc_job_info;

/* SolveResult: strategy in the reference's cell order (Solver::soff), root
 * values per carried root as [player 0 configs | player 1 configs], carried
 * beliefs per kept snapshot except the last as f16 over the exit nodes
 * (network rows then terminal leaves, both players). */
typedef struct wc_result {
    float* strategy;
    uint64_t ncells;
    float* root_values;
    uint64_t nroots;
    uint64_t root_width;
    uint16_t* carries;
    uint64_t carry_snapshots;
    uint64_t carry_width;
    uint64_t weight_version;
    /* SolveResult::oversize_route / card_exclusive_route: the job's device
     * reservation (mutable bytes plus the tables rounded up to a power of two,
     * serialize.rs:166-203) reached 4 / 6 GiB, so it was solved in a wave of
     * its own. */
    int32_t oversize_route;
    int32_t card_exclusive_route;
} wc_result;

/* ---- service ------------------------------------------------------------ */
/* Network arithmetic of a service (net_mode):
 *   WC_NET_EXACT  fp32 in the reference CPU network's operation order
 *                 (bit-identical to it);
 *   WC_NET_F16    tcgen05 tensor cores, f16 operands, fp32 accumulation: the
 *                 precision class of the reference GPU service's fast mode
 *                 (cuBLAS COMPUTE_32F_FAST_16F, engine/src/gpu/device.rs:2306-2330);
 *   WC_NET_BF16   the same kernels with bf16 operands for the per-iteration
 *                 chain (the pooling product, the four join layers and the
 *                 join output product: nearly all of a solve's network
 *                 work); the once-per-solve board trunk, its stored rows and
 *                 the readout <f(c), h> keep f16 operands, since the
 *                 readout amplifies operand rounding several times.
 * The values 0 / 1 keep the meaning of a `precise` flag (0 = tensor cores in
 * bf16, 1 = exact). */
enum { WC_NET_BF16 = 0, WC_NET_EXACT = 1, WC_NET_F16 = 2 };
int wc_init(int ndev, const int* devices, const wc_weights* w, int net_mode, wc_ctx** out);
int wc_publish(wc_ctx* ctx, const wc_weights* w, uint64_t* version);
/* Publish weights already resident on device `dev_index` (e.g. after an
 * NCCL broadcast): pointers to w_len / b_len / ln_len f32 device arrays. */
int wc_publish_device(wc_ctx* ctx, int dev_index, const float* w, const float* b, const float* ln,
                      uint64_t* version);
void wc_shutdown(wc_ctx* ctx);
int wc_last_error(char* buf, size_t n);
/* The v5 blob sizes: w, b, ln element counts. */
void wc_net_layout(uint64_t* w_len, uint64_t* b_len, uint64_t* ln_len);
/* Seeded weights: kind 0 He-normal, kind 1 the reference GPU tests' uniform
 * +-0.05 blob. Arrays sized by wc_net_layout. */
int wc_weights_fill(int kind, uint64_t seed, float* w, float* b, float* ln);
/* Horizon payoff per marker of lead (engine/src/state.rs:27-43). */
void wc_set_cap_marker_value(float v);

/* ---- roots and jobs ------------------------------------------------------ */
/* Root bytes are the reference's own root encoding, format v3
 * (engine/src/roots.rs:247-313, write_root / read_root): the State field by
 * field in little-endian (write_state, roots.rs:150-180), then per player a
 * u32 count n, n configs (hand[5], fd[5], inflight or 0xff) and n f32
 * weights. A Rust engine hands `roots::write_root(&mut buf, &state, &bel)`'s
 * bytes straight to wc_job_build. */

/* A seeded root: make_game(seed, random draft) then `plies` uniform decisions
 * with the Bayes belief filter, then on to the next MainPlay
 * (engine/src/selfplay.rs:59-81,588-905), in the root encoding above. */
int wc_root_generate(uint64_t seed, int plies, int random_draft, uint8_t* buf, size_t cap, size_t* len);
/* A belief-heavy root: wc_root_generate's position,
 * each player's belief replaced by up to ncfg configs drawn (seeded, without
 * replacement) from every config consistent with the public counts
 * (rebel.rs:270 enumerate_configs), the true config always among them, with
 * Dirichlet(1) weights. Same byte form as wc_root_generate. */
int wc_root_generate_wide(uint64_t seed, int plies, int random_draft, uint32_t ncfg, uint8_t* buf, size_t cap,
                          size_t* len);
/* Build and flatten the subgame tree at a serialized root. carried holds
 * ncarried root pairs (player 0 then player 1 over the root supports); with
 * ncarried == 0 the live root belief is valued. */
int wc_job_build(const uint8_t* root, size_t len, const wc_solve_cfg* cfg, const float* carried, uint32_t ncarried,
                 wc_job** out);
/* Build many jobs at once on `threads` host threads (0: one per hardware
 * thread), each root taken in turn from a shared queue: the parallel form of
 * the reference tape builder's loop (engine/examples/wave_tape.rs:48-61,
 * Solver::new + PackedJob::from_solver per root, with capped roots counted and
 * skipped). All roots share cfg. carried and ncarried are wc_job_build's
 * arguments per root (carried[i] holds ncarried[i] root pairs); either array
 * may be NULL for no carried beliefs anywhere. status[i] is wc_job_build's
 * status for root i; out[i] is its job, or NULL when the build did not succeed
 * (WC_E_CAPPED for a tree over the node cap). Each job is the one
 * wc_job_build makes from the same arguments, byte for byte. Returns WC_OK
 * when every root either built or was capped, else the first other failure
 * (its message through wc_last_error); the jobs that did build are the
 * caller's in either case. */
int wc_job_build_batch(const uint8_t* const* roots, const size_t* lens, size_t n, const wc_solve_cfg* cfg,
                       const float* const* carried, const uint32_t* ncarried, int threads, wc_job** out,
                       int* status);
int wc_job_info_get(const wc_job* job, wc_job_info* out);
void wc_job_free(wc_job* job);
/* A 64-bit digest (FNV-1a) of the job's flattened tables, for checking that
 * two builds are identical and as a cache key. */
int wc_job_digest(const wc_job* job, uint64_t* out);
/* The reference's job bytes, WCJ8 (engine/src/serialize.rs:1051-1262 to_bytes
 * / from_bytes, the tables of serialize.rs:689-955 from_solver; docs/TREE.md),
 * for interop with tapes and services that speak it.
 * wc_wcj8_from_root: the subgame of a root (root encoding above) built and
 * written as PackedJob::from_solver(...).to_bytes() would write it, with
 * `net_dims` as the meta's network shape; *len is set to the byte count,
 * and WC_E_ARG returned when cap is smaller (call with cap 0 to size).
 * wc_job_from_wcj8: a solvable job from WCJ8 bytes (the reference's count
 * checks; a snapshot list other than snapshot_iters(iters) is refused). The
 * job equals the one wc_job_build makes from the same root (wc_job_digest). */
int wc_wcj8_from_root(const uint8_t* root, size_t len, const wc_solve_cfg* cfg, const float* carried,
                      uint32_t ncarried, const uint32_t* net_dims, uint32_t ndims, uint8_t* buf, size_t cap,
                      size_t* out_len);
int wc_job_from_wcj8(const uint8_t* bytes, size_t len, wc_job** out);
/* Work counts for roofline accounting, 20 slots, [p] = player 0 / 1:
 * [0+p] regret-matching cells of p's nodes, [2+p] their rows, [4+p] value-
 * gather entries for traverser p, [6+p] value-gather outputs, [8+p] reach
 * entries through p's decision cells, [10+p] reach entries through p's draws,
 * [12+p] reach outputs of mover p, [14+p] network-row configs of p, [16+p]
 * terminal-leaf configs of p, [18] reach slots, [19] value slots; with n > 20
 * also [20] the distinct public rows among the network rows (the rows the
 * tensor-core board trunk runs on; the others share a row's board pieces). */
int wc_job_counts(const wc_job* job, uint64_t* out, int n);
/* The job's root belief: player 0's then player 1's weights over the root
 * supports (root_nc0 + root_nc1 floats). */
int wc_job_root_belief(const wc_job* job, float* out);
/* Carry layout: nexit + 1 offsets into a carry row, and the exit nodes'
 * reference ids (network rows then terminal leaves). Either may be NULL. */
int wc_job_carry_offsets(const wc_job* job, uint32_t* offsets, uint32_t* exit_nodes);

/* A roots file as write_roots writes it (engine/src/roots.rs:323-363: magic
 * 0x57107207, version 3, u32 count, the roots back to back): the byte offset
 * and length of each root, for wc_job_build. Replaces read_roots. cap bounds
 * offsets / lengths; *n receives the root count. */
int wc_roots_file_split(const uint8_t* file, size_t len, uint64_t* offsets, uint64_t* lengths, size_t cap,
                        size_t* n);

/* ---- rules over encoded states ------------------------------------------- */
/* A State in the reference's write_state encoding (the State part of a root).
 * wc_state_legal_actions replaces State::legal_actions
 * (engine/src/rules.rs:1027-1146): the action codes (Action::encode,
 * engine/src/actions.rs:252-295) in the engine's order, deduplicated; cap
 * bounds codes, *n receives the count. wc_state_apply replaces
 * State::apply (engine/src/rules.rs:1155): the successor state, in the same
 * encoding. With unchecked == 0 an action that is not legal in the state is
 * refused (WC_E_ARG). With unchecked != 0 it is applied as the reference's
 * apply does, without a legality test (its own tests apply hand-picked
 * actions that way, e.g. an attack between non-adjacent hexes): the action
 * must still name in-range fields and a unit on its source hex, else it is
 * refused (where the reference would panic). Every call refuses a state
 * whose fields are out of range (WC_E_ARG).
 * wc_state_query writes 4 values: to_act (state.rs), winner (-1 = none),
 * is_terminal, is_chance. */
int wc_state_legal_actions(const uint8_t* state, size_t len, uint32_t* codes, size_t cap, size_t* n);
int wc_state_apply(const uint8_t* state, size_t len, uint32_t code, int unchecked, uint8_t* out, size_t cap,
                   size_t* out_len);
int wc_state_query(const uint8_t* state, size_t len, int32_t* out);

/* ---- batched solves ------------------------------------------------------ */
/* Synchronous: upload, solve and download n jobs on the context's devices.
 * Jobs go to devices longest-first by the reference router's cost
 * (engine/src/gpu/client.rs:282-291), each to the least-loaded device. On a
 * device they run in memory-bounded waves (at most 44% of the free device
 * memory each, or WC_WAVE_BYTES; at least two above 4 GiB so a wave's tables
 * upload while the previous wave solves), in two device arenas the context
 * keeps across calls. out has n entries, filled with library-owned arrays. */
int wc_solve_batch(wc_ctx* ctx, wc_job* const* jobs, size_t n, wc_result* out);
void wc_result_free(wc_result* r);
/* Device-resident form: upload once, solve any number of times, read back. */
int wc_batch_upload(wc_ctx* ctx, int dev_index, wc_job* const* jobs, size_t n, wc_batch** out);
int wc_batch_solve(wc_batch* b);
/* A solve with CUDA-event timing per kernel class, in milliseconds:
 * [0] per-solve network, [1] leaf evaluation, [2] regret-matching rows,
 * [3] value gathers, [4] reach gathers (+ average), [5] snapshots, [6] Phase 2,
 * [7] init, [8] whole solve; on the tensor-core path also the parts
 * [9] pooling, [10] join, [11] head (of [1]) and [12] trunk (of [0]).
 * class_ms needs 13 entries. */
int wc_batch_solve_profiled(wc_batch* b, double* class_ms, int nclass);
int wc_batch_download(wc_batch* b, size_t job, float* strategy, float* root_values, uint16_t* carries);
/* After a solve: each job's exploitability under its average strategy, from
 * its live root belief (Solver::nash_conv, engine/src/search.rs:1884-1907):
 * nash[j] = sum over players of (best-response value - value under the
 * average), zero_sum[j] = sum of the values under the average (0 for a
 * zero-sum game up to rounding). Both of the depth-limited game the tree
 * defines, with the network valuing its leaves. One float per job each. */
int wc_batch_nash_conv(wc_batch* b, float* nash, float* zero_sum);
/* Leaf evaluation alone (the per-solve network, then every network row's
 * values for traverser p at the initial uniform-strategy reaches), and its
 * read-back: rows in the reference's leaf_rows order, each row's p-configs
 * in support order (counterfactual values: network value x opponent reach).
 * class_ms, if non-NULL, receives the same 13 timing classes as
 * wc_batch_solve_profiled (leaf evaluation alone in [1]). */
int wc_batch_leaf_values(wc_batch* b, int p, double* class_ms);
int wc_batch_download_leaf_values(wc_batch* b, size_t job, int p, float* out);
/* After a solve or wc_batch_leaf_values: one job's board vectors P
 * (net_rows x 256) and join projections jp (net_rows x 128) as the network
 * path stores them; the 16-bit paths store P plus the join output bias, and
 * each row of both minus its mean (every consumer is a LayerNorm input, which
 * ignores a per-row constant). */
int wc_batch_download_board_rows(wc_batch* b, size_t job, float* pb, float* jp);
/* Totals of the batch: node-updates per solve, network-row evaluations per
 * solve, table bytes, device bytes. */
void wc_batch_stats(const wc_batch* b, double* node_updates, double* leaf_evals, uint64_t* table_bytes,
                    uint64_t* device_bytes);
void wc_batch_free(wc_batch* b);
/* Kernel launches of the batch's last solve or leaf evaluation. */
uint64_t wc_batch_launches(const wc_batch* b);

/* ---- diagnostics --------------------------------------------------------- */
/* D[128, n] = A[128, k] * B[n, k]^T (bf16 bit patterns, row-major) through one
 * CTA's tcgen05 path on the current device: the descriptor and swizzle
 * self-test of the tensor-core kernels. k % 64 == 0, n % 16 == 0, n <= 256. */
int wc_debug_umma_gemm(const uint16_t* a, const uint16_t* b, int k, int n, float* d);

/* The time limit of every mbarrier wait in the tensor-core kernels (ns of
 * %globaltimer; 0 restores the default, 2 s). A debug control with no
 * counterpart in the reference: with a limit shorter than the work waited on,
 * the kernels give up, drain what they issued, release their tensor memory
 * and report the failure through the solve's status (WC_E_CUDA, "a
 * tensor-core wait exceeded its time limit (code c)"), and the context stays
 * usable; codes above 10 mean in-flight work did not drain. */
int wc_debug_set_wait_limit(wc_ctx* ctx, uint64_t ns);

/* wc_debug_umma_gemm without any device allocation; it has no counterpart in
 * the reference. For callers that cannot call cudaMalloc: a host engine whose
 * device memory is owned by another allocator (a caching allocator holding
 * the free memory, or an arena fixed at start-up), or a latency-bound caller
 * for whom cudaMalloc / cudaFree would synchronise the device. Same inputs,
 * outputs and kernel; the device copies of a and b, the result and a status
 * word live in one static device array of 327,936 bytes that every GPU
 * loading this library holds until exit, so k <= 256 (n <= 256 as before);
 * larger k is rejected with WC_E_ARG. The call runs on a private
 * non-blocking stream and waits for that stream only (copies from and to
 * pageable host memory). The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress) and creates that stream; make that
 * first call before any stream capture. All calls share the one array: calls
 * that overlap on the GPU (from several host threads, say) race and must be
 * serialised by the caller. */
int wc_debug_umma_gemm_static(const uint16_t* a, const uint16_t* b, int k, int n, float* d);

/* ---- continual re-solving ------------------------------------------------- */
/* A game whose seats both play by solving: at a decision it builds the
 * depth-limited subgame (Solver::new), the caller solves it, and the game
 * then walks the solved tree with the real play (each decision sampled from
 * the CFR average of the true config, both beliefs Bayes-filtered on the
 * public observations and the draws), until the walk leaves the tree at a
 * leaf. The next decision re-solves, and its Phase 2 values the carried
 * beliefs: the exit's beliefs under the solve's per-iterate averages (from
 * the carry store, f16) and the live belief. Replaces the reference's game
 * actor (engine/src/selfplay.rs:466-905: finish_walk, Game::advance,
 * Game::resume; engine/src/gpu/client.rs:20-92 CarryStore::select); as
 * there, a subgame over the node cap falls back to one uniform decision and
 * drops the carried beliefs. Snapshots are always kept. */
typedef struct wc_game wc_game;
enum { WC_GAME_SOLVE = 1, WC_GAME_ENDED = 2 };
/* From a seeded game (make_game, selfplay.rs:59-81) or from a root (root
 * encoding above: the state and both beliefs, e.g. wc_root_generate_wide's
 * belief-heavy roots). `seed` drives the game's own draws and sampling. */
int wc_game_new(uint64_t seed, int random_draft, const wc_solve_cfg* cfg, wc_game** out);
int wc_game_from_root(const uint8_t* root, size_t len, uint64_t seed, const wc_solve_cfg* cfg, wc_game** out);
/* Stop (WC_GAME_ENDED) once n subgames have been solved and the walk of the
 * last has left its tree (0: play to the end of the game). */
int wc_game_set_max_solves(wc_game* g, uint32_t n);
/* Play until the next solve: *step = WC_GAME_SOLVE with *job a new job (the
 * subgame with its carried roots, owned by the caller: solve it, pass its
 * result to wc_game_resume, then free it), or WC_GAME_ENDED with *job NULL. */
int wc_game_advance(wc_game* g, wc_job** job, int* step);
/* Start the walk of the pending subgame with its solve's result. */
int wc_game_resume(wc_game* g, const wc_job* job, const wc_result* res);
/* decisions, solves, capped solves, walk decisions, walk draws, ended,
 * winner (-1: none), walking. */
int wc_game_counters(const wc_game* g, int64_t* out8);
/* The game's current state and beliefs in the root encoding. */
int wc_game_root(const wc_game* g, uint8_t* buf, size_t cap, size_t* len);
void wc_game_free(wc_game* g);

/* ---- training batch ------------------------------------------------------- */
/* The step after solving in the training loop: compact replay rows expanded
 * on the training device into the value network's input for both canonical
 * seat views. Replaces train/gpu_batch.py:119-163 (make_batch's Triton
 * expansion, train/gpu_batch.py:22-117) with the same outputs as the CPU
 * batch (train/train.py:249-270: engine/src/rebel.rs:1353 expand_row of each
 * row and of its mirror, train/mirror.py:60-85).
 *
 * wc_replay_pack_row: the replay row (WC_ROW_BYTES bytes, rebel.rs:935-964)
 * of a state given in the reference's state encoding (write_state), or of
 * the state that starts a root in the root encoding (bytes after the state
 * are not read); the row's rules-table hash is rebel.rs:996's.
 *
 * wc_replay_expand: every pointer is device memory of the current device,
 * and the call only enqueues work on `stream` (a cudaStream_t; NULL is the
 * legacy default stream):
 *   rows  nrows x WC_ROW_BYTES replay rows;
 *   cc    m x 15 config counts (hand[5], face-down[5], bag[5]) of the rows'
 *         belief supports, and seg their span ids 2 row + seat,
 *         non-decreasing, every span non-empty (train/train.py:70-79);
 *   x     out, 2 nrows x WC_PUBFEAT floats: view 2r is row r, view 2r + 1
 *         its mirror, each with its seats' hand / face-down / bag sizes
 *         (the mirror's exchanged);
 *   phi   out, m x 15 floats, cc / 5 (CNORM).
 * The caller checks seg (train.py's np.searchsorted would raise on a span
 * past the end); unit ids past the table expand to zero facts. */
enum { WC_ROW_BYTES = 215, WC_PUBFEAT = 897 };
int wc_replay_pack_row(const uint8_t* state, size_t len, uint8_t* out);
int wc_replay_expand(const uint8_t* rows, size_t nrows, const uint8_t* cc, const int64_t* seg, size_t m, float* x,
                     float* phi, void* stream);

/* ---- streaming submit / wait ---------------------------------------------- */
/* The job stays owned by the caller and must outlive the wc_wait of its
 * ticket; free it (wc_job_free) after that wait returns. */
int wc_submit(wc_ctx* ctx, wc_job* job, uint64_t* ticket);
int wc_wait(wc_ctx* ctx, uint64_t ticket, wc_result* out);
/* Outstanding submitted cells, for routing (GpuClient::queued_work). */
uint64_t wc_queued_work(wc_ctx* ctx);

#ifdef __cplusplus
}
#endif
#endif /* WC_B200_H */
