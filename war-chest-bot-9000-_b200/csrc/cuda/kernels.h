// Kernel launchers, called by the runtime.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "../host/netlayout.h"
#include "device.h"

namespace wcdev {

enum StratSel { STRAT_CUR = 0, STRAT_SNAP = 1 };
enum BackMode { BACK_REGRET = 0, BACK_VALUE = 1, BACK_BEST = 2 };

// cfr_kernels.cu
void launch_init_rows(const JobDev* jobs, const WorkItem* items, uint32_t n, cudaStream_t s);
// leaf_col of every job from its uploaded leaf_cidx and cfg_col (at upload)
void launch_leaf_col(const JobDev* jobs, uint32_t njobs, cudaStream_t s);
void launch_rows(const JobDev* jobs, const WorkItem* items, uint32_t n, int p, int mode, int strat_sel, float da,
                 float db, float predict, cudaStream_t s);
void launch_vgather(const JobDev* jobs, const WorkItem* items, uint32_t n, int p, cudaStream_t s);
void launch_rgather(const JobDev* jobs, const WorkItem* items, uint32_t n, int strat_sel, int which_reach,
                    int sum_update, float dg, cudaStream_t s);
void launch_terminal(const JobDev* jobs, const WorkItem* items, uint32_t n, int p, cudaStream_t s);
void launch_netrows_zero(const JobDev* jobs, const WorkItem* items, uint32_t n, int p, cudaStream_t s);
void launch_seed_root(const JobDev* jobs, uint32_t njobs, int which_reach, int carried_index, cudaStream_t s);
void launch_snapshot(const JobDev* jobs, const WorkItem* items, uint32_t n, int t0, int t1, cudaStream_t s);
void launch_copy_cur_to_snap(const JobDev* jobs, const WorkItem* items, uint32_t n, cudaStream_t s);
void launch_unsort(const JobDev* jobs, const WorkItem* items, uint32_t n, cudaStream_t s);
void launch_collect_root(const JobDev* jobs, uint32_t njobs, int root_index, int p, cudaStream_t s);
void launch_carry(const JobDev* jobs, const WorkItem* items, uint32_t n, int snap_index, cudaStream_t s);
void launch_collect_conv(const JobDev* jobs, uint32_t njobs, int slot, int p, cudaStream_t s);

// net_precise.cu
void net_set_constants(const wc::NetLayout& L, const uint8_t* neighbors, const uint8_t* is_location);
void launch_cards(const JobDev* jobs, uint32_t njobs, const float* W, const float* B, cudaStream_t s);
void launch_trunk(const JobDev* jobs, const uint32_t* row_job, const uint32_t* row_local, uint32_t nrows,
                  const float* W, const float* B, const float* LN, cudaStream_t s);
void launch_configs(const JobDev* jobs, const uint32_t* cfg_job, const uint32_t* cfg_local, uint32_t ncfg,
                    const float* W, const float* B, const float* LN, cudaStream_t s);
void launch_pool(const JobDev* jobs, const uint32_t* row_job, const uint32_t* row_local, uint32_t nrows, int mask,
                 cudaStream_t s);
void launch_join_readout(const JobDev* jobs, const uint32_t* row_job, const uint32_t* row_local, uint32_t nrows,
                         int p, const float* W, const float* B, const float* LN, cudaStream_t s);

// net_fast.cu
// Raise a kernel's dynamic shared-memory limit on the current device, once
// per (device, kernel); false if the driver refuses (the launch is skipped
// and the runtime's launch check reports it).
bool raise_smem_limit(const void* fn, size_t smem);
int umma_selftest(const uint16_t* A, const uint16_t* B, int K, int N, float* D);
// The same with device staging in a static array (no allocation): 0 ok,
// 1 bad shape, 2 CUDA error, 3 tcgen05 wait timed out, 4 k beyond 256,
// 5 the array's device address could not be looked up.
int umma_selftest_static(const uint16_t* A, const uint16_t* B, int K, int N, float* D);
void launch_pool_fast(const JobDev* jobs, const void* tiles, uint32_t ntiles, int mask, uint16_t* pool_img, float* mass,
                      bool half, int* err, uint64_t wait_ns, cudaStream_t s);
void launch_join_fast(const JobDev* jobs, const void* tiles, uint32_t ntiles, const FastNetDev& fn, int p,
                      const uint16_t* pool_img, const uint16_t* jp, uint16_t* zout_img, int* err, cudaStream_t s);
void launch_head_fast(const JobDev* jobs, const void* tiles, uint32_t ntiles, const FastNetDev& fn, int p,
                      const uint16_t* zout, const uint16_t* pb, const float* mass, int* err, cudaStream_t s);
void launch_pack_f16(const JobDev* jobs, const uint32_t* cfg_job, const uint32_t* cfg_local, uint32_t total_cfgs,
                     bool half, cudaStream_t s);
// trunk_fast.cu
void trunk_set_constants(const wc::NetLayout& L, const uint8_t* neighbors, const uint8_t* is_location);
size_t trunk_tiles_bytes();
void launch_tokproj(const JobDev* jobs, uint32_t njobs, const float* W, cudaStream_t s);
// The rows (row_job[i], row_local[i]) may be any subset of the batch's
// network rows: each writes its own P tile-image row and jp row.
void launch_trunk_fast(const JobDev* jobs, const uint32_t* row_job, const uint32_t* row_local, uint32_t total_rows,
                       const uint8_t* tiles, const float* W, const float* B, const float* LN, const FastNetDev& fn,
                       uint16_t* g_pb, uint16_t* g_jp, int* err, cudaStream_t s);
// dup: n triples (job, row, representative row): P and jp of the row copied
// from the representative's, after launch_trunk_fast computed it.
void launch_board_dup(const JobDev* jobs, const uint32_t* dup, uint32_t n, uint16_t* g_pb, uint16_t* g_jp,
                      cudaStream_t s);

// replay.cu: the training batch (all pointers device memory). Uploads the
// card-fact, location and mirror tables to the current device once; false if
// that fails.
bool replay_tables_ready();
// rows: nrows x ROW_BYTES; cc: m x CCOUNTS config counts; seg: m span ids
// (2 row + seat, non-decreasing); x: 2 nrows x PUBFEAT; phi: m x CCOUNTS.
void launch_replay_expand(const uint8_t* rows, uint32_t nrows, const uint8_t* cc, const int64_t* seg, uint64_t m,
                          float* x, float* phi, cudaStream_t s);

}  // namespace wcdev
