// TEST INFRASTRUCTURE — the CPU oracle. Only tests/, __graft_entry__.smoke()
// and bench.py's CPU-baseline leg use anything under oracle/.
//
// The reference's single-threaded subgame solver (engine/src/search.rs:724-
// 1986) over a tree built by the host builder: uniform initial strategy,
// reach propagation (search.rs:1273-1351), leaf evaluation through the CPU
// value network (search.rs:1464-1636), the fused regret backprop with regret
// matching (search.rs:1654-1803), the average-strategy accumulation and the
// log-spaced snapshots (search.rs:882-940, 1805-1841), and Phase 2:
// value_under, nash_conv, carried_beliefs (search.rs:1851-1957).
#pragma once
#include <vector>

#include "../war-chest-bot-9000-_b200/csrc/host/tree.h"
#include "net_cpu.h"

namespace oracle {

enum class Back { Regret, Value, BestResponse };

struct Solver {
    const wc::Tree& t;
    const Net* net;  // nullptr or empty: every network row is valued 0
    std::vector<float> regret, cur, sum;
    std::vector<uint32_t> roff, voff;
    std::vector<float> reach, vals;
    std::vector<std::vector<float>> snaps;
    std::vector<int> snap_list;
    int snap_t = 0;
    bool avg_touched[2] = {false, false};
    int steps[2] = {0, 0};
    int last_traverser = -1;
    // leaf batch
    bool batch_ready = false;
    std::vector<float> cards, pb, jp, cf, cg, xb, h;

    Solver(const wc::Tree& tree, const Net* n);
    bool net_ready() const { return net && !net->empty; }

    void multistep(int iters);
    void step(int traverser);
    void propagate(const std::vector<float>& strat, const float* root0, const float* root1);
    void precompute_reaches();
    void backprop(int traverser, const std::vector<float>* strat, Back mode);
    void leaf_values(int traverser);
    void avg_block(int traverser);
    void snapshot();
    std::vector<std::vector<float>> value_under(const std::vector<std::vector<float>>& roots /*pairs: [p0, p1]*/);
    void nash_conv(float* nash, float* zero_sum);
    std::vector<std::vector<float>> carried_beliefs(uint32_t leaf);  // per snapshot: p0 then p1
    const std::vector<float>& average() const { return snaps.back(); }

    void ensure_leaf_batch();
    void belief_blocks(int only);
    void pbs_head(int traverser);
    void readout(int p);
    const float* reach_of(uint32_t i, int p) const;
    float* reach_of(uint32_t i, int p);
};

}  // namespace oracle
