// Launch schedule and arena plan of a compiled program.
#pragma once

#include <string>
#include <vector>

#include "program.hpp"

namespace ttb {

enum StoreKind { SK_REG = 0, SK_IMM = 1, SK_BUF = 2 };

// How a node's value can be read once computed.
struct Storage {
    int kind = SK_REG;
    float imm = 0.f;
    int root = -1;                  // node owning the buffer (SK_BUF)
    int64_t offset = 0;             // element offset into the root buffer
    std::vector<int64_t> strides;   // element strides per dim of the node's shape
};

struct Plan {
    Graph g;                        // the scheduled graph
    std::vector<Storage> st;        // per node
    std::vector<int> region_of;     // per node, -1 if none
    std::vector<Region> regions;
    std::vector<Launch> launches;   // in execution order
    std::vector<BufRef> root_ref;   // per node: where its buffer lives (roots only)
    // arena layout (bytes)
    int64_t const_bytes = 0, slot_bytes = 0, stage_in_offset = 0, stage_out_offset = 0;
    int64_t status_offset = 0, arena_bytes = 0;
    std::vector<int64_t> stage_in, stage_out;       // staging offsets per input / output
    std::vector<std::pair<int64_t, int>> constants; // (arena offset, node) to upload
    std::vector<Slot> slots;
    // MemoryPlanner-style report (src/optimizer/memory_planner.cpp:100-109)
    int64_t total_alloc_bytes = 0, peak_planned_bytes = 0, theoretical_peak_bytes = 0;
    size_t reused_buffers = 0, num_intermediates = 0;
    size_t fused_regions = 0;
    // per graph output: index of the launch after which it is complete (-1: written by
    // no launch, complete when the program starts)
    std::vector<int> output_step;
    std::vector<int> input_last_step;  // per graph input: the last launch reading it (-1: none)
};

struct ScheduleOptions {
    bool fuse = true;
    bool gemm_epilogue = true;
    bool concurrent_gemms = true;
};

Plan schedule(const Graph& g, const ScheduleOptions& opt);
std::string generate_source(Plan& p);         // CUDA translation unit for all regions (sets vec/grid)
std::string plan_text(const Plan& p);         // arena map + launch list

}  // namespace ttb
