// Compiled-program structures of the B200 backend: the launch schedule, the
// arena layout produced by the memory planner, and the descriptors of the
// hand-written kernels (reductions, GEMM, SGD) that the schedule calls.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "ttb.hpp"

namespace ttb {

// Where a kernel argument points: arena offset, or a caller buffer (+ offset).
enum BufKind { BK_NONE = 0, BK_ARENA = 1, BK_INPUT = 2, BK_OUTPUT = 3 };
struct BufRef {
    int kind = BK_NONE;
    int index = 0;          // input/output position
    int64_t offset = 0;     // bytes
};

// ---- reductions (kernels_reduce.cu) ----
enum ReduceKind { RK_ROW = 0, RK_COL = 1, RK_GENERIC = 2 };
enum ReduceOp { RO_SUM = 0, RO_MEAN = 1, RO_MAX = 2 };
struct ReduceDesc {
    int op = RO_SUM;
    int kind = RK_ROW;
    // ROW: out[o] = red_{r<R} x[o*s_outer + r*s_red]            (s_red == 1 when vec)
    // COL: out[o] = red_{r<R} x[r*s_red + o]                     (o contiguous)
    int64_t outer = 1, R = 1, s_outer = 0, s_red = 1;
    int splits = 1;          // partial sums per output (scratch = outer*splits doubles)
    int vec = 1;             // 4 when rows/columns can use float4 loads
    float mean_scale = 1.f;  // float(1/count) for mean
    // GENERIC: kept/reduced dims with element strides; output contiguous over kept dims
    int nk = 0, nr = 0;
    int64_t ksize[TT_MAX_RANK], kstride[TT_MAX_RANK], rsize[TT_MAX_RANK], rstride[TT_MAX_RANK];
    int64_t in_offset = 0;   // element offset of the view
};
// Fixes the split count / vector width of d and returns the scratch bytes its
// launch needs (double partials).  Launchers return cudaError_t as int.
int64_t reduce_prepare(ReduceDesc& d);
int launch_reduce(const ReduceDesc& d, const float* in, float* out, void* scratch, void* stream);

// ---- GEMM (kernels_gemm.cu) ----
enum Epilogue { EP_NONE = 0, EP_RELU = 1, EP_TANH = 2 };
#ifdef __CUDACC__
// The activation a GEMM applies to each output element in its epilogue: the same
// expressions as the generated elementwise kernels (ReLU as x > 0 ? x : 0, so NaN and
// -0 give +0; tanh as tanhf).
__device__ __forceinline__ float gemm_epilogue(float v, int ep) {
    return ep == EP_RELU ? (v > 0.0f ? v : 0.0f) : ep == EP_TANH ? tanhf(v) : v;
}
#endif
struct GemmDesc {
    int64_t M = 0, N = 0, K = 0, batch = 1;
    int64_t a_sm = 0, a_sk = 0, a_sb = 0;  // A[b][m][k] element strides
    int64_t b_sk = 0, b_sn = 0, b_sb = 0;  // B[b][k][n]
    int64_t c_sb = 0;                      // C[b][m][n] row stride N
    int64_t a_off = 0, b_off = 0;          // element offsets of the operand views
    int epilogue = EP_NONE;                // activation applied to C (a ReLU / tanh folded into the GEMM)
    int algo = 0;                          // chosen by plan_gemm
    int ksplit = 1;                        // tensor-core kernel: K split across CTAs
    int chunk_kb = 8;                      // tensor-core kernel: K blocks per TMEM chunk
    int bk = 32;                           // tensor-core kernel: K per pipeline stage (16 or 32)
    int pair = 0;                          // tensor-core kernel: 2-CTA (cta_group::2) 256x256 tiles
    // Pair kernel, ksplit 1: the last `tail_tiles` tiles (those of a last, part-filled round
    // of clusters) are split along K in `tail_split` pieces, one per cluster; the pieces go
    // to partial tiles that a reduce adds in piece order.  0 = no tail split.
    int tail_tiles = 0, tail_split = 0;
    // Tensor-core kernel only: operands whose hi/lo copies the elementwise region that
    // produced them already wrote (no pre-pass for them here).
    int a_presplit = 0, b_presplit = 0;
};
// Device pointers of pre-split operands' hi/lo copies (compact K-major, rows padded to
// round4(K) floats), null for operands split by the GEMM's own pre-pass.
struct GemmSplitIO {
    const float* a_hi = nullptr;
    const float* a_lo = nullptr;
    const float* b_hi = nullptr;
    const float* b_lo = nullptr;
};
// Hi/lo operand copies of a row-major [R][C] matrix, one buffer: layout 0 = its own
// layout [R][round4(C)] (hi, then lo), layout 1 = transposed [C][round4(R)] (hi, lo).
// A GEMM reading the matrix along its rows (A = X or B = X^T) uses layout 0, one
// reading it across (A = X^T or B = X) layout 1.
int64_t split_copies_bytes(int64_t R, int64_t C, bool rows, bool t);
int64_t split_copies_offset(int64_t R, int64_t C, bool rows, int layout, int lo);
void plan_gemm(GemmDesc& d);  // picks the kernel variant for the shape/layout
const char* gemm_algo_name(int algo);
int64_t gemm_scratch_bytes(const GemmDesc& d);  // device scratch the chosen variant needs
int gemm_launch_count(const GemmDesc& d);        // kernels one launch_gemm issues
int64_t gemm_tc_ctas(const GemmDesc& d);         // CTAs of a tensor-core GEMM's main kernel (0 otherwise)
int launch_gemm(const GemmDesc& d, const float* A, const float* B, float* C, void* scratch, int* status,
                void* stream, const GemmSplitIO* io = nullptr);
// Sums split-K partials P[b][s][0..per) in split order into C[b*c_sb + i] and applies
// the epilogue (deterministic).
int launch_splitk_reduce(const float* P, float* C, int64_t per, int ksplit, int64_t batch, int64_t c_sb, int epilogue,
                         void* stream);

// Diagnostic: one CTA waits on an mbarrier nothing arrives at, with the GEMM kernels'
// bounded wait and the given clock budget; the wait records its timeout code in *status.
int launch_bounded_wait_selftest(int* status, long long budget, void* stream);

// ---- misc kernels (kernels_misc.cu) ----
int launch_sgd(int n, float* const* params, const float* const* grads, float* const* vel, const int64_t* numels,
               float lr, float momentum, void* stream);
int launch_fill_f32(float* p, int64_t n, float v, void* stream);

// ---- elementwise regions (generated, NVRTC) ----
struct Access {
    bool imm = false;
    float value = 0.f;                  // immediate scalar constant
    int node = -1;                      // graph node whose storage is read
    int64_t offset = 0;                 // element offset into that storage
    std::vector<int64_t> strides;       // element strides per dim of the READ shape
    // Operand of a small-K matmul evaluated in the region (node `mm`): role 1 = A (varies
    // with the row, strides {row, 0}), role 2 = B (varies with the column, {0, column});
    // the K index steps by kstride, kcount values.  role 0: a plain elementwise read.
    int role = 0, mm = -1;
    int64_t kstride = 0, kcount = 0;
};

struct Region {
    Shape shape;                        // iteration shape
    std::vector<int> nodes;             // nodes computed in registers, topological
    std::vector<int> ext;               // external nodes read (order of kernel params)
    std::vector<Access> ext_access;     // how each ext node is read, strides per `shape` dim
    std::vector<int> stores;            // nodes written (contiguous over `shape`)
    std::vector<BufRef> store_ref;      // filled by the planner
    bool is_copy = false;               // materialise ext[0] into stores[0]
    std::string kernel;                 // generated kernel name
    int vec = 1, unroll = 4;
    int64_t grid = 0;
    // Hi/lo operand copies of stores[copy_store] (an [copy_R][copy_C] matrix) for later
    // tensor-core GEMMs, set by the scheduler; the kernel is then the tiled variant.
    int copy_store = -1;
    bool copy_rows = false, copy_t = false;
    bool drop_f32 = false;              // that store has no other reader: its fp32 value is not written
    int64_t copy_R = 0, copy_C = 0;
};

enum LaunchType { LT_REGION = 0, LT_REDUCE = 1, LT_GEMM = 2 };

struct Launch {
    int type = LT_REGION;
    int region = -1;                    // LT_REGION
    ReduceDesc rd;                      // LT_REDUCE
    GemmDesc gd;                        // LT_GEMM
    int in_node = -1, in_node2 = -1;    // reduce input / gemm A,B (storage nodes)
    int out_node = -1;                  // reduce / gemm output node
    BufRef in_ref, in_ref2, out_ref, scratch_ref;
    int64_t scratch_bytes = 0;
    std::string label;                  // for profiles and the execution plan
    bool concurrent_next = false;       // this GEMM and the next launch (a GEMM) run side by side
    BufRef split_ref;                   // region: its hi/lo operand copies (split_copies_bytes)
    // GEMM: for a pre-split operand, the region launch that wrote its copies and the layout read
    int a_split_src = -1, a_split_layout = 0;
    int b_split_src = -1, b_split_layout = 0;
};

struct Slot {
    int64_t offset = 0, capacity = 0;
    int last_step = -1;
};

}  // namespace ttb
