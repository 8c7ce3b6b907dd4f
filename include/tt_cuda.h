/*
 * tt_cuda.h — C ABI of libtt_cuda.so, the B200 (sm_100a) execution backend for
 * TinyTensor graphs.
 *
 * The reference backend boundary this replaces is the generated-kernel ABI
 *     using KernelEntryFn = int (*)(void** input_ptrs, void** output_ptrs, void** temp_ptrs);
 *     (include/tinytensor/runtime/executable.hpp:14, exported as
 *      tinytensor_kernel_entry by src/codegen/cpp_backend.cpp:55-57)
 * together with the C++ classes that produce and drive it:
 *     CppBackend::generate_code / compile   include/tinytensor/codegen/cpp_backend.hpp:21-33
 *     Executable::run                       src/runtime/executable.cpp:7-63
 *     Executor (mode dispatch, diagnostics) src/runtime/executor.cpp:9-136
 *     MemoryPlanner::compute_plan           src/optimizer/memory_planner.cpp:8-112
 *     KernelCache (SHA-256 key, flock)      src/codegen/kernel_cache.cpp:190-313
 *     Autodiff::compute_gradients           src/autodiff/gradient.cpp:52-332
 *     SGD.step                              python/tinytensor/optim.py:18-35
 *
 * Conventions kept from the reference:
 *  - pointer arrays follow graph-input order and graph-output order
 *    (cpp_backend.cpp:61-66, 81-85);
 *  - the caller owns input and output buffers; the backend writes outputs in place;
 *  - every call returns 0 on success and a nonzero status otherwise; the host maps
 *    statuses to the reference exception types (TT_ERR_SHAPE -> ShapeError, ...),
 *    and tt_last_error() holds the message (thread-local).
 *
 * No PyTorch or CUDA types appear in the signatures: streams are passed as void*
 * (a cudaStream_t, NULL = legacy default stream).
 */
#ifndef TT_CUDA_H
#define TT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (reference exception hierarchy, include/tinytensor/utils/errors.hpp:8-66) ---- */
enum tt_status {
    TT_OK = 0,
    TT_ERR_SHAPE = 1,         /* ShapeError */
    TT_ERR_DIMENSION = 2,     /* DimensionError */
    TT_ERR_BROADCAST = 3,     /* BroadcastError */
    TT_ERR_TYPE = 4,          /* TypeError */
    TT_ERR_MEMORY = 5,        /* MemoryError: device/host allocation failed */
    TT_ERR_IR = 6,            /* IRError: the graph failed verification */
    TT_ERR_COMPILE = 7,       /* CompileError: NVRTC failure, unsupported op or dtype */
    TT_ERR_RUNTIME = 8,       /* RuntimeExecutionError: arity, CUDA launch/copy error */
    TT_ERR_DEVICE_STATUS = 9, /* a kernel gave up a bounded wait and set the status word */
    TT_ERR_NO_DEVICE = 10,    /* no usable sm_100 GPU */
    TT_ERR_INVALID = 11,      /* null handle or bad argument */
    TT_ERR_COMM = 12          /* NCCL failure */
};

/* ---- op codes: the reference OpType order (include/tinytensor/ir/operation.hpp:7-22),
 *      then the ops this backend adds ---- */
enum tt_op {
    TT_OP_INPUT = 0,
    TT_OP_CONSTANT = 1,
    TT_OP_ADD = 2,
    TT_OP_SUB = 3,
    TT_OP_MUL = 4,
    TT_OP_DIV = 5,
    TT_OP_RELU = 6,
    TT_OP_SIGMOID = 7,
    TT_OP_MATMUL = 8,
    TT_OP_TRANSPOSE = 9,
    TT_OP_REDUCE_SUM = 10,
    TT_OP_REDUCE_MEAN = 11,
    TT_OP_OUTPUT = 12,            /* never appears as a node (outputs are marked) */
    TT_OP_FUSED_ELEMENTWISE = 13, /* reference fusion node; expr = "relu(op(@0, @1))" */
    /* additions (no reference OpType) */
    TT_OP_EXP = 14,
    TT_OP_NEG = 15,
    TT_OP_TANH = 16,
    TT_OP_REDUCE_MAX = 17,
    TT_OP_STEP = 18,    /* x > 0 ? 1 : 0, the ReLU derivative mask (gradient.cpp:200-222) */
    TT_OP_RESHAPE = 19, /* row-major reshape (a view) */
    TT_OP_EXPAND = 20   /* broadcast_to the node's shape (a view) */
};

enum tt_dtype { TT_FLOAT32 = 0, TT_FLOAT64 = 1 }; /* include/tinytensor/core/dtype.hpp:10-13 */

#define TT_MAX_RANK 8
#define TT_MAX_NODE_INPUTS 2

/* One graph node, the C image of tinytensor::Node (include/tinytensor/graph/node.hpp). */
typedef struct tt_node {
    int32_t op;                         /* enum tt_op */
    int32_t dtype;                      /* enum tt_dtype */
    int32_t num_inputs;
    int32_t inputs[TT_MAX_NODE_INPUTS]; /* indices of EARLIER entries of tt_graph.nodes */
    int32_t rank;
    int64_t shape[TT_MAX_RANK];
    int64_t id;                         /* the reference node id, printed as %id in IR text */
    int64_t dim0, dim1;                 /* Transpose */
    int32_t num_axes;                   /* Reduce*: 0 = all axes */
    int32_t keepdims;
    int64_t axes[TT_MAX_RANK];
    const void* data;                   /* Constant: numel*itemsize bytes, row-major (copied) */
    const char* name;                   /* Input name, may be NULL */
    const char* expr;                   /* FusedElementwise expression, may be NULL */
} tt_node;

typedef struct tt_graph {
    int32_t num_nodes;
    const tt_node* nodes;      /* topologically ordered: inputs[] refer to earlier nodes */
    int32_t num_inputs;
    const int32_t* inputs;     /* node indices, graph-input order (Graph::inputs()) */
    int32_t num_outputs;
    const int32_t* outputs;    /* node indices, graph-output order (Graph::outputs()) */
} tt_graph;

typedef struct tt_compile_options {
    int32_t optimize;          /* run the backend's CSE + DCE before scheduling */
    int32_t device;            /* CUDA device ordinal */
    const char* cache_dir;     /* kernel cache directory; NULL or "" = no disk cache */
    int32_t grad_loss;         /* -1, or the node index of a loss to differentiate */
    int32_t num_grad_wrt;      /* with grad_loss: gradients of loss w.r.t. these nodes are */
    const int32_t* grad_wrt;   /*   appended to the program outputs, in this order */
    int32_t flags;             /* TT_FLAG_* */
} tt_compile_options;

#define TT_FLAG_NO_FUSION 1       /* one kernel per elementwise node (diagnostics) */
#define TT_FLAG_NO_GEMM_FUSION 2  /* no GEMM-adjacent fusion (diagnostics): activations stay separate
                                   * passes, every tensor-core GEMM splits its own operands, small-K
                                   * products are GEMM launches */
#define TT_FLAG_HOST_ONLY 4       /* plan + generate + NVRTC-compile only: no device, no arena
                                     (tt_program_info works; tt_program_run reports no device) */
#define TT_FLAG_SERIAL 8          /* every launch on the run's stream, one after another (by
                                     default two adjacent independent GEMMs run side by side
                                     on a second stream of the program) */

typedef struct tt_program tt_program;

/* where buffers passed to tt_program_run live */
enum tt_where { TT_HOST = 0, TT_DEVICE = 1 };

/* what tt_program_info returns */
enum tt_info {
    TT_INFO_ORIGINAL_IR = 0,  /* Executor::original_ir  (executor.cpp:12) */
    TT_INFO_OPTIMIZED_IR = 1, /* Executor::optimized_ir (executor.cpp:24) */
    TT_INFO_SOURCE = 2,       /* Executor::generated_source: the CUDA translation unit */
    TT_INFO_PLAN = 3,         /* Executor::execution_plan (executor.cpp:62-98) + arena map */
    TT_INFO_CUBIN_PATH = 4    /* cached cubin path ("" without a cache) */
};

/* ---- library / device ---- */
const char* tt_last_error(void);
int tt_version(void); /* 10000*major + 100*minor + patch */
/* Selects `device`, checks it is an sm_100 part and creates the primary context. */
int tt_device_init(int32_t device);
/* Number of kernels this library launched since load (all programs, all helpers). */
uint64_t tt_launch_count(void);

/* ---- graph utilities (no GPU needed) ---- */
/* Canonical IR text of a graph in the reference IRPrinter format (src/ir/printer.cpp:6-62).
 * Writes at most cap bytes (NUL-terminated) and sets *needed to the full size + 1. */
int tt_graph_ir(const tt_graph* g, char* buf, size_t cap, size_t* needed);
/* Verifies a graph (src/ir/verifier.cpp:7-202 rules); 0 or TT_ERR_IR/… with a message. */
int tt_graph_verify(const tt_graph* g);

/* ---- compile / run: CppBackend::compile + Executable::run ---- */
int tt_compile(const tt_graph* g, const tt_compile_options* opt, tt_program** out);
int tt_program_info(const tt_program* p, int32_t what, char* buf, size_t cap, size_t* needed);
int tt_program_num_io(const tt_program* p, int32_t* num_inputs, int32_t* num_outputs);
int tt_program_output_shape(const tt_program* p, int32_t index, int32_t* rank, int64_t* shape);
/* Runs once.  TT_HOST: inputs/outputs are host pointers; the call copies inputs in,
 * runs, copies outputs out and synchronises (Executable::run semantics).
 * TT_DEVICE: device pointers; the work is queued on `stream` and the call returns
 * without synchronising (check tt_program_status after a sync). */
int tt_program_run(tt_program* p, const void* const* inputs, void* const* outputs, int32_t where,
                   void* stream);
/* Synchronises the program's last stream and reads its device status word
 * (0 = fine; nonzero = a bounded wait gave up).  Returns TT_ERR_DEVICE_STATUS then. */
int tt_program_status(tt_program* p, int32_t* device_status);
/* Per-launch profiling (Profiler::record_node for compiled mode): when enabled, each
 * run records CUDA events around every launch on the run's stream; enabling resets the
 * sums.  A profiled run waits for the previous profiled run's events before queueing. */
int tt_program_set_profiling(tt_program* p, int32_t enable);
/* Average per-launch device time over the profiled runs: up to cap entries of
 * (label, ms).  names is an array of cap buffers of name_cap bytes each. */
int tt_program_profile(const tt_program* p, int32_t cap, char* names, int32_t name_cap, float* ms,
                       int32_t* count);
int tt_program_destroy(tt_program* p);
/* Output-ready events (no counterpart in the reference, whose Executable::run is
 * synchronous and single-stream).  events[k] (a tt_event_create handle, or NULL) is
 * recorded on the run's stream as soon as output k is complete, so another stream can
 * start work on it — e.g. the data-parallel all-reduce of one weight gradient — while
 * the rest of the program still runs.  n <= number of outputs; n = 0 clears.  The
 * program keeps the handles; the caller keeps them alive while it runs. */
int tt_program_set_output_events(tt_program* p, void* const* events, int32_t n);
/* Index of the launch after which output `output` is complete (-1: before the first),
 * i.e. the order in which the output events fire. */
int tt_program_output_step(tt_program* p, int32_t output, int32_t* step);
/* Input-released events (no counterpart in the reference: its inputs are host tensors
 * copied per call).  events[k] (a tt_event_create handle, or NULL) is recorded on the
 * run's stream as soon as the last launch reading input k is complete, so the caller
 * may overwrite that device buffer from another stream — e.g. the SGD update of a
 * parameter whose gradient is already exchanged — while the rest of the program still
 * runs.  n <= number of inputs; n = 0 clears.  The caller keeps the handles alive. */
int tt_program_set_input_events(tt_program* p, void* const* events, int32_t n);
/* Index of the launch after which input `input` is no longer read (-1: never read). */
int tt_program_input_step(tt_program* p, int32_t input, int32_t* step);

/* ---- buffers (plain cudaMalloc / cudaMallocHost / cudaMemcpyAsync) ---- */
enum tt_copy { TT_H2D = 1, TT_D2H = 2, TT_D2D = 3 };
int tt_device_alloc(size_t bytes, void** ptr);
int tt_device_free(void* ptr);
int tt_host_alloc(size_t bytes, void** ptr); /* pinned */
int tt_host_free(void* ptr);
int tt_memcpy(void* dst, const void* src, size_t bytes, int32_t kind, void* stream);
int tt_stream_create(void** stream);
int tt_stream_destroy(void* stream);
int tt_stream_sync(void* stream);
/* Events for cross-stream ordering (cudaEventCreateWithFlags(DisableTiming) /
 * cudaEventRecord / cudaStreamWaitEvent); no counterpart in the reference. */
int tt_event_create(void** event);
int tt_event_destroy(void* event);
int tt_event_record(void* event, void* stream);
int tt_stream_wait_event(void* stream, void* event);
/* CUDA graphs of queued work (no counterpart in the reference): everything queued on
 * `stream` between begin and end — program runs in TT_DEVICE mode, SGD steps,
 * all-reduces, and work on other streams joined through events — becomes one graph
 * that tt_graph_launch replays with the same buffers.  For launch-bound loops (small
 * programs called many times, a whole training step). */
int tt_stream_begin_capture(void* stream);
int tt_stream_end_capture(void* stream, void** graph_exec);
int tt_graph_launch(void* graph_exec, void* stream);
int tt_graph_destroy(void* graph_exec);

/* ---- diagnostics (no counterpart in the reference) ----
 * Runs one CTA that waits on an mbarrier nothing arrives at, through the same bounded
 * wait every tensor-core GEMM wait uses, with a budget of `budget_cycles` SM clock
 * cycles (at most 4e9), then synchronises.  *status_out receives the code the wait
 * records on giving up (0x200 = a timed-out data wait); the context stays usable.  Shows
 * that a missing arrival ends in a status the host reads, not in a hang. */
int tt_selftest_bounded_wait(int64_t budget_cycles, int32_t* status_out);

/* ---- optimiser: SGD.step (python/tinytensor/optim.py:18-35) on device ----
 * For each i: v = momentum*v + g (when momentum > 0, velocities[i] != NULL);
 * p -= lr * (momentum > 0 ? v : g).  One fused launch over all parameters. */
int tt_sgd_step(int32_t n, float* const* params, const float* const* grads, float* const* velocities,
                const int64_t* numels, float lr, float momentum, void* stream);

/* ---- fp32-accurate GEMM that allocates nothing (no counterpart in the reference) ----
 * C[M,N] = A[M,K] . B[K,N], row-major contiguous float32 device arrays, queued on
 * `stream`, same kernels and accuracy as a compiled matmul.  For callers that cannot
 * call cudaMalloc: its scratch is a static device array of 32 MiB per GPU that loads
 * the library (held until exit); products needing more are rejected with
 * TT_ERR_MEMORY.  The first call on a device resolves the array's address
 * (cudaGetSymbolAddress); under lazy module loading that also loads the module and
 * reserves the array, and the kernels load on their first launch, so make the first
 * call on each device a warm-up outside any no-allocation window and before any
 * stream capture.  All calls share the array: calls that overlap on the GPU race, so
 * order them on one stream.  A, B may be NULL when they hold no elements (K = 0).
 * device_status: optional zeroed device int that the kernels set if a bounded wait
 * gives up; check it after synchronising.  With NULL an internal word takes the code
 * and such a timeout is NOT reported (the call still returns TT_OK, C partly written). */
int tt_gemm_f32_noalloc(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                        int32_t* device_status, void* stream);

/* ---- data parallel: NCCL over NVLink (no reference counterpart) ---- */
typedef struct tt_dp tt_dp;
#define TT_DP_ID_BYTES 128
int tt_dp_unique_id(char* id_out /* TT_DP_ID_BYTES */);
int tt_dp_init(int32_t rank, int32_t world, const char* id /* TT_DP_ID_BYTES */, int32_t device,
               tt_dp** out);
/* In-place sum all-reduce of `count` floats on `stream`; scale (e.g. 1/world) is
 * applied by the caller's SGD step, so replicas stay bit-identical. */
int tt_dp_allreduce_sum(tt_dp* dp, float* buf, size_t count, void* stream);
int tt_dp_destroy(tt_dp* dp);

#ifdef __cplusplus
}
#endif

#endif /* TT_CUDA_H */
