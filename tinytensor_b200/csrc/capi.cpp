// The C ABI of include/tt_cuda.h: compile (CppBackend::compile), run
// (Executable::run), diagnostics (Executor::original_ir / optimized_ir /
// generated_source / execution_plan), buffers and the SGD step.
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>
#include <memory>
#include <mutex>
#include <sstream>

#include "jit.hpp"
#include "schedule.hpp"

using namespace ttb;

namespace {

thread_local std::string g_last_error;
thread_local std::string g_last_message;  // g_last_error without the exception-name prefix
std::atomic<uint64_t> g_launches{0};

int set_error(int status, const std::string& msg) {
    static const char* names[] = {"",
                                  "ShapeError: ",
                                  "DimensionError: ",
                                  "BroadcastError: ",
                                  "TypeError: ",
                                  "MemoryError: ",
                                  "IRError: ",
                                  "CompileError: ",
                                  "RuntimeExecutionError: ",
                                  "RuntimeExecutionError: device status: ",
                                  "RuntimeExecutionError: no device: ",
                                  "InvalidArgument: ",
                                  "CommError: "};
    g_last_message = msg;
    g_last_error = (status > 0 && status <= 12 ? names[status] : "") + msg;
    return status;
}

template <typename F>
int guarded(F&& f) {
    try {
        f();
        return TT_OK;
    } catch (const Error& e) {
        return set_error(e.status, e.what());
    } catch (const std::bad_alloc&) {
        return set_error(TT_ERR_MEMORY, "host allocation failed");
    } catch (const std::exception& e) {
        return set_error(TT_ERR_RUNTIME, e.what());
    }
}

void check_cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return;
    int st = (e == cudaErrorMemoryAllocation) ? TT_ERR_MEMORY : TT_ERR_RUNTIME;
    cudaGetLastError();
    fail(st, std::string(what) + ": " + cudaGetErrorString(e));
}

std::string tuple_str(const Shape& s) {  // Shape::to_string (include/tinytensor/core/shape.hpp:63-74)
    std::string r = "(";
    for (size_t i = 0; i < s.size(); ++i) {
        r += std::to_string(s[i]);
        if (i + 1 < s.size() || s.size() == 1) {
            r += ",";
            if (i + 1 < s.size()) r += " ";
        }
    }
    return r + ")";
}

void copy_out(const std::string& s, char* buf, size_t cap, size_t* needed) {
    if (needed) *needed = s.size() + 1;
    if (buf && cap) {
        size_t n = std::min(cap - 1, s.size());
        std::memcpy(buf, s.data(), n);
        buf[n] = '\0';
    }
}

}  // namespace

int ttb::record_error(int status, const std::string& msg) { return set_error(status, msg); }

struct tt_program {
    int device = 0;
    Plan plan;
    std::string original_ir, optimized_ir, source, plan_text, cubin_path;
    LoadedModule mod;
    std::vector<CUfunction> region_fn;  // per region index
    char* arena = nullptr;
    std::vector<Shape> in_shapes, out_shapes;
    std::vector<int64_t> in_bytes, out_bytes;
    size_t cse_removed = 0, dce_removed = 0, original_nodes = 0;
    cudaStream_t last_stream = nullptr;
    bool profiling = false;
    std::vector<cudaEvent_t> events;
    std::vector<double> prof_sum;   // per launch: summed ms over profiled runs
    int64_t prof_runs = 0;
    bool prof_pending = false;
    bool has_tc = false;
    std::vector<cudaEvent_t> out_events;  // caller's events, recorded when an output is complete
    std::vector<cudaEvent_t> in_events;   // caller's events, recorded after an input's last reader
    cudaStream_t side = nullptr;          // second stream for concurrent GEMM pairs
    cudaEvent_t fork_ev = nullptr, join_ev = nullptr;
    std::mutex run_mutex;
    // per-run scratch, reused under run_mutex so a run allocates no host memory after the first
    std::vector<char*> in_ptr, out_ptr;
    std::vector<void*> arg_vals, arg_ptrs;

    ~tt_program() {
        for (cudaEvent_t e : events) cudaEventDestroy(e);
        if (fork_ev) cudaEventDestroy(fork_ev);
        if (join_ev) cudaEventDestroy(join_ev);
        if (side) cudaStreamDestroy(side);
        if (mod.module) driver().moduleUnload(mod.module);
        if (arena) cudaFree(arena);
    }
};

static int launches_of(const Plan& p, const Launch& L) {
    if (L.type == LT_REGION) return p.regions[static_cast<size_t>(L.region)].grid > 0 ? 1 : 0;
    if (L.type == LT_REDUCE) return L.rd.outer == 0 ? 0 : (L.rd.R == 0 ? 1 : (L.rd.splits > 1 ? 2 : 1));
    return gemm_launch_count(L.gd);
}

static std::string execution_plan(const tt_program& p) {
    const Graph& g = p.plan.g;
    std::ostringstream ss;
    ss << "=== TinyTensor Execution Plan ===\n";
    ss << "Execution Mode: Compiled CUDA (sm_100a)\n";
    ss << "Input Nodes (" << g.inputs.size() << "):\n";
    for (int k : g.inputs) {
        const Node& n = g.nodes[static_cast<size_t>(k)];
        ss << "  %" << n.id << " [" << tuple_str(n.shape) << ", float32]";
        if (!n.name.empty()) ss << " name=\"" << n.name << "\"";
        ss << "\n";
    }
    ss << "Output Nodes (" << g.outputs.size() << "):\n";
    for (int k : g.outputs) {
        const Node& n = g.nodes[static_cast<size_t>(k)];
        ss << "  %" << n.id << " [" << tuple_str(n.shape) << ", float32]\n";
    }
    ss << "Execution Sequence (Topological, " << g.nodes.size() << " nodes):\n";
    for (const Node& n : g.nodes)
        ss << "  %" << n.id << " = " << op_name(n.op) << " " << tuple_str(n.shape) << " (float32)\n";
    ss << "Binary Object: " << (p.cubin_path.empty() ? std::string("(in-memory cubin)") : p.cubin_path) << "\n";
    const Plan& pl = p.plan;
    int64_t saved = pl.total_alloc_bytes > pl.peak_planned_bytes ? pl.total_alloc_bytes - pl.peak_planned_bytes : 0;
    ss << "Memory Planning: Peak " << pl.peak_planned_bytes << " bytes (saved " << saved << " bytes via "
       << pl.reused_buffers << " reused buffers)\n";
    ss << "Fused Regions: " << pl.fused_regions << ", CSE Replacements: " << p.cse_removed
       << ", DCE Eliminated Nodes: " << p.dce_removed << "\n";
    ss << p.plan_text;
    ss << "=================================";
    return ss.str();
}

extern "C" {

const char* tt_last_error(void) { return g_last_error.c_str(); }
int tt_version(void) { return 100; }
uint64_t tt_launch_count(void) { return g_launches.load(); }

int tt_device_init(int32_t device) {
    return guarded([&] {
        int n = 0;
        cudaError_t e = cudaGetDeviceCount(&n);
        if (e != cudaSuccess || n == 0) {
            cudaGetLastError();
            fail(TT_ERR_NO_DEVICE, "no CUDA device is available");
        }
        if (device < 0 || device >= n) fail(TT_ERR_NO_DEVICE, "device ordinal out of range");
        cudaDeviceProp prop;
        check_cuda(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
        if (prop.major != 10 || prop.minor != 0)
            fail(TT_ERR_NO_DEVICE, std::string("device is ") + prop.name + " (sm_" + std::to_string(prop.major) +
                                       std::to_string(prop.minor) + "); this backend is built for sm_100a (B200)");
        check_cuda(cudaSetDevice(device), "cudaSetDevice");
        check_cuda(cudaFree(nullptr), "context creation");
    });
}

int tt_graph_ir(const tt_graph* g, char* buf, size_t cap, size_t* needed) {
    return guarded([&] { copy_out(ir_text(import_graph(g)), buf, cap, needed); });
}

int tt_graph_verify(const tt_graph* g) {
    return guarded([&] { verify(import_graph(g)); });
}

int tt_compile(const tt_graph* cg, const tt_compile_options* opt, tt_program** out) {
    return guarded([&] {
        if (!out) fail(TT_ERR_INVALID, "null output handle");
        *out = nullptr;
        tt_compile_options o{};
        o.optimize = 1;
        o.grad_loss = -1;
        if (opt) o = *opt;
        auto p = std::make_unique<tt_program>();
        p->device = o.device;
        Graph g = import_graph(cg);
        p->original_ir = ir_text(g);
        p->original_nodes = g.nodes.size();
        verify(g);
        if (o.grad_loss >= 0) {
            std::vector<int> wrt(o.grad_wrt, o.grad_wrt + o.num_grad_wrt);
            append_gradients(g, o.grad_loss, wrt);
        }
        g = expand_fused(g);
        if (o.optimize) g = cse(g, &p->cse_removed);
        g = dce(g, &p->dce_removed);
        verify(g);
        p->optimized_ir = ir_text(g);
        ScheduleOptions so;
        so.fuse = !(o.flags & TT_FLAG_NO_FUSION);
        so.gemm_epilogue = !(o.flags & TT_FLAG_NO_GEMM_FUSION);
        so.concurrent_gemms = !(o.flags & TT_FLAG_SERIAL);
        p->plan = schedule(g, so);
        p->source = generate_source(p->plan);
        for (int k : p->plan.g.inputs) {
            p->in_shapes.push_back(p->plan.g.nodes[static_cast<size_t>(k)].shape);
            p->in_bytes.push_back(numel(p->in_shapes.back()) * 4);
        }
        for (int k : p->plan.g.outputs) {
            p->out_shapes.push_back(p->plan.g.nodes[static_cast<size_t>(k)].shape);
            p->out_bytes.push_back(numel(p->out_shapes.back()) * 4);
        }
        for (const Launch& L : p->plan.launches) p->has_tc |= (L.type == LT_GEMM && L.gd.algo == 2);

        // Generated kernels: NVRTC -> cubin (cached); loaded unless host-only.
        const bool host_only = (o.flags & TT_FLAG_HOST_ONLY) != 0;
        if (!host_only && tt_device_init(o.device) != TT_OK) throw Error(TT_ERR_NO_DEVICE, g_last_message);
        std::vector<std::string> used;
        std::vector<int> used_idx;
        for (size_t i = 0; i < p->plan.regions.size(); ++i)
            if (!p->plan.regions[i].kernel.empty()) {
                used.push_back(p->plan.regions[i].kernel);
                used_idx.push_back(static_cast<int>(i));
            }
        p->region_fn.assign(p->plan.regions.size(), nullptr);
        p->plan_text = plan_text(p->plan);
        if (!used.empty()) {
            std::string key = cache_key(p->optimized_ir, p->source);
            if (host_only) {
                p->cubin_path = compile_to_cache(key, p->source, o.cache_dir ? o.cache_dir : "");
            } else {
                p->mod = load_program_module(key, p->source, o.cache_dir ? o.cache_dir : "", used);
                for (size_t i = 0; i < used_idx.size(); ++i)
                    p->region_fn[static_cast<size_t>(used_idx[i])] = p->mod.functions[i];
                p->cubin_path = p->mod.cubin_path;
            }
        }
        if (host_only) {
            p->device = -1;
            *out = p.release();
            return;
        }
        check_cuda(cudaMalloc(reinterpret_cast<void**>(&p->arena), static_cast<size_t>(p->plan.arena_bytes)),
                   "cudaMalloc(arena)");
        for (const auto& c : p->plan.constants) {
            const Node& n = p->plan.g.nodes[static_cast<size_t>(c.second)];
            check_cuda(cudaMemcpy(p->arena + c.first, n.cdata.data(), n.cdata.size() * sizeof(float),
                                  cudaMemcpyHostToDevice),
                       "constant upload");
        }
        check_cuda(cudaMemset(p->arena + p->plan.status_offset, 0, 256), "status word init");
        bool pairs = false;
        for (const Launch& L : p->plan.launches) pairs |= L.concurrent_next;
        if (pairs) {
            check_cuda(cudaStreamCreateWithFlags(&p->side, cudaStreamNonBlocking), "cudaStreamCreate(side)");
            check_cuda(cudaEventCreateWithFlags(&p->fork_ev, cudaEventDisableTiming), "cudaEventCreate(fork)");
            check_cuda(cudaEventCreateWithFlags(&p->join_ev, cudaEventDisableTiming), "cudaEventCreate(join)");
        }
        *out = p.release();
    });
}

int tt_program_info(const tt_program* p, int32_t what, char* buf, size_t cap, size_t* needed) {
    return guarded([&] {
        if (!p) fail(TT_ERR_INVALID, "null program");
        switch (what) {
            case TT_INFO_ORIGINAL_IR: copy_out(p->original_ir, buf, cap, needed); break;
            case TT_INFO_OPTIMIZED_IR: copy_out(p->optimized_ir, buf, cap, needed); break;
            case TT_INFO_SOURCE: copy_out(p->source, buf, cap, needed); break;
            case TT_INFO_PLAN: copy_out(execution_plan(*p), buf, cap, needed); break;
            case TT_INFO_CUBIN_PATH: copy_out(p->cubin_path, buf, cap, needed); break;
            default: fail(TT_ERR_INVALID, "unknown info selector");
        }
    });
}

int tt_program_num_io(const tt_program* p, int32_t* ni, int32_t* no) {
    return guarded([&] {
        if (!p) fail(TT_ERR_INVALID, "null program");
        if (ni) *ni = static_cast<int32_t>(p->in_shapes.size());
        if (no) *no = static_cast<int32_t>(p->out_shapes.size());
    });
}

int tt_program_output_shape(const tt_program* p, int32_t index, int32_t* rank, int64_t* shape) {
    return guarded([&] {
        if (!p) fail(TT_ERR_INVALID, "null program");
        if (index < 0 || static_cast<size_t>(index) >= p->out_shapes.size()) fail(TT_ERR_INVALID, "output index");
        const Shape& s = p->out_shapes[static_cast<size_t>(index)];
        if (rank) *rank = static_cast<int32_t>(s.size());
        if (shape)
            for (size_t i = 0; i < s.size(); ++i) shape[i] = s[i];
    });
}

static void collect_profile(tt_program* p);

static void run_launches(tt_program* p, char* const* in_ptr, char* const* out_ptr, cudaStream_t stream) {
    const Plan& pl = p->plan;
    if (p->prof_pending) collect_profile(p);  // waits for the previous profiled run only
    auto resolve = [&](const BufRef& r) -> char* {
        switch (r.kind) {
            case BK_ARENA: return p->arena + r.offset;
            case BK_INPUT: return in_ptr[r.index] + r.offset;
            case BK_OUTPUT: return out_ptr[r.index] + r.offset;
            default: return nullptr;
        }
    };
    int* status = reinterpret_cast<int*>(p->arena + pl.status_offset);
    const size_t n = pl.launches.size();
    if (p->profiling) {
        // start and end event per launch (launches of a concurrent pair overlap)
        while (p->events.size() < 2 * n) {
            cudaEvent_t e;
            check_cuda(cudaEventCreate(&e), "cudaEventCreate");
            p->events.push_back(e);
        }
    }
    auto record_outputs = [&](int step, cudaStream_t st) {
        for (size_t k = 0; k < p->out_events.size(); ++k)
            if (p->out_events[k] && pl.output_step[k] == step)
                check_cuda(cudaEventRecord(p->out_events[k], st), "cudaEventRecord(output)");
        for (size_t k = 0; k < p->in_events.size(); ++k)
            if (p->in_events[k] && pl.input_last_step[k] == step)
                check_cuda(cudaEventRecord(p->in_events[k], st), "cudaEventRecord(input)");
    };
    auto launch_one = [&](size_t s, cudaStream_t st) {
        const Launch& L = pl.launches[s];
        if (p->profiling) check_cuda(cudaEventRecord(p->events[2 * s], st), "cudaEventRecord");
        int rc = 0;
        if (L.type == LT_REGION) {
            const Region& r = pl.regions[static_cast<size_t>(L.region)];
            if (r.grid > 0) {
                std::vector<void*>& vals = p->arg_vals;
                vals.clear();
                for (size_t e = 0; e < r.ext.size(); ++e) {
                    const Access& a = r.ext_access[e];
                    vals.push_back(a.imm ? nullptr : resolve(pl.root_ref[static_cast<size_t>(a.node)]));
                }
                for (const BufRef& b : r.store_ref) vals.push_back(resolve(b));
                if (r.copy_store >= 0) {  // hi/lo operand copies: [R][C] hi, lo, then [C][R] hi, lo
                    char* base = resolve(L.split_ref);
                    for (int layout = 0; layout < 2; ++layout)
                        for (int lo = 0; lo < 2; ++lo)
                            vals.push_back((layout == 0 ? r.copy_rows : r.copy_t)
                                               ? base + split_copies_offset(r.copy_R, r.copy_C, r.copy_rows, layout, lo)
                                               : nullptr);
                }
                std::vector<void*>& args = p->arg_ptrs;
                args.resize(vals.size());
                for (size_t i = 0; i < vals.size(); ++i) args[i] = &vals[i];
                CUresult cr = driver().launchKernel(p->region_fn[static_cast<size_t>(L.region)],
                                                    static_cast<unsigned>(r.grid), 1, 1, 256, 1, 1, 0, st,
                                                    args.data(), nullptr);
                if (cr != CUDA_SUCCESS) fail(TT_ERR_RUNTIME, "cuLaunchKernel(" + r.kernel + "): " + cu_error(cr));
            }
        } else if (L.type == LT_REDUCE) {
            rc = launch_reduce(L.rd, reinterpret_cast<const float*>(resolve(L.in_ref)),
                               reinterpret_cast<float*>(resolve(L.out_ref)), resolve(L.scratch_ref), st);
        } else {
            // operands whose hi/lo copies the producing region wrote
            GemmSplitIO io;
            auto copies = [&](int src, int layout, const float*& hi, const float*& lo) {
                const Launch& P = pl.launches[static_cast<size_t>(src)];
                const Region& r = pl.regions[static_cast<size_t>(P.region)];
                char* base = resolve(P.split_ref);
                hi = reinterpret_cast<const float*>(base + split_copies_offset(r.copy_R, r.copy_C, r.copy_rows, layout, 0));
                lo = reinterpret_cast<const float*>(base + split_copies_offset(r.copy_R, r.copy_C, r.copy_rows, layout, 1));
            };
            if (L.gd.a_presplit) copies(L.a_split_src, L.a_split_layout, io.a_hi, io.a_lo);
            if (L.gd.b_presplit) copies(L.b_split_src, L.b_split_layout, io.b_hi, io.b_lo);
            rc = launch_gemm(L.gd, reinterpret_cast<const float*>(resolve(L.in_ref)),
                             reinterpret_cast<const float*>(resolve(L.in_ref2)),
                             reinterpret_cast<float*>(resolve(L.out_ref)), resolve(L.scratch_ref), status, st, &io);
        }
        if (rc) fail(TT_ERR_RUNTIME, L.label + ": " + cudaGetErrorString(static_cast<cudaError_t>(rc)));
        g_launches += static_cast<uint64_t>(launches_of(pl, L));
        if (p->profiling) check_cuda(cudaEventRecord(p->events[2 * s + 1], st), "cudaEventRecord");
        record_outputs(static_cast<int>(s), st);
    };
    record_outputs(-1, stream);
    for (size_t s = 0; s < n; ++s) {
        if (pl.launches[s].concurrent_next && p->side) {
            // fork: the side stream starts after everything queued so far; join: the run's
            // stream continues after both
            check_cuda(cudaEventRecord(p->fork_ev, stream), "cudaEventRecord(fork)");
            check_cuda(cudaStreamWaitEvent(p->side, p->fork_ev, 0), "cudaStreamWaitEvent(fork)");
            launch_one(s, stream);
            launch_one(s + 1, p->side);
            check_cuda(cudaEventRecord(p->join_ev, p->side), "cudaEventRecord(join)");
            check_cuda(cudaStreamWaitEvent(stream, p->join_ev, 0), "cudaStreamWaitEvent(join)");
            ++s;
        } else {
            launch_one(s, stream);
        }
    }
    p->prof_pending = p->profiling;
}

// Adds the last profiled run's per-launch times to the running sums.
static void collect_profile(tt_program* p) {
    if (!p->prof_pending) return;
    p->prof_pending = false;
    const size_t n = p->plan.launches.size();
    if (n == 0) return;
    for (size_t s = 0; s < n; ++s) check_cuda(cudaEventSynchronize(p->events[2 * s + 1]), "profile event");
    if (p->prof_sum.size() != n) p->prof_sum.assign(n, 0.0);
    for (size_t s = 0; s < n; ++s) {
        float ms = 0.f;
        check_cuda(cudaEventElapsedTime(&ms, p->events[2 * s], p->events[2 * s + 1]), "cudaEventElapsedTime");
        p->prof_sum[s] += ms;
    }
    p->prof_runs++;
}

int tt_program_run(tt_program* p, const void* const* inputs, void* const* outputs, int32_t where, void* stream_v) {
    return guarded([&] {
        if (!p) fail(TT_ERR_INVALID, "null program");
        std::lock_guard<std::mutex> lk(p->run_mutex);
        const size_t ni = p->in_shapes.size(), no = p->out_shapes.size();
        if (ni && !inputs) fail(TT_ERR_RUNTIME, "Expected " + std::to_string(ni) + " inputs, but got none");
        if (no && !outputs) fail(TT_ERR_RUNTIME, "Expected " + std::to_string(no) + " output buffers, but got none");
        cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
        if (p->device < 0) fail(TT_ERR_NO_DEVICE, "program was compiled host-only (TT_FLAG_HOST_ONLY)");
        check_cuda(cudaSetDevice(p->device), "cudaSetDevice");
        std::vector<char*>& in_ptr = p->in_ptr;
        std::vector<char*>& out_ptr = p->out_ptr;
        in_ptr.assign(ni, nullptr);
        out_ptr.assign(no, nullptr);
        for (size_t k = 0; k < ni; ++k)
            if (!inputs[k] && p->in_bytes[k]) fail(TT_ERR_RUNTIME, "Input " + std::to_string(k) + " is null");
        for (size_t k = 0; k < no; ++k)
            if (!outputs[k] && p->out_bytes[k]) fail(TT_ERR_RUNTIME, "Output " + std::to_string(k) + " is null");
        if (where == TT_HOST) {
            for (size_t k = 0; k < ni; ++k) {
                in_ptr[k] = p->arena + p->plan.stage_in[k];
                if (p->in_bytes[k])
                    check_cuda(cudaMemcpyAsync(in_ptr[k], inputs[k], static_cast<size_t>(p->in_bytes[k]),
                                               cudaMemcpyHostToDevice, stream),
                               "input copy");
            }
            for (size_t k = 0; k < no; ++k) out_ptr[k] = p->arena + p->plan.stage_out[k];
        } else if (where == TT_DEVICE) {
            for (size_t k = 0; k < ni; ++k) {
                in_ptr[k] = const_cast<char*>(static_cast<const char*>(inputs[k]));
                if (reinterpret_cast<uintptr_t>(in_ptr[k]) % 16)
                    fail(TT_ERR_RUNTIME, "device input " + std::to_string(k) + " is not 16-byte aligned");
            }
            for (size_t k = 0; k < no; ++k) {
                out_ptr[k] = static_cast<char*>(outputs[k]);
                if (reinterpret_cast<uintptr_t>(out_ptr[k]) % 16)
                    fail(TT_ERR_RUNTIME, "device output " + std::to_string(k) + " is not 16-byte aligned");
            }
        } else {
            fail(TT_ERR_INVALID, "where must be TT_HOST or TT_DEVICE");
        }
        run_launches(p, in_ptr.data(), out_ptr.data(), stream);
        p->last_stream = stream;
        if (where == TT_HOST) {
            for (size_t k = 0; k < no; ++k)
                if (p->out_bytes[k])
                    check_cuda(cudaMemcpyAsync(outputs[k], out_ptr[k], static_cast<size_t>(p->out_bytes[k]),
                                               cudaMemcpyDeviceToHost, stream),
                               "output copy");
            int32_t status = 0;
            if (p->has_tc)
                check_cuda(cudaMemcpyAsync(&status, p->arena + p->plan.status_offset, sizeof(status),
                                           cudaMemcpyDeviceToHost, stream),
                           "status copy");
            check_cuda(cudaStreamSynchronize(stream), "kernel execution");
            collect_profile(p);
            if (status != 0) {
                cudaMemsetAsync(p->arena + p->plan.status_offset, 0, 4, stream);
                fail(TT_ERR_DEVICE_STATUS, "a kernel gave up a bounded wait (status " + std::to_string(status) + ")");
            }
        }
    });
}

int tt_program_set_output_events(tt_program* p, void* const* events, int32_t n) {
    return guarded([&] {
        if (!p) fail(TT_ERR_INVALID, "null program");
        if (n < 0 || static_cast<size_t>(n) > p->out_shapes.size() || (n > 0 && !events))
            fail(TT_ERR_INVALID, "events: expected at most " + std::to_string(p->out_shapes.size()) + " entries");
        std::lock_guard<std::mutex> lk(p->run_mutex);
        p->out_events.assign(static_cast<size_t>(n), nullptr);
        for (int32_t k = 0; k < n; ++k) p->out_events[static_cast<size_t>(k)] = static_cast<cudaEvent_t>(events[k]);
    });
}

int tt_program_set_input_events(tt_program* p, void* const* events, int32_t n) {
    return guarded([&] {
        if (!p) fail(TT_ERR_INVALID, "null program");
        if (n < 0 || static_cast<size_t>(n) > p->in_shapes.size() || (n > 0 && !events))
            fail(TT_ERR_INVALID, "events: expected at most " + std::to_string(p->in_shapes.size()) + " entries");
        std::lock_guard<std::mutex> lk(p->run_mutex);
        p->in_events.assign(static_cast<size_t>(n), nullptr);
        for (int32_t k = 0; k < n; ++k) p->in_events[static_cast<size_t>(k)] = static_cast<cudaEvent_t>(events[k]);
    });
}

int tt_program_input_step(tt_program* p, int32_t input, int32_t* step) {
    return guarded([&] {
        if (!p || !step) fail(TT_ERR_INVALID, "null argument");
        if (input < 0 || static_cast<size_t>(input) >= p->plan.input_last_step.size())
            fail(TT_ERR_INVALID, "input index out of range");
        *step = p->plan.input_last_step[static_cast<size_t>(input)];
    });
}

int tt_program_output_step(tt_program* p, int32_t output, int32_t* step) {
    return guarded([&] {
        if (!p || !step) fail(TT_ERR_INVALID, "null argument");
        if (output < 0 || static_cast<size_t>(output) >= p->plan.output_step.size())
            fail(TT_ERR_INVALID, "output index out of range");
        *step = p->plan.output_step[static_cast<size_t>(output)];
    });
}

int tt_event_create(void** event) {
    return guarded([&] {
        if (!event) fail(TT_ERR_INVALID, "null argument");
        cudaEvent_t e;
        check_cuda(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
        *event = e;
    });
}

int tt_event_destroy(void* event) {
    return guarded([&] {
        if (event) check_cuda(cudaEventDestroy(static_cast<cudaEvent_t>(event)), "cudaEventDestroy");
    });
}

int tt_event_record(void* event, void* stream) {
    return guarded([&] {
        if (!event) fail(TT_ERR_INVALID, "null event");
        check_cuda(cudaEventRecord(static_cast<cudaEvent_t>(event), static_cast<cudaStream_t>(stream)),
                   "cudaEventRecord");
    });
}

int tt_stream_wait_event(void* stream, void* event) {
    return guarded([&] {
        if (!event) fail(TT_ERR_INVALID, "null event");
        check_cuda(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), static_cast<cudaEvent_t>(event), 0),
                   "cudaStreamWaitEvent");
    });
}

int tt_selftest_bounded_wait(int64_t budget_cycles, int32_t* status_out) {
    return guarded([&] {
        if (!status_out) fail(TT_ERR_INVALID, "null argument");
        if (budget_cycles < 0 || budget_cycles > 4000000000LL) fail(TT_ERR_INVALID, "budget must be 0..4e9 cycles");
        int* d = nullptr;
        check_cuda(cudaMalloc(reinterpret_cast<void**>(&d), sizeof(int)), "cudaMalloc(status)");
        cudaError_t e = cudaMemset(d, 0, sizeof(int));
        if (e == cudaSuccess) e = static_cast<cudaError_t>(launch_bounded_wait_selftest(d, budget_cycles, nullptr));
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        int32_t v = 0;
        if (e == cudaSuccess) e = cudaMemcpy(&v, d, sizeof(int), cudaMemcpyDeviceToHost);
        cudaFree(d);
        check_cuda(e, "bounded-wait self-test");
        *status_out = v;
    });
}

int tt_stream_begin_capture(void* stream) {
    return guarded([&] {
        if (!stream) fail(TT_ERR_INVALID, "capture needs a created stream, not the legacy default stream");
        check_cuda(cudaStreamBeginCapture(static_cast<cudaStream_t>(stream), cudaStreamCaptureModeThreadLocal),
                   "cudaStreamBeginCapture");
    });
}

int tt_stream_end_capture(void* stream, void** graph_exec) {
    return guarded([&] {
        if (!stream || !graph_exec) fail(TT_ERR_INVALID, "null argument");
        *graph_exec = nullptr;
        cudaGraph_t graph = nullptr;
        check_cuda(cudaStreamEndCapture(static_cast<cudaStream_t>(stream), &graph), "cudaStreamEndCapture");
        cudaGraphExec_t exec = nullptr;
        cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        check_cuda(e, "cudaGraphInstantiate");
        *graph_exec = exec;
    });
}

int tt_graph_launch(void* graph_exec, void* stream) {
    return guarded([&] {
        if (!graph_exec) fail(TT_ERR_INVALID, "null graph");
        check_cuda(cudaGraphLaunch(static_cast<cudaGraphExec_t>(graph_exec), static_cast<cudaStream_t>(stream)),
                   "cudaGraphLaunch");
    });
}

int tt_graph_destroy(void* graph_exec) {
    return guarded([&] {
        if (graph_exec) check_cuda(cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(graph_exec)), "cudaGraphExecDestroy");
    });
}

int tt_program_status(tt_program* p, int32_t* device_status) {
    return guarded([&] {
        if (!p) fail(TT_ERR_INVALID, "null program");
        if (p->device < 0) fail(TT_ERR_NO_DEVICE, "program was compiled host-only (TT_FLAG_HOST_ONLY)");
        check_cuda(cudaSetDevice(p->device), "cudaSetDevice");
        int32_t status = 0;
        check_cuda(cudaMemcpyAsync(&status, p->arena + p->plan.status_offset, sizeof(status), cudaMemcpyDeviceToHost,
                                   p->last_stream),
                   "status copy");
        check_cuda(cudaStreamSynchronize(p->last_stream), "kernel execution");
        collect_profile(p);
        if (device_status) *device_status = status;
        if (status != 0) {
            cudaMemset(p->arena + p->plan.status_offset, 0, 4);
            fail(TT_ERR_DEVICE_STATUS, "a kernel gave up a bounded wait (status " + std::to_string(status) + ")");
        }
    });
}

int tt_program_set_profiling(tt_program* p, int32_t enable) {
    return guarded([&] {
        if (!p) fail(TT_ERR_INVALID, "null program");
        if (p->prof_pending) collect_profile(p);
        p->profiling = enable != 0;
        p->prof_sum.clear();
        p->prof_runs = 0;
    });
}

int tt_program_profile(const tt_program* pc, int32_t cap, char* names, int32_t name_cap, float* ms, int32_t* count) {
    return guarded([&] {
        if (!pc) fail(TT_ERR_INVALID, "null program");
        tt_program* p = const_cast<tt_program*>(pc);
        if (p->prof_pending) collect_profile(p);
        int32_t n = static_cast<int32_t>(p->prof_sum.size());
        if (count) *count = n;
        for (int32_t i = 0; i < n && i < cap; ++i) {
            if (ms) ms[i] = static_cast<float>(p->prof_sum[static_cast<size_t>(i)] / static_cast<double>(p->prof_runs));
            if (names && name_cap > 0) {
                const std::string& l = p->plan.launches[static_cast<size_t>(i)].label;
                size_t m = std::min(static_cast<size_t>(name_cap - 1), l.size());
                std::memcpy(names + static_cast<size_t>(i) * static_cast<size_t>(name_cap), l.data(), m);
                names[static_cast<size_t>(i) * static_cast<size_t>(name_cap) + m] = '\0';
            }
        }
    });
}

int tt_program_destroy(tt_program* p) {
    return guarded([&] {
        if (!p) return;
        if (p->device >= 0) cudaSetDevice(p->device);
        delete p;
    });
}

int tt_device_alloc(size_t bytes, void** ptr) {
    return guarded([&] {
        if (!ptr) fail(TT_ERR_INVALID, "null pointer slot");
        check_cuda(cudaMalloc(ptr, bytes ? bytes : 1), "cudaMalloc");
    });
}
int tt_device_free(void* ptr) {
    return guarded([&] { check_cuda(cudaFree(ptr), "cudaFree"); });
}
int tt_host_alloc(size_t bytes, void** ptr) {
    return guarded([&] {
        if (!ptr) fail(TT_ERR_INVALID, "null pointer slot");
        check_cuda(cudaMallocHost(ptr, bytes ? bytes : 1), "cudaMallocHost");
    });
}
int tt_host_free(void* ptr) {
    return guarded([&] { check_cuda(cudaFreeHost(ptr), "cudaFreeHost"); });
}
int tt_memcpy(void* dst, const void* src, size_t bytes, int32_t kind, void* stream) {
    return guarded([&] {
        cudaMemcpyKind k = kind == TT_H2D ? cudaMemcpyHostToDevice
                           : kind == TT_D2H ? cudaMemcpyDeviceToHost
                                            : cudaMemcpyDeviceToDevice;
        check_cuda(cudaMemcpyAsync(dst, src, bytes, k, static_cast<cudaStream_t>(stream)), "cudaMemcpyAsync");
    });
}
int tt_stream_create(void** stream) {
    return guarded([&] {
        if (!stream) fail(TT_ERR_INVALID, "null stream slot");
        check_cuda(cudaStreamCreateWithFlags(reinterpret_cast<cudaStream_t*>(stream), cudaStreamNonBlocking),
                   "cudaStreamCreate");
    });
}
int tt_stream_destroy(void* stream) {
    return guarded([&] { check_cuda(cudaStreamDestroy(static_cast<cudaStream_t>(stream)), "cudaStreamDestroy"); });
}
int tt_stream_sync(void* stream) {
    return guarded([&] { check_cuda(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "cudaStreamSynchronize"); });
}

int tt_sgd_step(int32_t n, float* const* params, const float* const* grads, float* const* velocities,
                const int64_t* numels, float lr, float momentum, void* stream) {
    return guarded([&] {
        if (n < 0 || (n > 0 && (!params || !grads || !numels))) fail(TT_ERR_INVALID, "bad SGD arguments");
        if (momentum > 0.0f && !velocities) fail(TT_ERR_INVALID, "momentum needs velocity buffers");
        int rc = launch_sgd(n, params, grads, momentum > 0.0f ? velocities : nullptr, numels, lr, momentum, stream);
        if (rc) fail(TT_ERR_RUNTIME, std::string("sgd: ") + cudaGetErrorString(static_cast<cudaError_t>(rc)));
        int64_t total = 0;
        for (int32_t i = 0; i < n; ++i) total += numels[i];
        if (total > 0) g_launches += static_cast<uint64_t>((n + 15) / 16);
    });
}

}  // extern "C"
