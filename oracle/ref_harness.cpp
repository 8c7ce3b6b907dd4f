// Test infrastructure: a plain C-ABI around the reference TinyTensor C++ library,
// compiled from the reference's own sources (see oracle/Makefile) into
// oracle/_ref/libttref.so.  It lets the tests and the CPU-baseline leg of bench.py
// drive the UNMODIFIED reference (its Graph builders, Optimizer, Interpreter,
// CppBackend/Executable and eager Autodiff) without pybind11.
//
// Nothing in the shipped tinytensor_b200 package links or loads this file.
//
// Reference entry points used (paths inside the reference project):
//   Graph builders            src/graph/graph.cpp:51-200
//   Executor (optimize, mode) src/runtime/executor.cpp:9-56, run :100-127
//   Autodiff                  src/autodiff/gradient.cpp:52-332
//
// Ops the reference has no OpType for are expressed through identities over
// reference ops, so that the reference itself evaluates them:
//   neg(x)  = 0 - x
//   exp(x)  = sigmoid(x) / sigmoid(-x)
//   tanh(x) = 2*sigmoid(2x) - 1
// reduce_max has no reference identity and is rejected here (the C restatement in
// oracle/tt_oracle.c defines it).

#include <chrono>
#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "tinytensor/autodiff/gradient.hpp"
#include "tinytensor/core/tensor.hpp"
#include "tinytensor/graph/graph.hpp"
#include "tinytensor/ir/printer.hpp"
#include "tinytensor/runtime/executor.hpp"
#ifdef TTREF_WITH_CUDA
// Built by integration/Makefile against the reference tree with the CompiledCUDA mode
// added (integration/executor.patch): mode 5 and the device-tensor entry points below.
#include "tinytensor/runtime/cuda_executable.hpp"
#endif

using namespace tinytensor;

namespace {

thread_local std::string g_err;

// Op codes shared with include/tt_cuda.h (same order as the reference OpType).
enum HOp {
    H_INPUT = 0, H_CONSTANT = 1, H_ADD = 2, H_SUB = 3, H_MUL = 4, H_DIV = 5,
    H_RELU = 6, H_SIGMOID = 7, H_MATMUL = 8, H_TRANSPOSE = 9,
    H_REDUCE_SUM = 10, H_REDUCE_MEAN = 11,
    H_EXP = 14, H_NEG = 15, H_TANH = 16, H_REDUCE_MAX = 17,
};

struct HGraph {
    Graph g;
    std::vector<Node*> nodes;  // index -> reference node (user-visible handle)
};

struct HExec {
    std::unique_ptr<Executor> ex;
    HGraph* hg;
    std::vector<Tensor> bound;  // inputs bound once for timed runs
};

Shape make_shape(const int64_t* dims, int rank) {
    std::vector<int64_t> v(dims, dims + rank);
    return Shape(v);
}

Node* scalar_const(Graph& g, double v) { return g.create_constant(Tensor::scalar(v, DType::Float32)); }

int push(HGraph* hg, Node* n) {
    hg->nodes.push_back(n);
    return static_cast<int>(hg->nodes.size()) - 1;
}

template <typename F>
int guarded(F&& f) {
    try {
        return f();
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

}  // namespace

extern "C" {

const char* ttref_last_error() { return g_err.c_str(); }

void* ttref_graph_new() { return new HGraph(); }
void ttref_graph_free(void* p) { delete static_cast<HGraph*>(p); }

int ttref_input(void* p, const int64_t* shape, int rank, const char* name) {
    auto* hg = static_cast<HGraph*>(p);
    return guarded([&] { return push(hg, hg->g.create_input(make_shape(shape, rank), DType::Float32, name ? name : "")); });
}

int ttref_constant(void* p, const float* data, const int64_t* shape, int rank) {
    auto* hg = static_cast<HGraph*>(p);
    return guarded([&] {
        Tensor t(make_shape(shape, rank), DType::Float32);
        std::memcpy(t.raw_data(), data, t.nbytes());
        return push(hg, hg->g.create_constant(t));
    });
}

int ttref_op(void* p, int op, int a, int b) {
    auto* hg = static_cast<HGraph*>(p);
    return guarded([&] {
        Graph& g = hg->g;
        Node* x = hg->nodes.at(static_cast<size_t>(a));
        Node* y = (b >= 0) ? hg->nodes.at(static_cast<size_t>(b)) : nullptr;
        Node* r = nullptr;
        switch (op) {
            case H_ADD: r = g.add(x, y); break;
            case H_SUB: r = g.sub(x, y); break;
            case H_MUL: r = g.mul(x, y); break;
            case H_DIV: r = g.div(x, y); break;
            case H_RELU: r = g.relu(x); break;
            case H_SIGMOID: r = g.sigmoid(x); break;
            case H_MATMUL: r = g.matmul(x, y); break;
            case H_NEG: r = g.sub(scalar_const(g, 0.0), x); break;
            case H_EXP: r = g.div(g.sigmoid(x), g.sigmoid(g.sub(scalar_const(g, 0.0), x))); break;
            case H_TANH:
                r = g.sub(g.mul(scalar_const(g, 2.0), g.sigmoid(g.mul(scalar_const(g, 2.0), x))),
                          scalar_const(g, 1.0));
                break;
            default: throw std::runtime_error("ttref_op: unsupported op " + std::to_string(op));
        }
        return push(hg, r);
    });
}

int ttref_transpose(void* p, int a, int64_t d0, int64_t d1) {
    auto* hg = static_cast<HGraph*>(p);
    return guarded([&] { return push(hg, hg->g.transpose(hg->nodes.at(static_cast<size_t>(a)), d0, d1)); });
}

int ttref_reduce(void* p, int op, int a, const int64_t* axes, int naxes, int keepdims) {
    auto* hg = static_cast<HGraph*>(p);
    return guarded([&] {
        std::vector<int64_t> ax(axes, axes + naxes);
        Node* x = hg->nodes.at(static_cast<size_t>(a));
        if (op == H_REDUCE_SUM) return push(hg, hg->g.reduce_sum(x, ax, keepdims != 0));
        if (op == H_REDUCE_MEAN) return push(hg, hg->g.reduce_mean(x, ax, keepdims != 0));
        throw std::runtime_error("ttref_reduce: the reference has no reduction op " + std::to_string(op));
    });
}

int ttref_mark_output(void* p, int n) {
    auto* hg = static_cast<HGraph*>(p);
    return guarded([&] {
        hg->g.mark_output(hg->nodes.at(static_cast<size_t>(n)));
        return 0;
    });
}

int ttref_node_rank(void* p, int n) {
    auto* hg = static_cast<HGraph*>(p);
    return static_cast<int>(hg->nodes.at(static_cast<size_t>(n))->shape().ndim());
}

void ttref_node_shape(void* p, int n, int64_t* out) {
    auto* hg = static_cast<HGraph*>(p);
    const Shape& s = hg->nodes.at(static_cast<size_t>(n))->shape();
    for (size_t i = 0; i < s.ndim(); ++i) out[i] = s[i];
}

// Canonical IR text of the graph (IRPrinter::to_string); returns bytes needed.
size_t ttref_ir(void* p, char* buf, size_t cap) {
    auto* hg = static_cast<HGraph*>(p);
    std::string s = IRPrinter::to_string(hg->g);
    if (buf && cap) {
        size_t n = std::min(cap - 1, s.size());
        std::memcpy(buf, s.data(), n);
        buf[n] = '\0';
    }
    return s.size() + 1;
}

// mode: 0 interpreted, 1 scalar, 2 avx2 (host ISA), 3 avx2_fma, 4 avx2_nofma,
//       5 cuda (only in the integration build)
void* ttref_compile(void* p, int mode, int optimize) {
    auto* hg = static_cast<HGraph*>(p);
    try {
        ExecutionMode m = ExecutionMode::Interpreted;
        switch (mode) {
            case 0: m = ExecutionMode::Interpreted; break;
            case 1: m = ExecutionMode::CompiledScalar; break;
            case 2: m = ExecutionMode::CompiledAVX2; break;
            case 3: m = ExecutionMode::CompiledAVX2_FMA; break;
            case 4: m = ExecutionMode::CompiledAVX2_NoFMA; break;
#ifdef TTREF_WITH_CUDA
            case 5: m = ExecutionMode::CompiledCUDA; break;
#endif
            default: throw std::runtime_error("ttref_compile: unknown mode " + std::to_string(mode));
        }
        auto* he = new HExec();
        he->hg = hg;
        he->ex = std::make_unique<Executor>(hg->g, m, optimize != 0, nullptr);
        return he;
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}

void ttref_exec_free(void* e) { delete static_cast<HExec*>(e); }

static std::unordered_map<const Node*, Tensor> bind(HGraph* hg, const float* const* inputs) {
    std::unordered_map<const Node*, Tensor> feed;
    const auto& ins = hg->g.inputs();
    for (size_t i = 0; i < ins.size(); ++i) {
        Tensor t(ins[i]->shape(), DType::Float32);
        std::memcpy(t.raw_data(), inputs[i], t.nbytes());
        feed[ins[i]] = t;
    }
    return feed;
}

// Runs the compiled program once.  inputs follow graph-input order, outputs
// graph-output order; every output buffer holds numel floats of that output.
int ttref_run(void* e, const float* const* inputs, float* const* outputs) {
    auto* he = static_cast<HExec*>(e);
    return guarded([&] {
        auto feed = bind(he->hg, inputs);
        std::vector<Tensor> outs = he->ex->run(feed);
        for (size_t i = 0; i < outs.size(); ++i) {
            Tensor c = outs[i].contiguous();
            std::memcpy(outputs[i], c.raw_data(), c.nbytes());
        }
        return 0;
    });
}

// Binds inputs once, then runs `reps` times; returns the seconds spent inside
// Executor::run (input copies excluded), or a negative value on error.
double ttref_time_runs(void* e, const float* const* inputs, int reps) {
    auto* he = static_cast<HExec*>(e);
    try {
        auto feed = bind(he->hg, inputs);
        auto t0 = std::chrono::steady_clock::now();
        for (int r = 0; r < reps; ++r) {
            std::vector<Tensor> outs = he->ex->run(feed);
            (void)outs;
        }
        auto t1 = std::chrono::steady_clock::now();
        return std::chrono::duration<double>(t1 - t0).count();
    } catch (const std::exception& ex) {
        g_err = ex.what();
        return -1.0;
    }
}

// Eager reverse-mode gradients (Autodiff::compute_gradients) of `loss` with
// respect to nodes `wrt`; grads[i] receives numel(wrt[i]) floats.
int ttref_gradients(void* p, int loss, const float* const* inputs, const int* wrt, int nwrt,
                    float* const* grads) {
    auto* hg = static_cast<HGraph*>(p);
    return guarded([&] {
        auto feed = bind(hg, inputs);
        auto gr = Autodiff::compute_gradients(hg->g, hg->nodes.at(static_cast<size_t>(loss)), feed);
        for (int i = 0; i < nwrt; ++i) {
            const Node* n = hg->nodes.at(static_cast<size_t>(wrt[i]));
            auto it = gr.find(n);
            if (it == gr.end()) throw std::runtime_error("no gradient reached node " + std::to_string(wrt[i]));
            Tensor c = it->second.contiguous();
            std::memcpy(grads[i], c.raw_data(), c.nbytes());
        }
        return 0;
    });
}

// Same as ttref_gradients, timed: seconds for `reps` calls of compute_gradients.
double ttref_time_gradients(void* p, int loss, const float* const* inputs, int reps) {
    auto* hg = static_cast<HGraph*>(p);
    try {
        auto feed = bind(hg, inputs);
        const Node* l = hg->nodes.at(static_cast<size_t>(loss));
        auto t0 = std::chrono::steady_clock::now();
        for (int r = 0; r < reps; ++r) {
            auto gr = Autodiff::compute_gradients(hg->g, l, feed);
            (void)gr;
        }
        auto t1 = std::chrono::steady_clock::now();
        return std::chrono::duration<double>(t1 - t0).count();
    } catch (const std::exception& ex) {
        g_err = ex.what();
        return -1.0;
    }
}

#ifdef TTREF_WITH_CUDA
int ttref_has_cuda() { return 1; }

// Executor::execution_plan / generated_source text (what = 0 plan, 1 source).
size_t ttref_exec_text(void* e, int what, char* buf, size_t cap) {
    auto* he = static_cast<HExec*>(e);
    const std::string s = what == 0 ? he->ex->execution_plan() : he->ex->generated_source();
    if (buf && cap) {
        const size_t n = s.size() < cap - 1 ? s.size() : cap - 1;
        std::memcpy(buf, s.data(), n);
        buf[n] = '\0';
    }
    return s.size() + 1;
}

// Device-resident run: the inputs are copied to device tensors once, Executor::run
// takes them (no host staging) and returns device tensors, which are copied back here.
// With e2 (may be NULL) the first executor's outputs feed the second one's inputs in
// order, still on the device, and `outputs` receives the second one's results.
// Returns 0, or -1 with the error text (also when an output is not a device tensor).
int ttref_run_device(void* e, void* e2, const float* const* inputs, float* const* outputs) {
    auto* he = static_cast<HExec*>(e);
    return guarded([&] {
        std::unordered_map<const Node*, Tensor> feed;
        const auto& ins = he->hg->g.inputs();
        for (size_t i = 0; i < ins.size(); ++i) {
            Tensor t(ins[i]->shape(), DType::Float32);
            std::memcpy(t.raw_data(), inputs[i], t.nbytes());
            feed[ins[i]] = cuda_to_device(t);
        }
        std::vector<Tensor> outs = he->ex->run(feed);
        if (e2) {
            auto* h2 = static_cast<HExec*>(e2);
            const auto& ins2 = h2->hg->g.inputs();
            if (ins2.size() != outs.size()) throw std::runtime_error("chain: output/input count mismatch");
            std::unordered_map<const Node*, Tensor> feed2;
            for (size_t i = 0; i < ins2.size(); ++i) {
                if (!cuda_is_device(outs[i])) throw std::runtime_error("chain: an output is not on the device");
                feed2[ins2[i]] = outs[i];
            }
            outs = h2->ex->run(feed2);
        }
        for (size_t i = 0; i < outs.size(); ++i) {
            if (!cuda_is_device(outs[i])) throw std::runtime_error("output " + std::to_string(i) + " is not on the device");
            Tensor c = cuda_to_host(outs[i]);
            std::memcpy(outputs[i], c.raw_data(), c.nbytes());
        }
        return 0;
    });
}
#endif

}  // extern "C"
