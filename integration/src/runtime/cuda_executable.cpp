// ExecutionMode::CompiledCUDA: the reference graph handed to libtt_cuda.so (include/tt_cuda.h).
// See include/tinytensor/runtime/cuda_executable.hpp for the contract.
#include "tinytensor/runtime/cuda_executable.hpp"

#include <cstring>
#include <string>
#include <unordered_map>

#include "tinytensor/utils/errors.hpp"
#include "tt_cuda.h"

namespace tinytensor {

namespace {

// tt_status -> the reference exception of the same meaning (errors.hpp:8-66).  The
// library's message already starts with that exception's name, which the exception
// adds again: drop it.
void tt_check(int st) {
    if (st == TT_OK) return;
    std::string m = tt_last_error();
    const size_t colon = m.find(": ");
    if (colon != std::string::npos && colon >= 5 && colon < 32 && m.find(' ') == colon + 1 &&
        m.compare(colon - 5, 5, "Error") == 0)
        m = m.substr(colon + 2);
    switch (st) {
        case TT_ERR_SHAPE: throw ShapeError(m);
        case TT_ERR_DIMENSION: throw DimensionError(m);
        case TT_ERR_BROADCAST: throw BroadcastError(m);
        case TT_ERR_TYPE: throw TypeError(m);
        case TT_ERR_MEMORY: throw MemoryError(m);
        case TT_ERR_IR: throw IRError(m);
        case TT_ERR_COMPILE: throw CompileError(m);
        default: throw RuntimeExecutionError(m);
    }
}

// Deleter of a device Storage: frees the device allocation, then the Storage object
// (which does not own its pointer).  Its type marks device tensors (std::get_deleter).
struct DeviceStorageDeleter {
    void operator()(Storage* s) const noexcept {
        if (s && s->data()) tt_device_free(s->data());
        delete s;
    }
};

StoragePtr device_storage(size_t nbytes) {
    void* p = nullptr;
    if (nbytes > 0) tt_check(tt_device_alloc(nbytes, &p));
    try {
        return StoragePtr(new Storage(p, nbytes, /*owning=*/false), DeviceStorageDeleter{});
    } catch (...) {
        if (p) tt_device_free(p);
        throw;
    }
}

int32_t dtype_code(DType d) { return d == DType::Float64 ? TT_FLOAT64 : TT_FLOAT32; }

}  // namespace

Tensor cuda_empty(const Shape& shape, DType dtype) {
    const size_t nbytes = static_cast<size_t>(shape.numel()) * dtype_size(dtype);
    return Tensor(shape, Strides::compute_contiguous(shape), 0, device_storage(nbytes), dtype);
}

bool cuda_is_device(const Tensor& t) noexcept {
    return t.storage() && std::get_deleter<DeviceStorageDeleter>(t.storage()) != nullptr;
}

Tensor cuda_to_device(const Tensor& host) {
    if (cuda_is_device(host)) return host;
    const Tensor c = host.contiguous();
    Tensor d = cuda_empty(c.shape(), c.dtype());
    if (c.nbytes()) tt_check(tt_memcpy(d.raw_data(), c.raw_data(), c.nbytes(), TT_H2D, nullptr));
    tt_check(tt_stream_sync(nullptr));
    return d;
}

Tensor cuda_to_host(const Tensor& t) {
    if (!cuda_is_device(t)) return t;
    if (!t.is_contiguous()) throw RuntimeExecutionError("cuda_to_host: device tensor views must be contiguous");
    Tensor h(t.shape(), t.dtype());
    if (h.nbytes()) tt_check(tt_memcpy(h.raw_data(), t.raw_data(), h.nbytes(), TT_D2H, nullptr));
    tt_check(tt_stream_sync(nullptr));
    return h;
}

CudaExecutable::CudaExecutable(const Graph& g, const std::string& cache_dir, int device) {
    // Graph -> tt_graph: nodes in topological order, inputs as indices of earlier nodes.
    const std::vector<Node*> topo = g.topological_sort();
    std::unordered_map<const Node*, int32_t> idx;
    std::vector<tt_node> nodes(topo.size());
    std::vector<Tensor> consts;  // contiguous copies of constant values, alive for tt_compile
    for (size_t i = 0; i < topo.size(); ++i) {
        const Node* n = topo[i];
        tt_node& c = nodes[i];
        std::memset(&c, 0, sizeof(c));
        c.op = static_cast<int32_t>(n->op_type());  // tt_op numbers the reference OpType in order
        c.dtype = dtype_code(n->dtype());
        if (n->inputs().size() > TT_MAX_NODE_INPUTS || n->shape().ndim() > TT_MAX_RANK ||
            n->axes().size() > TT_MAX_RANK)
            throw CompileError("CompiledCUDA: node %" + std::to_string(n->id()) + " exceeds the backend's limits");
        c.num_inputs = static_cast<int32_t>(n->inputs().size());
        for (size_t k = 0; k < n->inputs().size(); ++k) c.inputs[k] = idx.at(n->inputs()[k]);
        c.rank = static_cast<int32_t>(n->shape().ndim());
        for (size_t k = 0; k < n->shape().ndim(); ++k) c.shape[k] = n->shape()[k];
        c.id = static_cast<int64_t>(n->id());
        c.dim0 = n->dim0();
        c.dim1 = n->dim1();
        c.num_axes = static_cast<int32_t>(n->axes().size());
        for (size_t k = 0; k < n->axes().size(); ++k) c.axes[k] = n->axes()[k];
        c.keepdims = n->keepdims() ? 1 : 0;
        if (n->is_constant()) {
            consts.push_back(n->constant_value().contiguous());
            c.data = consts.back().raw_data();
        }
        c.name = n->name().c_str();
        c.expr = n->fusion_expression().empty() ? nullptr : n->fusion_expression().c_str();
        idx[n] = static_cast<int32_t>(i);
    }
    std::vector<int32_t> ins, outs;
    for (Node* n : g.inputs()) {
        ins.push_back(idx.at(n));
        in_shapes_.push_back(n->shape());
        in_dtypes_.push_back(n->dtype());
    }
    for (Node* n : g.outputs()) {
        outs.push_back(idx.at(n));
        out_shapes_.push_back(n->shape());
        out_dtypes_.push_back(n->dtype());
    }
    tt_graph cg{static_cast<int32_t>(nodes.size()), nodes.data(), static_cast<int32_t>(ins.size()), ins.data(),
                static_cast<int32_t>(outs.size()), outs.data()};
    tt_compile_options o;
    std::memset(&o, 0, sizeof(o));
    o.optimize = 1;
    o.device = device;
    o.cache_dir = cache_dir.empty() ? nullptr : cache_dir.c_str();
    o.grad_loss = -1;
    tt_check(tt_compile(&cg, &o, &prog_));
}

CudaExecutable::~CudaExecutable() {
    if (prog_) tt_program_destroy(prog_);
}

std::vector<Tensor> CudaExecutable::run(const std::vector<Tensor>& inputs, Profiler* profiler) {
    // the checks of Executable::run (executable.cpp:12-28), before any device work
    if (inputs.size() != in_shapes_.size())
        throw RuntimeExecutionError("Expected " + std::to_string(in_shapes_.size()) + " inputs, but got " +
                                    std::to_string(inputs.size()));
    bool on_device = false;
    for (size_t i = 0; i < inputs.size(); ++i) {
        if (inputs[i].shape() != in_shapes_[i])
            throw ShapeError("Input " + std::to_string(i) + " shape mismatch: expected " + in_shapes_[i].to_string() +
                             " but got " + inputs[i].shape().to_string());
        if (inputs[i].dtype() != in_dtypes_[i]) throw TypeError("Input " + std::to_string(i) + " dtype mismatch");
        on_device = on_device || cuda_is_device(inputs[i]);
    }
    std::vector<Tensor> keep;  // contiguous host copies, or device copies of host inputs
    std::vector<const void*> ip(inputs.size());
    for (size_t i = 0; i < inputs.size(); ++i) {
        const Tensor& t = inputs[i];
        if (on_device) {
            if (cuda_is_device(t)) {
                if (!t.is_contiguous())
                    throw RuntimeExecutionError("Input " + std::to_string(i) + ": device tensor views must be contiguous");
                ip[i] = t.raw_data();
            } else {
                keep.push_back(cuda_to_device(t));
                ip[i] = keep.back().raw_data();
            }
        } else {
            keep.push_back(t.contiguous());
            ip[i] = keep.back().raw_data();
        }
    }
    std::vector<Tensor> outputs;
    outputs.reserve(out_shapes_.size());
    std::vector<void*> op(out_shapes_.size());
    for (size_t i = 0; i < out_shapes_.size(); ++i) {
        outputs.push_back(on_device ? cuda_empty(out_shapes_[i], out_dtypes_[i])
                                    : Tensor::empty(out_shapes_[i], out_dtypes_[i]));
        op[i] = outputs[i].raw_data();
    }
    if (profiler) {
        profiler->clear();
        profiler->start_timer();
    }
    if (on_device) {
        tt_check(tt_program_run(prog_, ip.data(), op.data(), TT_DEVICE, nullptr));
        int32_t status = 0;
        tt_check(tt_program_status(prog_, &status));  // synchronises: the call stays synchronous
    } else {
        tt_check(tt_program_run(prog_, ip.data(), op.data(), TT_HOST, nullptr));
    }
    if (profiler) profiler->stop_timer();
    return outputs;
}

std::string CudaExecutable::info(int what) const {
    size_t need = 0;
    tt_check(tt_program_info(prog_, what, nullptr, 0, &need));
    std::string s(need, '\0');
    tt_check(tt_program_info(prog_, what, s.data(), need, &need));
    s.resize(need ? need - 1 : 0);
    return s;
}

std::string CudaExecutable::generated_source() const { return info(TT_INFO_SOURCE); }
std::string CudaExecutable::plan() const { return info(TT_INFO_PLAN); }
std::string CudaExecutable::cubin_path() const { return info(TT_INFO_CUBIN_PATH); }

}  // namespace tinytensor
