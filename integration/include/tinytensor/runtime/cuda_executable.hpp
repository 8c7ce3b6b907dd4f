#pragma once
// The B200 backend as a TinyTensor execution mode (ExecutionMode::CompiledCUDA).
//
// This header and src/runtime/cuda_executable.cpp are the reference-side code a
// TinyTensor maintainer adds to the reference tree, next to
// include/tinytensor/runtime/executable.hpp; together with integration/executor.patch
// (the enum value and the Executor branch) they are the whole integration.  The
// backend itself is libtt_cuda.so behind include/tt_cuda.h.
//
//   CudaExecutable   what CppBackend::compile + Executable give the other modes
//                    (src/codegen/cpp_backend.cpp:547-823, src/runtime/executable.cpp:7-63):
//                    the graph is handed to tt_compile once, and run() keeps
//                    Executable::run's contract (arity, shape and dtype checks before
//                    any work, outputs allocated per call, synchronous, profiler total).
//   device tensors   a reference Tensor whose Storage is device memory
//                    (include/tinytensor/core/storage.hpp:13-87 has no device kind; the
//                    storage here is a non-owning Storage whose shared_ptr deleter frees
//                    the device allocation).  run() takes them without host copies and
//                    returns its outputs on the device when any input is there, so
//                    chained programs and a device SGD step never round-trip through
//                    the host.  Their data must not be read on the host: cuda_to_host()
//                    copies them back.

#include <memory>
#include <string>
#include <vector>

#include "tinytensor/core/tensor.hpp"
#include "tinytensor/graph/graph.hpp"
#include "tinytensor/runtime/profiler.hpp"

struct tt_program;

namespace tinytensor {

// ---- device-resident tensors ----------------------------------------------------------
// A contiguous float32 tensor in device memory of the current device (uninitialised).
Tensor cuda_empty(const Shape& shape, DType dtype = DType::Float32);
// Copies a host tensor (any strides) into a new device tensor.
Tensor cuda_to_device(const Tensor& host);
// Copies a device tensor back into a new host tensor (host tensors are returned as is).
Tensor cuda_to_host(const Tensor& t);
// True when t's storage is device memory made by cuda_empty / cuda_to_device.
bool cuda_is_device(const Tensor& t) noexcept;

// ---- the executable ------------------------------------------------------------------
class CudaExecutable {
public:
    // Compiles `graph` (already optimised and verified by the Executor) for the B200.
    // cache_dir: the KernelCache directory of the Executor ("" = no disk cache).
    CudaExecutable(const Graph& graph, const std::string& cache_dir, int device = 0);
    ~CudaExecutable();
    CudaExecutable(const CudaExecutable&) = delete;
    CudaExecutable& operator=(const CudaExecutable&) = delete;

    // Executable::run semantics.  Host inputs give host outputs; if any input is a device
    // tensor, host inputs are copied to the device for the call and the outputs are
    // device tensors.
    std::vector<Tensor> run(const std::vector<Tensor>& inputs, Profiler* profiler = nullptr);

    std::string generated_source() const;  // the CUDA translation unit (NVRTC input)
    std::string plan() const;               // launches, fused regions and arena map
    std::string cubin_path() const;         // cached cubin ("" without a cache)

private:
    std::string info(int what) const;
    tt_program* prog_ = nullptr;
    std::vector<Shape> in_shapes_, out_shapes_;
    std::vector<DType> in_dtypes_, out_dtypes_;
};

}  // namespace tinytensor
