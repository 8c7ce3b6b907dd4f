// NVRTC compilation, kernel cache and driver entry points (see jit.cpp).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include <string>
#include <vector>

#include "ttb.hpp"

namespace ttb {

struct Driver {
    PFN_cuModuleLoadData_v2000 moduleLoadData;
    PFN_cuModuleGetFunction_v2000 moduleGetFunction;
    PFN_cuModuleUnload_v2000 moduleUnload;
    PFN_cuLaunchKernel_v4000 launchKernel;
    PFN_cuTensorMapEncodeTiled_v12000 tensorMapEncodeTiled;
    PFN_cuGetErrorString_v6000 getErrorString;
};
const Driver& driver();
std::string cu_error(CUresult r);

struct LoadedModule {
    CUmodule module = nullptr;
    std::vector<CUfunction> functions;
    std::string cubin_path;
    bool from_cache = false;
};

std::string nvrtc_info();
std::string nvrtc_compile(const std::string& source);
std::string cache_key(const std::string& canonical_ir, const std::string& metadata);
LoadedModule load_program_module(const std::string& key, const std::string& source, const std::string& cache_dir,
                                 const std::vector<std::string>& kernels);
// Host-only: compiles (or finds) the cubin in the cache without loading it; returns
// its path ("" without a cache directory).
std::string compile_to_cache(const std::string& key, const std::string& source, const std::string& cache_dir);
uint64_t cache_hits();
uint64_t cache_misses();

}  // namespace ttb
