// tcgen05 / TMEM 3xTF32 GEMM for sm_100a (placeholder until the tensor-core kernel lands).
#include <cuda_runtime.h>

#include "program.hpp"

namespace ttb {

bool gemm_tc_supported(const GemmDesc&) { return false; }

int launch_gemm_tc(const GemmDesc&, const float*, const float*, float*, int*, void*) {
    return static_cast<int>(cudaErrorNotSupported);
}

}  // namespace ttb
