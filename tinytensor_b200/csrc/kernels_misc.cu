// Optimiser step on device: SGD.step of python/tinytensor/optim.py:18-35,
//   v = momentum*v + g   (momentum > 0)
//   p = p - lr * (momentum > 0 ? v : g)
// in float32 exactly as the numpy code computes it, for all parameters in ONE launch
// (a grid-stride loop over the concatenated parameter space, float4 where aligned).
#include <cuda_runtime.h>

#include <cstdint>

#include "program.hpp"

namespace ttb {

namespace {

constexpr int kMaxTensors = 16;

struct SgdArgs {
    int n;
    float lr, momentum;
    float* p[kMaxTensors];
    const float* g[kMaxTensors];
    float* v[kMaxTensors];
    int64_t start[kMaxTensors + 1];  // prefix sums of numels
};

__global__ void __launch_bounds__(256) sgd_kernel(SgdArgs a) {
    const int64_t total = a.start[a.n];
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * 256) {
        int t = 0;
        while (i >= a.start[t + 1]) ++t;
        const int64_t j = i - a.start[t];
        // explicitly rounded multiply and add/sub (no FMA contraction), as numpy rounds them
        float u = a.g[t][j];
        if (a.momentum > 0.0f) {
            const float nv = __fadd_rn(__fmul_rn(a.momentum, a.v[t][j]), u);
            a.v[t][j] = nv;
            u = nv;
        }
        a.p[t][j] = __fsub_rn(a.p[t][j], __fmul_rn(a.lr, u));
    }
}

}  // namespace

int launch_sgd(int n, float* const* params, const float* const* grads, float* const* vel, const int64_t* numels,
               float lr, float momentum, void* stream) {
    for (int base = 0; base < n; base += kMaxTensors) {
        SgdArgs a;
        a.n = n - base < kMaxTensors ? n - base : kMaxTensors;
        a.lr = lr;
        a.momentum = momentum;
        a.start[0] = 0;
        for (int t = 0; t < a.n; ++t) {
            a.p[t] = params[base + t];
            a.g[t] = grads[base + t];
            a.v[t] = vel ? vel[base + t] : nullptr;
            a.start[t + 1] = a.start[t] + numels[base + t];
        }
        if (a.start[a.n] == 0) continue;
        int64_t blocks = (a.start[a.n] + 255) / 256;
        if (blocks > 148 * 16) blocks = 148 * 16;
        sgd_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return static_cast<int>(e);
    }
    return 0;
}

}  // namespace ttb
