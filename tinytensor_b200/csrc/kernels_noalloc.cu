// tt_gemm_f32_noalloc: the fp32-accurate GEMM for callers that cannot allocate device
// memory.  Some callers cannot call cudaMalloc at all: code that must not touch the
// device allocator (it would synchronise the device or break a caller-managed memory
// budget), plug-in hosts that hand the library only the buffers of one call, or work
// queued while another component owns allocation.  This entry point takes device
// pointers for A, B and C and performs no allocation of any kind: its scratch (the
// hi/lo operand copies of the 3xTF32 split and the split-K partials) lives in the
// file-scope array below, which every GPU that loads the library holds until exit.
//
// Limits and behaviour:
//  - scratch capacity TT_NOALLOC_SCRATCH_BYTES (32 MiB); products whose plan needs more
//    are rejected with TT_ERR_MEMORY and a message naming the need and the capacity;
//  - the first call on a device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current).  Under lazy module loading that
//    lookup is also what loads this module and reserves the array, and the GEMM kernels
//    load on their first launch, so the first call on each device can itself need
//    device memory: make it once as a warm-up, outside any no-allocation window and
//    before any stream capture.  The address is cached only once a lookup succeeds, so a
//    failed first attempt can be retried;
//  - every call shares the one array, which keeps the previous call's contents.  All
//    of it is rewritten before it is read, except the status word, which each call
//    clears on its stream.  Calls whose work overlaps on the GPU (other streams, or
//    other host threads) race on the array: order them on one stream;
//  - device_status NULL: a bounded wait that gives up inside the tensor-core kernels
//    records its code in an internal word that nothing reports, so the call still
//    returns TT_OK with C partly written.  Callers that need to detect that pass their
//    own zeroed device int and check it after synchronising the stream.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "program.hpp"

#define TT_NOALLOC_SCRATCH_BYTES (32u << 20)
#define TT_NOALLOC_STATUS_BYTES 256u

namespace {

// Scratch for every call of tt_gemm_f32_noalloc on this device, then the status word.
static __device__ __align__(256) unsigned char g_noalloc_scratch[TT_NOALLOC_SCRATCH_BYTES + TT_NOALLOC_STATUS_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices];  // non-null once a lookup on that device succeeded

// Device address of the scratch array on the current device `dev` (looked up once).
cudaError_t scratch_address(int dev, void** out) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_addr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            return e != cudaSuccess ? e : cudaErrorInvalidSymbol;
        }
        g_addr[dev] = p;
    }
    *out = g_addr[dev];
    return cudaSuccess;
}

}  // namespace

extern "C" int tt_gemm_f32_noalloc(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                                   int32_t* device_status, void* stream) {
    using namespace ttb;
    if (M < 0 || N < 0 || K < 0) return record_error(TT_ERR_INVALID, "tt_gemm_f32_noalloc: negative dimension");
    // Operands are only dereferenced when they hold elements.
    if ((M > 0 && N > 0 && !C) || (M > 0 && K > 0 && !A) || (K > 0 && N > 0 && !B))
        return record_error(TT_ERR_INVALID, "tt_gemm_f32_noalloc: null pointer for a non-empty operand");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return record_error(TT_ERR_NO_DEVICE, "no current CUDA device");
    }
    void* addr = nullptr;
    const cudaError_t se = scratch_address(dev, &addr);
    if (se != cudaSuccess)
        return record_error(TT_ERR_RUNTIME, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(se));
    if (M == 0 || N == 0) return TT_OK;

    GemmDesc d;
    d.M = M;
    d.N = N;
    d.K = K;
    d.a_sm = K;
    d.a_sk = 1;
    d.b_sk = N;
    d.b_sn = 1;
    d.c_sb = M * N;
    plan_gemm(d);
    const int64_t need = gemm_scratch_bytes(d);
    if (need > static_cast<int64_t>(TT_NOALLOC_SCRATCH_BYTES))
        return record_error(TT_ERR_MEMORY, "tt_gemm_f32_noalloc: this " + std::to_string(M) + "x" + std::to_string(N) +
                                               "x" + std::to_string(K) + " product needs " + std::to_string(need) +
                                               " bytes of scratch; the static capacity is " +
                                               std::to_string(TT_NOALLOC_SCRATCH_BYTES));
    char* base = static_cast<char*>(addr);
    int* status = device_status ? device_status : reinterpret_cast<int*>(base + TT_NOALLOC_SCRATCH_BYTES);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (!device_status) {
        cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int), st);
        if (e != cudaSuccess) return record_error(TT_ERR_RUNTIME, std::string("status clear: ") + cudaGetErrorString(e));
    }
    const int rc = launch_gemm(d, A, B, C, base, status, stream);
    if (rc) return record_error(TT_ERR_RUNTIME, std::string("tt_gemm_f32_noalloc: ") +
                                                    cudaGetErrorString(static_cast<cudaError_t>(rc)));
    return TT_OK;
}
