// Data-parallel gradient exchange: one NCCL communicator per process/GPU, an
// in-place float32 sum all-reduce over NVLink / NVSwitch.  The reference has no
// distributed code; the batch-sharded training step (rank r owns rows
// [r*B/N, (r+1)*B/N) of the global batch) sums the per-rank gradients here and
// folds 1/N into the SGD learning rate, so every replica applies the same update.
//
// Communicators are created non-blocking (ncclConfig_t.blocking = 0) and every wait
// polls ncclCommGetAsyncError against a deadline, so a missing peer ends in an
// error (and ncclCommAbort) instead of a hang.
//
// NCCL is bound at the first call, not at load time: the library resolves its entry
// points from the libnccl.so.2 already loaded in the process (e.g. PyTorch's, which
// may be newer than the system one), else loads libnccl.so.2 itself.  Linking NCCL
// directly would pin whichever copy loads first and break a later `import torch`
// whose libtorch_cuda.so needs symbols of its own, newer NCCL.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

#include "ttb.hpp"

struct tt_dp {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1, device = 0;
};

namespace {

int dp_fail(int st, const std::string& m) { return ttb::record_error(st, m); }

struct NcclApi {
    decltype(&::ncclGetUniqueId) GetUniqueId = nullptr;
    decltype(&::ncclCommInitRankConfig) CommInitRankConfig = nullptr;
    decltype(&::ncclCommGetAsyncError) CommGetAsyncError = nullptr;
    decltype(&::ncclAllReduce) AllReduce = nullptr;
    decltype(&::ncclCommAbort) CommAbort = nullptr;
    decltype(&::ncclCommFinalize) CommFinalize = nullptr;
    decltype(&::ncclCommDestroy) CommDestroy = nullptr;
    decltype(&::ncclGetErrorString) GetErrorString = nullptr;
    std::string error;  // empty when every entry point resolved
};

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) {
            const char* e = dlerror();
            api.error = std::string("cannot load libnccl.so.2: ") + (e ? e : "unknown");
            return;
        }
        auto sym = [&](const char* name, auto& fn) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            if (!fn && api.error.empty()) api.error = std::string("libnccl.so.2 lacks ") + name;
        };
        sym("ncclGetUniqueId", api.GetUniqueId);
        sym("ncclCommInitRankConfig", api.CommInitRankConfig);
        sym("ncclCommGetAsyncError", api.CommGetAsyncError);
        sym("ncclAllReduce", api.AllReduce);
        sym("ncclCommAbort", api.CommAbort);
        sym("ncclCommFinalize", api.CommFinalize);
        sym("ncclCommDestroy", api.CommDestroy);
        sym("ncclGetErrorString", api.GetErrorString);
    });
    return api;
}

// The resolved API, or nullptr after recording why NCCL is unavailable.
const NcclApi* nccl_or_fail() {
    const NcclApi& a = nccl();
    if (!a.error.empty()) {
        dp_fail(TT_ERR_COMM, a.error);
        return nullptr;
    }
    return &a;
}

// Waits for a non-blocking communicator to leave ncclInProgress, up to `seconds`.
ncclResult_t wait_comm(ncclComm_t comm, double seconds) {
    auto t0 = std::chrono::steady_clock::now();
    ncclResult_t state = ncclInProgress;
    while (true) {
        ncclResult_t r = nccl().CommGetAsyncError(comm, &state);
        if (r != ncclSuccess) return r;
        if (state != ncclInProgress) return state;
        double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (el > seconds) return ncclInProgress;
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

}  // namespace

extern "C" {

int tt_dp_unique_id(char* id_out) {
    if (!id_out) return TT_ERR_INVALID;
    const NcclApi* api = nccl_or_fail();
    if (!api) return TT_ERR_COMM;
    ncclUniqueId id;
    ncclResult_t r = api->GetUniqueId(&id);
    if (r != ncclSuccess) return dp_fail(TT_ERR_COMM, std::string("ncclGetUniqueId: ") + api->GetErrorString(r));
    static_assert(sizeof(id.internal) == TT_DP_ID_BYTES, "NCCL unique id size");
    std::memcpy(id_out, id.internal, TT_DP_ID_BYTES);
    return TT_OK;
}

int tt_dp_init(int32_t rank, int32_t world, const char* id_bytes, int32_t device, tt_dp** out) {
    if (!out || !id_bytes || world < 1 || rank < 0 || rank >= world) return TT_ERR_INVALID;
    *out = nullptr;
    const NcclApi* api = nccl_or_fail();
    if (!api) return TT_ERR_COMM;
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        return dp_fail(TT_ERR_NO_DEVICE, "cudaSetDevice failed");
    }
    ncclUniqueId id;
    std::memcpy(id.internal, id_bytes, TT_DP_ID_BYTES);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    auto* dp = new tt_dp();
    dp->rank = rank;
    dp->world = world;
    dp->device = device;
    ncclResult_t r = api->CommInitRankConfig(&dp->comm, world, id, rank, &cfg);
    if (r == ncclInProgress || r == ncclSuccess) r = wait_comm(dp->comm, 120.0);
    if (r != ncclSuccess) {
        if (dp->comm) api->CommAbort(dp->comm);
        delete dp;
        return dp_fail(TT_ERR_COMM, std::string("ncclCommInitRankConfig: ") +
                                        (r == ncclInProgress ? "timed out" : api->GetErrorString(r)));
    }
    *out = dp;
    return TT_OK;
}

int tt_dp_allreduce_sum(tt_dp* dp, float* buf, size_t count, void* stream) {
    if (!dp || (!buf && count)) return TT_ERR_INVALID;
    if (dp->world == 1 || count == 0) return TT_OK;
    if (!dp->comm) return dp_fail(TT_ERR_COMM, "communicator was aborted by an earlier error");
    const NcclApi& api = nccl();
    ncclResult_t r = api.AllReduce(buf, buf, count, ncclFloat32, ncclSum, dp->comm, static_cast<cudaStream_t>(stream));
    if (r == ncclInProgress) r = wait_comm(dp->comm, 120.0);
    if (r != ncclSuccess) {
        api.CommAbort(dp->comm);
        dp->comm = nullptr;
        return dp_fail(TT_ERR_COMM, std::string("ncclAllReduce: ") +
                                        (r == ncclInProgress ? "enqueue timed out" : api.GetErrorString(r)));
    }
    return TT_OK;
}

int tt_dp_destroy(tt_dp* dp) {
    if (!dp) return TT_OK;
    if (dp->comm) {
        const NcclApi& api = nccl();
        cudaSetDevice(dp->device);
        api.CommFinalize(dp->comm);
        wait_comm(dp->comm, 60.0);
        api.CommDestroy(dp->comm);
    }
    delete dp;
    return TT_OK;
}

}  // extern "C"

