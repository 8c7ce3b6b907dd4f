// Data-parallel gradient exchange: one NCCL communicator per process/GPU, an
// in-place float32 sum all-reduce over NVLink / NVSwitch.  The reference has no
// distributed code; the batch-sharded training step (rank r owns rows
// [r*B/N, (r+1)*B/N) of the global batch) sums the per-rank gradients here and
// folds 1/N into the SGD learning rate, so every replica applies the same update.
//
// Communicators are created non-blocking (ncclConfig_t.blocking = 0) and every wait
// polls ncclCommGetAsyncError against a deadline, so a missing peer ends in an
// error (and ncclCommAbort) instead of a hang.
#include <cuda_runtime.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <string>
#include <thread>

#include "ttb.hpp"

struct tt_dp {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1, device = 0;
};

namespace {

int dp_fail(int st, const std::string& m) { return ttb::record_error(st, m); }

// Waits for a non-blocking communicator to leave ncclInProgress, up to `seconds`.
ncclResult_t wait_comm(ncclComm_t comm, double seconds) {
    auto t0 = std::chrono::steady_clock::now();
    ncclResult_t state = ncclInProgress;
    while (true) {
        ncclResult_t r = ncclCommGetAsyncError(comm, &state);
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
    ncclUniqueId id;
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) return dp_fail(TT_ERR_COMM, std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
    static_assert(sizeof(id.internal) == TT_DP_ID_BYTES, "NCCL unique id size");
    std::memcpy(id_out, id.internal, TT_DP_ID_BYTES);
    return TT_OK;
}

int tt_dp_init(int32_t rank, int32_t world, const char* id_bytes, int32_t device, tt_dp** out) {
    if (!out || !id_bytes || world < 1 || rank < 0 || rank >= world) return TT_ERR_INVALID;
    *out = nullptr;
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
    ncclResult_t r = ncclCommInitRankConfig(&dp->comm, world, id, rank, &cfg);
    if (r == ncclInProgress || r == ncclSuccess) r = wait_comm(dp->comm, 120.0);
    if (r != ncclSuccess) {
        if (dp->comm) ncclCommAbort(dp->comm);
        delete dp;
        return dp_fail(TT_ERR_COMM, std::string("ncclCommInitRankConfig: ") +
                                        (r == ncclInProgress ? "timed out" : ncclGetErrorString(r)));
    }
    *out = dp;
    return TT_OK;
}

int tt_dp_allreduce_sum(tt_dp* dp, float* buf, size_t count, void* stream) {
    if (!dp || (!buf && count)) return TT_ERR_INVALID;
    if (dp->world == 1 || count == 0) return TT_OK;
    ncclResult_t r = ncclAllReduce(buf, buf, count, ncclFloat32, ncclSum, dp->comm, static_cast<cudaStream_t>(stream));
    if (r == ncclInProgress) r = wait_comm(dp->comm, 120.0);
    if (r != ncclSuccess) {
        ncclCommAbort(dp->comm);
        dp->comm = nullptr;
        return dp_fail(TT_ERR_COMM, std::string("ncclAllReduce: ") +
                                        (r == ncclInProgress ? "enqueue timed out" : ncclGetErrorString(r)));
    }
    return TT_OK;
}

int tt_dp_destroy(tt_dp* dp) {
    if (!dp) return TT_OK;
    if (dp->comm) {
        cudaSetDevice(dp->device);
        ncclCommFinalize(dp->comm);
        wait_comm(dp->comm, 60.0);
        ncclCommDestroy(dp->comm);
    }
    delete dp;
    return TT_OK;
}

}  // extern "C"

