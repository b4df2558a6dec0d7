// nccl_wrappers.cu -- libncclwrap: the reference's 15 ncw* entry points
// (csrc/nccl_wrappers.h:47-61) over NCCL, plus the expert-parallel pieces the
// MoE layer needs: a variable all-to-all built from grouped send/recv (NCCL
// 2.27 has no all-to-all), a bounded communicator init and an async-error
// watchdog that aborts a communicator instead of letting a rank hang.
//
// The FP8 datatypes map to NCCL's ncclFloat8e4m3 / ncclFloat8e5m2 (the names
// NCCL >= 2.24 uses; the reference's ncclFp8E4M3 spelling does not compile
// against NCCL 2.27, csrc/nccl_wrappers.cu:31-32).
#include <nccl.h>
#include <cuda_runtime.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <thread>

#include "nccl_wrappers.h"

namespace {

ncwResult_t to_ncw(ncclResult_t e) {
    switch (e) {
        case ncclSuccess: return NCW_SUCCESS;
        case ncclUnhandledCudaError: return NCW_ERROR_UNHANDLED;
        case ncclSystemError: return NCW_ERROR_SYSTEM;
        case ncclInternalError: return NCW_ERROR_INTERNAL;
        case ncclInvalidArgument: return NCW_ERROR_INVALID_ARGUMENT;
        case ncclInvalidUsage: return NCW_ERROR_INVALID_USAGE;
        default: return NCW_ERROR_INTERNAL;
    }
}

ncwResult_t report(ncclResult_t e, const char* what) {
    if (e != ncclSuccess && e != ncclInProgress) std::fprintf(stderr, "%s failed: %s\n", what, ncclGetErrorString(e));
    return e == ncclInProgress ? NCW_SUCCESS : to_ncw(e);
}

ncclDataType_t dt(ncwDataType_t t) {
    switch (t) {
        case NCW_INT8: return ncclInt8;
        case NCW_UINT8: return ncclUint8;
        case NCW_INT32: return ncclInt32;
        case NCW_UINT32: return ncclUint32;
        case NCW_INT64: return ncclInt64;
        case NCW_UINT64: return ncclUint64;
        case NCW_FLOAT16: return ncclFloat16;
        case NCW_FLOAT64: return ncclFloat64;
        case NCW_BFLOAT16: return ncclBfloat16;
        case NCW_FP8_E4M3: return ncclFloat8e4m3;
        case NCW_FP8_E5M2: return ncclFloat8e5m2;
        default: return ncclFloat32;
    }
}

size_t dt_size(ncwDataType_t t) {
    switch (t) {
        case NCW_INT8: case NCW_UINT8: case NCW_FP8_E4M3: case NCW_FP8_E5M2: return 1;
        case NCW_FLOAT16: case NCW_BFLOAT16: return 2;
        case NCW_INT64: case NCW_UINT64: case NCW_FLOAT64: return 8;
        default: return 4;
    }
}

ncclRedOp_t rop(ncwReduceOp_t o) {
    switch (o) {
        case NCW_PROD: return ncclProd;
        case NCW_MAX: return ncclMax;
        case NCW_MIN: return ncclMin;
        case NCW_AVG: return ncclAvg;
        default: return ncclSum;
    }
}

inline ncclComm_t C(ncwComm_t c) { return static_cast<ncclComm_t>(c); }
inline cudaStream_t S(cwStream_t s) { return static_cast<cudaStream_t>(s); }

// A non-blocking communicator (ncwCommInitRankTimeout) may answer a call with
// ncclInProgress while it is still enqueueing; the next call on it must wait
// until the state settles.  Bounded: after 60 s the communicator is aborted.
ncclResult_t settle(ncclComm_t comm, ncclResult_t e) {
    if (e != ncclInProgress) return e;
    const auto t0 = std::chrono::steady_clock::now();
    ncclResult_t st = ncclInProgress;
    while (true) {
        const ncclResult_t q = ncclCommGetAsyncError(comm, &st);
        if (q != ncclSuccess) return q;
        if (st != ncclInProgress) return st;
        if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(60)) {
            ncclCommAbort(comm);
            return ncclSystemError;
        }
        std::this_thread::yield();
    }
}

}  // namespace

extern "C" {

ncwResult_t ncwGetUniqueId(ncwUniqueId* uniqueId) {
    static_assert(sizeof(ncclUniqueId) == sizeof(ncwUniqueId), "unique id size");
    ncclUniqueId id;
    ncclResult_t e = ncclGetUniqueId(&id);
    if (e == ncclSuccess) std::memcpy(uniqueId->internal, id.internal, sizeof(id.internal));
    return report(e, "ncclGetUniqueId");
}

ncwResult_t ncwCommInitRank(ncwComm_t* comm, int nranks, ncwUniqueId uniqueId, int rank) {
    ncclUniqueId id;
    std::memcpy(id.internal, uniqueId.internal, sizeof(id.internal));
    ncclComm_t c = nullptr;
    ncclResult_t e = ncclCommInitRank(&c, nranks, id, rank);
    *comm = (e == ncclSuccess) ? static_cast<ncwComm_t>(c) : nullptr;
    return report(e, "ncclCommInitRank");
}

ncwResult_t ncwCommDestroy(ncwComm_t comm) {
    if (!comm) return NCW_SUCCESS;
    return report(ncclCommDestroy(C(comm)), "ncclCommDestroy");
}

ncwResult_t ncwCommCount(ncwComm_t comm, int* count) { return to_ncw(ncclCommCount(C(comm), count)); }
ncwResult_t ncwCommUserRank(ncwComm_t comm, int* rank) { return to_ncw(ncclCommUserRank(C(comm), rank)); }

ncwResult_t ncwAllReduce(const void* sendbuff, void* recvbuff, size_t count, ncwDataType_t datatype, ncwReduceOp_t op,
                         ncwComm_t comm, cwStream_t stream) {
    return report(ncclAllReduce(sendbuff, recvbuff, count, dt(datatype), rop(op), C(comm), S(stream)), "ncclAllReduce");
}

ncwResult_t ncwBroadcast(const void* sendbuff, void* recvbuff, size_t count, ncwDataType_t datatype, int root,
                         ncwComm_t comm, cwStream_t stream) {
    return report(ncclBroadcast(sendbuff, recvbuff, count, dt(datatype), root, C(comm), S(stream)), "ncclBroadcast");
}

ncwResult_t ncwReduce(const void* sendbuff, void* recvbuff, size_t count, ncwDataType_t datatype, ncwReduceOp_t op,
                      int root, ncwComm_t comm, cwStream_t stream) {
    return report(ncclReduce(sendbuff, recvbuff, count, dt(datatype), rop(op), root, C(comm), S(stream)), "ncclReduce");
}

ncwResult_t ncwAllGather(const void* sendbuff, void* recvbuff, size_t sendcount, ncwDataType_t datatype, ncwComm_t comm,
                         cwStream_t stream) {
    return report(ncclAllGather(sendbuff, recvbuff, sendcount, dt(datatype), C(comm), S(stream)), "ncclAllGather");
}

ncwResult_t ncwReduceScatter(const void* sendbuff, void* recvbuff, size_t recvcount, ncwDataType_t datatype,
                             ncwReduceOp_t op, ncwComm_t comm, cwStream_t stream) {
    return report(ncclReduceScatter(sendbuff, recvbuff, recvcount, dt(datatype), rop(op), C(comm), S(stream)),
                  "ncclReduceScatter");
}

ncwResult_t ncwSend(const void* sendbuff, size_t count, ncwDataType_t datatype, int peer, ncwComm_t comm, cwStream_t stream) {
    return report(ncclSend(sendbuff, count, dt(datatype), peer, C(comm), S(stream)), "ncclSend");
}

ncwResult_t ncwRecv(void* recvbuff, size_t count, ncwDataType_t datatype, int peer, ncwComm_t comm, cwStream_t stream) {
    return report(ncclRecv(recvbuff, count, dt(datatype), peer, C(comm), S(stream)), "ncclRecv");
}

ncwResult_t ncwGroupStart(void) { return to_ncw(ncclGroupStart()); }
ncwResult_t ncwGroupEnd(void) { return report(ncclGroupEnd(), "ncclGroupEnd"); }

const char* ncwGetErrorString(ncwResult_t result) {
    switch (result) {
        case NCW_SUCCESS: return "Success";
        case NCW_ERROR_UNHANDLED: return "Unhandled CUDA error";
        case NCW_ERROR_SYSTEM: return "System error";
        case NCW_ERROR_INTERNAL: return "Internal error";
        case NCW_ERROR_INVALID_ARGUMENT: return "Invalid argument";
        case NCW_ERROR_INVALID_USAGE: return "Invalid usage";
        default: return "Unknown error";
    }
}

ncwResult_t ncwAllToAllv(const void* sendbuff, const size_t* send_counts, const size_t* send_offsets, void* recvbuff,
                         const size_t* recv_counts, const size_t* recv_offsets, ncwDataType_t datatype, ncwComm_t comm,
                         cwStream_t stream) {
    int n = 0, me = 0;
    ncclResult_t e = ncclCommCount(C(comm), &n);
    if (e != ncclSuccess) return to_ncw(e);
    e = ncclCommUserRank(C(comm), &me);
    if (e != ncclSuccess) return to_ncw(e);
    const size_t es = dt_size(datatype);
    const ncclDataType_t t = dt(datatype);
    const char* sb = static_cast<const char*>(sendbuff);
    char* rb = static_cast<char*>(recvbuff);
    if (send_counts[me] != recv_counts[me]) return NCW_ERROR_INVALID_ARGUMENT;
    if (send_counts[me]) {
        if (cudaMemcpyAsync(rb + recv_offsets[me] * es, sb + send_offsets[me] * es, send_counts[me] * es,
                            cudaMemcpyDeviceToDevice, S(stream)) != cudaSuccess)
            return NCW_ERROR_UNHANDLED;
    }
    e = ncclGroupStart();
    if (e != ncclSuccess) return to_ncw(e);
    for (int p = 0; p < n; ++p) {
        if (p == me) continue;
        if (send_counts[p]) {
            e = ncclSend(sb + send_offsets[p] * es, send_counts[p], t, p, C(comm), S(stream));
            if (e != ncclSuccess && e != ncclInProgress) break;
        }
        if (recv_counts[p]) {
            e = ncclRecv(rb + recv_offsets[p] * es, recv_counts[p], t, p, C(comm), S(stream));
            if (e != ncclSuccess && e != ncclInProgress) break;
        }
    }
    ncclResult_t e2 = settle(C(comm), ncclGroupEnd());
    if (e != ncclSuccess && e != ncclInProgress) return report(e, "ncwAllToAllv send/recv");
    return report(e2, "ncwAllToAllv group");
}

ncwResult_t ncwCommInitRankTimeout(ncwComm_t* comm, int nranks, ncwUniqueId uniqueId, int rank, int timeout_ms) {
    ncclUniqueId id;
    std::memcpy(id.internal, uniqueId.internal, sizeof(id.internal));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclComm_t c = nullptr;
    ncclResult_t e = ncclCommInitRankConfig(&c, nranks, id, rank, &cfg);
    *comm = nullptr;
    if (e != ncclSuccess && e != ncclInProgress) return report(e, "ncclCommInitRankConfig");
    const auto t0 = std::chrono::steady_clock::now();
    ncclResult_t st = ncclInProgress;
    while (true) {
        ncclResult_t q = ncclCommGetAsyncError(c, &st);
        if (q != ncclSuccess) { st = q; break; }
        if (st != ncclInProgress) break;
        if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
            ncclCommAbort(c);
            std::fprintf(stderr, "ncwCommInitRankTimeout: peers did not join within %d ms\n", timeout_ms);
            return NCW_ERROR_SYSTEM;
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
    if (st != ncclSuccess) {
        ncclCommAbort(c);
        return report(st, "ncclCommInitRankConfig (async)");
    }
    *comm = static_cast<ncwComm_t>(c);
    return NCW_SUCCESS;
}

ncwResult_t ncwCommGetAsyncError(ncwComm_t comm) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t e = ncclCommGetAsyncError(C(comm), &st);
    if (e != ncclSuccess) return to_ncw(e);
    return st == ncclInProgress ? NCW_SUCCESS : to_ncw(st);
}

ncwResult_t ncwCommAbort(ncwComm_t comm) {
    if (!comm) return NCW_SUCCESS;
    return to_ncw(ncclCommAbort(C(comm)));
}

ncwResult_t ncwStreamSynchronizeTimeout(ncwComm_t comm, cwStream_t stream, int timeout_ms) {
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        cudaError_t q = cudaStreamQuery(S(stream));
        if (q == cudaSuccess) return NCW_SUCCESS;
        if (q != cudaErrorNotReady) return NCW_ERROR_UNHANDLED;
        if (comm) {
            ncclResult_t st = ncclSuccess;
            if (ncclCommGetAsyncError(C(comm), &st) == ncclSuccess && st != ncclSuccess && st != ncclInProgress) {
                ncclCommAbort(C(comm));
                std::fprintf(stderr, "ncwStreamSynchronizeTimeout: NCCL async error %s\n", ncclGetErrorString(st));
                return NCW_ERROR_SYSTEM;
            }
        }
        if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
            if (comm) ncclCommAbort(C(comm));
            std::fprintf(stderr, "ncwStreamSynchronizeTimeout: no progress within %d ms\n", timeout_ms);
            return NCW_ERROR_SYSTEM;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

}  // extern "C"
