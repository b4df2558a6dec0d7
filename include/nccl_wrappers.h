/*
 * nccl_wrappers.h -- collective shim (libncclwrap.so), drop-in for the
 * reference engine's csrc/nccl_wrappers.h.
 *
 * The 15 ncw* entry points, the enums and the 128-byte by-value unique id
 * are kept as the reference declares them (csrc/nccl_wrappers.h:12-61).
 * The reference declares them but never calls them from the engine; here they
 * carry the expert-parallel exchange (NCCL over NVLink).
 *
 * New: ncwAllToAllv (grouped send/recv, NCCL 2.27 has no all-to-all), the
 * counts exchange used by the EP MoE layer, and abort/async-error helpers.
 */
#ifndef NCCL_WRAPPERS_H
#define NCCL_WRAPPERS_H

#include <stdint.h>
#include <stddef.h>
#include "cuda_wrappers.h"

#ifdef __cplusplus
extern "C" {
#endif

/* csrc/nccl_wrappers.h:12-19 */
typedef enum {
    NCW_SUCCESS = 0,
    NCW_ERROR_UNHANDLED = 1,
    NCW_ERROR_SYSTEM = 2,
    NCW_ERROR_INTERNAL = 3,
    NCW_ERROR_INVALID_ARGUMENT = 4,
    NCW_ERROR_INVALID_USAGE = 5
} ncwResult_t;

/* csrc/nccl_wrappers.h:21-34 */
typedef enum {
    NCW_INT8 = 0,
    NCW_UINT8 = 1,
    NCW_INT32 = 2,
    NCW_UINT32 = 3,
    NCW_INT64 = 4,
    NCW_UINT64 = 5,
    NCW_FLOAT16 = 6,
    NCW_FLOAT32 = 7,
    NCW_FLOAT64 = 8,
    NCW_BFLOAT16 = 9,
    NCW_FP8_E4M3 = 10,
    NCW_FP8_E5M2 = 11
} ncwDataType_t;

/* csrc/nccl_wrappers.h:36-42 */
typedef enum {
    NCW_SUM = 0,
    NCW_PROD = 1,
    NCW_MAX = 2,
    NCW_MIN = 3,
    NCW_AVG = 4
} ncwReduceOp_t;

/* csrc/nccl_wrappers.h:44-45 */
typedef void* ncwComm_t;
typedef struct { char internal[128]; } ncwUniqueId;

/* csrc/nccl_wrappers.h:47 */ ncwResult_t ncwGetUniqueId(ncwUniqueId* uniqueId);
/* csrc/nccl_wrappers.h:48 */ ncwResult_t ncwCommInitRank(ncwComm_t* comm, int nranks, ncwUniqueId uniqueId, int rank);
/* csrc/nccl_wrappers.h:49 */ ncwResult_t ncwCommDestroy(ncwComm_t comm);
/* csrc/nccl_wrappers.h:50 */ ncwResult_t ncwCommCount(ncwComm_t comm, int* count);
/* csrc/nccl_wrappers.h:51 */ ncwResult_t ncwCommUserRank(ncwComm_t comm, int* rank);
/* csrc/nccl_wrappers.h:52 */ ncwResult_t ncwAllReduce(const void* sendbuff, void* recvbuff, size_t count, ncwDataType_t datatype, ncwReduceOp_t op, ncwComm_t comm, cwStream_t stream);
/* csrc/nccl_wrappers.h:53 */ ncwResult_t ncwBroadcast(const void* sendbuff, void* recvbuff, size_t count, ncwDataType_t datatype, int root, ncwComm_t comm, cwStream_t stream);
/* csrc/nccl_wrappers.h:54 */ ncwResult_t ncwReduce(const void* sendbuff, void* recvbuff, size_t count, ncwDataType_t datatype, ncwReduceOp_t op, int root, ncwComm_t comm, cwStream_t stream);
/* csrc/nccl_wrappers.h:55 */ ncwResult_t ncwAllGather(const void* sendbuff, void* recvbuff, size_t sendcount, ncwDataType_t datatype, ncwComm_t comm, cwStream_t stream);
/* csrc/nccl_wrappers.h:56 */ ncwResult_t ncwReduceScatter(const void* sendbuff, void* recvbuff, size_t recvcount, ncwDataType_t datatype, ncwReduceOp_t op, ncwComm_t comm, cwStream_t stream);
/* csrc/nccl_wrappers.h:57 */ ncwResult_t ncwSend(const void* sendbuff, size_t count, ncwDataType_t datatype, int peer, ncwComm_t comm, cwStream_t stream);
/* csrc/nccl_wrappers.h:58 */ ncwResult_t ncwRecv(void* recvbuff, size_t count, ncwDataType_t datatype, int peer, ncwComm_t comm, cwStream_t stream);
/* csrc/nccl_wrappers.h:59 */ ncwResult_t ncwGroupStart(void);
/* csrc/nccl_wrappers.h:60 */ ncwResult_t ncwGroupEnd(void);
/* csrc/nccl_wrappers.h:61 */ const char* ncwGetErrorString(ncwResult_t result);

/* New.  Variable all-to-all (the spec's all_to_all, src/futhark/kernels.fut:612-617):
 * for every peer p, send send_counts[p] elements starting at element
 * send_offsets[p] of sendbuff and receive recv_counts[p] elements at
 * recv_offsets[p] of recvbuff, as one NCCL group of send/recv.  Counts and
 * offsets are HOST arrays of length nranks, in elements of `datatype`.  The
 * self-slice is copied with cudaMemcpyAsync on `stream`. */
ncwResult_t ncwAllToAllv(const void* sendbuff, const size_t* send_counts, const size_t* send_offsets,
                         void* recvbuff, const size_t* recv_counts, const size_t* recv_offsets,
                         ncwDataType_t datatype, ncwComm_t comm, cwStream_t stream);

/* New.  Initialise a communicator with NCCL's blocking mode off and a bounded
 * wait: returns NCW_ERROR_SYSTEM if the peers do not all join within
 * timeout_ms (the communicator is aborted). */
ncwResult_t ncwCommInitRankTimeout(ncwComm_t* comm, int nranks, ncwUniqueId uniqueId, int rank,
                                   int timeout_ms);
/* New.  ncclCommGetAsyncError: NCW_SUCCESS while the communicator is healthy. */
ncwResult_t ncwCommGetAsyncError(ncwComm_t comm);
/* New.  ncclCommAbort. */
ncwResult_t ncwCommAbort(ncwComm_t comm);
/* New.  Polls `stream` until its work finishes; on an asynchronous NCCL error
 * or after timeout_ms the communicator is aborted and NCW_ERROR_SYSTEM is
 * returned. */
ncwResult_t ncwStreamSynchronizeTimeout(ncwComm_t comm, cwStream_t stream, int timeout_ms);

#ifdef __cplusplus
}
#endif

#endif /* NCCL_WRAPPERS_H */
