// gx_comm.h — NCCL for the expert-parallel group, loaded at run time.
//
// The library resolves NCCL with dlopen("libnccl.so.2") only when a context is created with
// world > 1, so single-GPU users need no NCCL at all, and in a process that already loaded
// NCCL (a PyTorch host, for one) the same copy is shared instead of a second one being mapped.
// Communicators are created non-blocking, so that initialisation and every grouped send/recv
// can be bounded by a timeout instead of hanging when a peer is missing.
#pragma once
#include <cuda_runtime.h>
#include <nccl.h>
#include <stdint.h>

namespace gx {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId *);
    ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *);
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *);
    ncclResult_t (*CommAbort)(ncclComm_t);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*GroupStart)();
    ncclResult_t (*GroupEnd)();
    ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*Broadcast)(const void *, void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    const char *(*GetErrorString)(ncclResult_t);
    ncclResult_t (*GetVersion)(int *);
};

// The loaded API, or nullptr when libnccl.so.2 (or one of its symbols) is not found.
const NcclApi *nccl_api();

// Polls the communicator until its pending operation settles or timeout_ms passes.
// Returns ncclSuccess, the communicator's error, or ncclInProgress on timeout.
ncclResult_t nccl_settle(const NcclApi *api, ncclComm_t comm, uint32_t timeout_ms);

}  // namespace gx
