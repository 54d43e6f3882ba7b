// NCCL entry points of the tensor-parallel NCCL exchange, loaded from libnccl.so.2 at first use: the
// library itself links no NCCL, so a process that never asks for this exchange needs none. The
// types and constants are NCCL's own (nccl.h).
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>

namespace vkb
{

struct NcclApi
{
    ncclResult_t (*GetUniqueId)(ncclUniqueId *id);
    ncclResult_t (*CommInitRank)(ncclComm_t *comm, int nranks, ncclUniqueId id, int rank);
    ncclResult_t (*AllReduce)(const void *send, void *recv, size_t count, ncclDataType_t type, ncclRedOp_t op,
                              ncclComm_t comm, cudaStream_t stream);
    ncclResult_t (*AllGather)(const void *send, void *recv, size_t count, ncclDataType_t type, ncclComm_t comm,
                              cudaStream_t stream);
    ncclResult_t (*CommDestroy)(ncclComm_t comm);
    const char *(*GetErrorString)(ncclResult_t result);
};

// The loaded entry points, or null (logged) when libnccl.so.2 or one of them is missing.
const NcclApi *nccl_api();

} // namespace vkb
