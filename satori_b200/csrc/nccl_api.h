// nccl_api.h -- NCCL loaded at run time (dlopen of libnccl.so.2), so a process that already loaded NCCL
// (for example through torch.distributed) shares that copy; shared by the sharded session and the sharded
// MatVec.
#pragma once

#include <nccl.h>

namespace satori {

struct NcclApi {
    void *lib = nullptr;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    const char *(*GetErrorString)(ncclResult_t) = nullptr;
};

// The loaded API, or null when libnccl.so.2 is missing or incomplete.
const NcclApi *nccl_api();
// Records an NCCL failure as SATORI_ERR_CUDA and returns it.
int nccl_fail(const NcclApi *api, ncclResult_t r, const char *what);

}  // namespace satori
