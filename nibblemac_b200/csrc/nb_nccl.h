// The NCCL entry points the vocab-sharded head uses (nb_nccl.cpp opens libnccl.so.2 lazily).
#pragma once
#include <cstddef>

#include <cuda_runtime.h>
#include <nccl.h>

namespace nb {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId *);
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t);
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*group_start)();
    ncclResult_t (*group_end)();
    const char *(*error_string)(ncclResult_t);
};

// The loaded API, or null with a message in err.
const NcclApi *nccl_api(char *err, size_t errlen);

}  // namespace nb
