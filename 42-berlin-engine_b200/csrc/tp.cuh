// tp.cuh -- NCCL for tensor parallelism, loaded on first use (dlopen of
// libnccl.so.2), so that contexts without tensor parallelism do not need it.
#pragma once
#include <cuda_runtime.h>
#include <nccl.h>

namespace ec {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*);
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*comm_destroy)(ncclComm_t);
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t,
                            cudaStream_t);
  const char* (*error_string)(ncclResult_t);
};

// nullptr when libnccl.so.2 cannot be loaded (the reason in *why)
const NcclApi* nccl_api(const char** why);

}  // namespace ec
