// NCCL entry points resolved at run time from libnccl.so.2 (the copy already loaded into
// the process, e.g. by PyTorch, or the system one), so that libce4b200 has no link-time
// NCCL dependency and never mixes two NCCL versions in one process.
#pragma once

#include <nccl.h>

namespace ce4b {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

// Loads the API once; fails (CE4B_ERR_UNSUPPORTED) if libnccl.so.2 cannot be opened.
const NcclApi& nccl();

// Throws CE4B_ERR_CUDA with NCCL's message when r != ncclSuccess.
void check_nccl(ncclResult_t r, const char* what);

}  // namespace ce4b
