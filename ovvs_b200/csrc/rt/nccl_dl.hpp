// NCCL entry points resolved at run time with dlopen("libnccl.so.2").
//
// The library does not link NCCL: single-GPU use never loads it, and when a sharded Resources
// is created the process's already-loaded libnccl.so.2 is reused (for example the newer copy
// that PyTorch bundles). Linking the system NCCL instead would pin an older libnccl.so.2 into
// the process and break a later `import torch`.
#pragma once

#include <nccl.h>

namespace ovvs {
namespace rt {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*CommAbort)(ncclComm_t);
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t);
  ncclResult_t (*GroupStart)();
  ncclResult_t (*GroupEnd)();
};

// Null when libnccl.so.2 cannot be loaded.
const NcclApi* nccl();

}  // namespace rt
}  // namespace ovvs
