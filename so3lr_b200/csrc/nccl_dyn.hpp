// NCCL entry points resolved at first use with dlopen instead of at link time.
//
// The library itself never links NCCL: a single-GPU user does not load it at
// all, and a process that already holds an NCCL (PyTorch bundles its own)
// gets that same library back from dlopen, so the two can never disagree on
// the version behind the `libnccl.so.2` name.
#pragma once

#include <nccl.h>

namespace so3lr_b200 {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId *);
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int);
  ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*comm_destroy)(ncclComm_t);
  ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*group_start)();
  ncclResult_t (*group_end)();
  const char *(*get_error_string)(ncclResult_t);
};

// Throws so3lr_b200::Error when no NCCL library can be loaded.
const NcclApi &nccl();

}  // namespace so3lr_b200
