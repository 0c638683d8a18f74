// NCCL entry points of libspmm_b200.so, resolved at run time.
//
// NCCL is loaded with dlopen("libnccl.so.2") rather than linked: a process that already holds
// an NCCL (the one PyTorch ships, for example) keeps using that one -- the loader hands back the
// library already mapped under the soname -- and loading this library never changes which NCCL
// the rest of the process sees.
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>

namespace spmm_b200 {

struct NcclApi {
    ncclResult_t (*comm_init_all)(ncclComm_t*, int, const int*) = nullptr;
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*comm_count)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*comm_user_rank)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*comm_cu_device)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    bool ok = false;       // the single-process calls (init-all, broadcast, group, destroy) resolved
    bool ranks_ok = false;  // the one-process-per-GPU calls resolved as well
};

// The process-wide table (loaded once; `ok` false when no libnccl.so.2 can be opened).
const NcclApi& nccl();

}  // namespace spmm_b200
