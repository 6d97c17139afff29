// NCCL entry points resolved at run time (dlopen), so the library carries no
// link-time NCCL dependency and shares the NCCL a host process (for example
// PyTorch) has already loaded. Types come from the NCCL header.
#pragma once

#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <mutex>
#include <thread>

namespace minq {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  // non-blocking communicators (initialisation under a host deadline)
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  bool ok = false;
  bool nonblocking = false;
};

// The process's NCCL (already loaded, else libnccl.so.2 from the library
// path); ok == false when none can be loaded.
inline const NcclApi& nccl_api() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
    api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(dlsym(h, "ncclAllReduce"));
    api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
    api.GetErrorString =
        reinterpret_cast<decltype(api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.GetUniqueId && api.CommInitRank && api.AllReduce && api.CommDestroy &&
             api.GetErrorString;
    api.CommInitRankConfig =
        reinterpret_cast<decltype(api.CommInitRankConfig)>(dlsym(h, "ncclCommInitRankConfig"));
    api.CommGetAsyncError =
        reinterpret_cast<decltype(api.CommGetAsyncError)>(dlsym(h, "ncclCommGetAsyncError"));
    api.CommAbort = reinterpret_cast<decltype(api.CommAbort)>(dlsym(h, "ncclCommAbort"));
    api.nonblocking = api.CommInitRankConfig && api.CommGetAsyncError && api.CommAbort;
  });
  return api;
}

// Wait until an operation on a non-blocking communicator (returned
// ncclInProgress) has finished its host-side part, up to `deadline`;
// ncclInProgress on a blocking one never occurs. On expiry the communicator
// is aborted and ncclInProgress returned.
inline ncclResult_t nccl_settle(ncclComm_t comm, ncclResult_t r,
                                std::chrono::steady_clock::time_point deadline) {
  const NcclApi& nc = nccl_api();
  while (r == ncclInProgress) {
    if (std::chrono::steady_clock::now() > deadline) {
      nc.CommAbort(comm);
      return ncclInProgress;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
    if (nc.CommGetAsyncError(comm, &r) != ncclSuccess) return ncclInternalError;
  }
  return r;
}

}  // namespace minq
