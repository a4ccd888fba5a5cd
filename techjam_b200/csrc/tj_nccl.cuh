// NCCL, resolved at run time from the process (dlopen "libnccl.so.2": the copy
// PyTorch already loaded, or TJ_NCCL_LIB), so libtj has no link-time NCCL
// dependency.  Communicators are created non-blocking and every NCCL call is
// polled with a host-side time limit; on expiry the communicator is aborted
// and the call fails with TJ_ERR_NCCL instead of waiting forever.
#pragma once
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <mutex>
#include <thread>

namespace tj {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  bool ok = false;
  const char* why = "not loaded";
};

inline NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* path = std::getenv("TJ_NCCL_LIB");
    void* h = dlopen(path ? path : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) { api.why = "libnccl.so.2 not found (set TJ_NCCL_LIB)"; return; }
    auto sym = [&](const char* n) { return dlsym(h, n); };
    api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(sym("ncclGetUniqueId"));
    api.CommInitRankConfig = reinterpret_cast<decltype(api.CommInitRankConfig)>(sym("ncclCommInitRankConfig"));
    api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(sym("ncclCommDestroy"));
    api.CommAbort = reinterpret_cast<decltype(api.CommAbort)>(sym("ncclCommAbort"));
    api.CommGetAsyncError = reinterpret_cast<decltype(api.CommGetAsyncError)>(sym("ncclCommGetAsyncError"));
    api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(sym("ncclAllReduce"));
    api.AllGather = reinterpret_cast<decltype(api.AllGather)>(sym("ncclAllGather"));
    api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(sym("ncclGetErrorString"));
    api.ok = api.GetUniqueId && api.CommInitRankConfig && api.CommDestroy && api.CommAbort && api.CommGetAsyncError &&
             api.AllReduce && api.AllGather && api.GetErrorString;
    api.why = api.ok ? "" : "libnccl.so.2 lacks a required symbol";
  });
  return api;
}

// Polls a non-blocking communicator until its pending operation settles.
inline ncclResult_t nccl_settle(ncclComm_t comm, int timeout_ms) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    const ncclResult_t r = nccl().CommGetAsyncError(comm, &st);
    if (r != ncclSuccess) return r;
    if (st != ncclInProgress) return st;
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) return ncclInProgress;
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

}  // namespace tj
