// nccl_dyn.h -- NCCL, loaded at the first use of the sharded search.
//
// The engine library does not link NCCL: a process that never shards never
// loads it, and a process that already holds an NCCL (PyTorch's, for one)
// shares that copy instead of loading a second one with the same soname.
// Only the public NCCL API used by the sharded search is resolved.
#pragma once

#include <dlfcn.h>
#include <nccl.h>

#include <mutex>

namespace frnn {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*Broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
};

// The process's NCCL: an already loaded libnccl.so.2 if there is one, else
// the first libnccl.so.2 the dynamic loader finds.  nullptr when none loads.
inline const NcclApi* nccl_api() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        auto sym = [&](auto& fn, const char* name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            return fn != nullptr;
        };
        api.ok = sym(api.GetUniqueId, "ncclGetUniqueId") && sym(api.CommInitRank, "ncclCommInitRank") &&
                 sym(api.CommDestroy, "ncclCommDestroy") && sym(api.CommAbort, "ncclCommAbort") &&
                 sym(api.CommGetAsyncError, "ncclCommGetAsyncError") && sym(api.Broadcast, "ncclBroadcast") &&
                 sym(api.AllReduce, "ncclAllReduce") && sym(api.Send, "ncclSend") && sym(api.Recv, "ncclRecv") &&
                 sym(api.GroupStart, "ncclGroupStart") && sym(api.GroupEnd, "ncclGroupEnd") &&
                 sym(api.GetErrorString, "ncclGetErrorString");
    });
    return api.ok ? &api : nullptr;
}

}  // namespace frnn
