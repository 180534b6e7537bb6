// nccl_dyn.cuh — NCCL entry points resolved at run time.
//
// The library does not link NCCL: a link-time dependency would load
// whatever libnccl.so.2 the loader finds first as soon as the library is
// loaded, and a process that later imports a framework built against a
// newer NCCL (same soname) would then fail to resolve that framework's
// symbols.  Instead the first expert-parallel call looks for an NCCL that
// is already loaded in the process (RTLD_NOLOAD) and only otherwise loads
// libnccl.so.2 by the usual search.
#pragma once
#include <nccl.h>
#include <dlfcn.h>
#include <mutex>

namespace moe {

struct NcclApi {
    decltype(&ncclGetUniqueId) GetUniqueId = nullptr;
    decltype(&ncclCommInitRank) CommInitRank = nullptr;
    decltype(&ncclCommInitRankConfig) CommInitRankConfig = nullptr;
    decltype(&ncclCommAbort) CommAbort = nullptr;
    decltype(&ncclCommFinalize) CommFinalize = nullptr;
    decltype(&ncclCommDestroy) CommDestroy = nullptr;
    decltype(&ncclCommGetAsyncError) CommGetAsyncError = nullptr;
    decltype(&ncclAllGather) AllGather = nullptr;
    decltype(&ncclAllReduce) AllReduce = nullptr;
    decltype(&ncclGetErrorString) GetErrorString = nullptr;
    bool ok = false;
};

inline const NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) return;
        api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
        api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
        api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
        api.CommInitRankConfig = reinterpret_cast<decltype(api.CommInitRankConfig)>(
            dlsym(h, "ncclCommInitRankConfig"));
        api.CommAbort = reinterpret_cast<decltype(api.CommAbort)>(dlsym(h, "ncclCommAbort"));
        api.CommFinalize =
            reinterpret_cast<decltype(api.CommFinalize)>(dlsym(h, "ncclCommFinalize"));
        api.CommGetAsyncError =
            reinterpret_cast<decltype(api.CommGetAsyncError)>(dlsym(h, "ncclCommGetAsyncError"));
        api.AllGather = reinterpret_cast<decltype(api.AllGather)>(dlsym(h, "ncclAllGather"));
        api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(dlsym(h, "ncclAllReduce"));
        api.GetErrorString =
            reinterpret_cast<decltype(api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
        api.ok = api.GetUniqueId && api.CommInitRank && api.CommInitRankConfig && api.CommAbort &&
                 api.CommFinalize &&
                 api.CommDestroy && api.CommGetAsyncError &&
                 api.AllGather && api.AllReduce && api.GetErrorString;
    });
    return api;
}

}  // namespace moe
