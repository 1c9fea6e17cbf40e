// NCCL for the sequence-sharded forward, reached at run time.
//
// The library does not link NCCL: a process that uses PyTorch has already loaded
// its own libnccl.so.2, and a second copy in the same process would be a second
// set of the same symbols.  dlopen("libnccl.so.2") returns the copy already
// loaded (or loads the system one), and the handful of functions the sharded
// forward needs are looked up once.  Processes that never shard never load it.
#pragma once

#include <nccl.h>

#include <cstdio>
#include <dlfcn.h>
#include <mutex>

namespace nxs {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*broadcast)(const void *, void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    const char * (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

// The process-wide table; ok == false (with a message) when NCCL cannot be loaded.
inline const NcclApi & nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, []() {
        void * h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
        if (!h) {
            fprintf(stderr, "nexterabert: sharding needs NCCL, and libnccl.so.2 could not be loaded: %s\n", dlerror());
            return;
        }
        bool all = true;
        auto sym = [&](auto & fn, const char * name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            if (!fn) {
                fprintf(stderr, "nexterabert: NCCL has no '%s'\n", name);
                all = false;
            }
        };
        sym(api.get_unique_id, "ncclGetUniqueId");
        sym(api.comm_init_rank, "ncclCommInitRank");
        sym(api.comm_destroy, "ncclCommDestroy");
        sym(api.all_gather, "ncclAllGather");
        sym(api.broadcast, "ncclBroadcast");
        sym(api.send, "ncclSend");
        sym(api.recv, "ncclRecv");
        sym(api.group_start, "ncclGroupStart");
        sym(api.group_end, "ncclGroupEnd");
        sym(api.error_string, "ncclGetErrorString");
        api.ok = all;
    });
    return api;
}

// true on success; otherwise prints what failed
inline bool nccl_ok(ncclResult_t r, const char * what) {
    if (r == ncclSuccess) return true;
    const NcclApi & a = nccl();
    fprintf(stderr, "nexterabert: NCCL %s failed: %s\n", what, a.error_string ? a.error_string(r) : "?");
    return false;
}

} // namespace nxs
