// NCCL for the vocab-sharded LM head, loaded at run time.
//
// Only a sharded head needs NCCL (one all-reduce of the per-row argmax keys per verify pass,
// plus an all-gather of logits rows for pinfer_eval), so libpinfer.so does not link it:
// libnccl.so.2 is opened on first use. In a process that already loaded NCCL (PyTorch's
// torch.distributed does), the same copy is returned.
#include <dlfcn.h>

#include <cstdio>
#include <mutex>
#include <type_traits>

#include "nb_nccl.h"

namespace nb {

const NcclApi *nccl_api(char *err, size_t errlen) {
    static NcclApi api;
    static bool ok = false;
    static std::once_flag once;
    static char why[200] = "";
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) {
            snprintf(why, sizeof why, "cannot load libnccl.so.2: %s", dlerror());
            return;
        }
        bool all = true;
        auto get = [&](auto &fn, const char *name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            all = all && fn != nullptr;
        };
        get(api.get_unique_id, "ncclGetUniqueId");
        get(api.comm_init_rank, "ncclCommInitRank");
        get(api.comm_destroy, "ncclCommDestroy");
        get(api.all_reduce, "ncclAllReduce");
        get(api.all_gather, "ncclAllGather");
        get(api.group_start, "ncclGroupStart");
        get(api.group_end, "ncclGroupEnd");
        get(api.error_string, "ncclGetErrorString");
        if (!all) {
            snprintf(why, sizeof why, "libnccl.so.2 lacks a required symbol");
            return;
        }
        ok = true;
    });
    if (!ok && err) snprintf(err, errlen, "%s", why);
    return ok ? &api : nullptr;
}

}  // namespace nb
