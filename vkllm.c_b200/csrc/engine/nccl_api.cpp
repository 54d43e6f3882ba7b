// Loader of the NCCL entry points (nccl_api.h).
#include "nccl_api.h"

#include <dlfcn.h>
#include <mutex>

#include "../runtime/internal.h"

namespace vkb
{

const NcclApi *nccl_api()
{
    static NcclApi api;
    static bool ok = false;
    static std::once_flag once;
    std::call_once(once, [] {
        // A process that already loaded NCCL (e.g. through PyTorch) gets that copy back by its soname.
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h)
        {
            log_error("tensor parallel NCCL exchange: cannot load libnccl.so.2: %s", dlerror());
            return;
        }
        api.GetUniqueId = (decltype(api.GetUniqueId))dlsym(h, "ncclGetUniqueId");
        api.CommInitRank = (decltype(api.CommInitRank))dlsym(h, "ncclCommInitRank");
        api.AllReduce = (decltype(api.AllReduce))dlsym(h, "ncclAllReduce");
        api.AllGather = (decltype(api.AllGather))dlsym(h, "ncclAllGather");
        api.CommDestroy = (decltype(api.CommDestroy))dlsym(h, "ncclCommDestroy");
        api.GetErrorString = (decltype(api.GetErrorString))dlsym(h, "ncclGetErrorString");
        ok = api.GetUniqueId && api.CommInitRank && api.AllReduce && api.AllGather && api.CommDestroy &&
             api.GetErrorString;
        if (!ok)
            log_error("tensor parallel NCCL exchange: libnccl.so.2 lacks an entry point");
    });
    return ok ? &api : nullptr;
}

} // namespace vkb
