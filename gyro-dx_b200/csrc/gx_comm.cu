// gx_comm.cu — run-time binding of NCCL (see gx_comm.h).
#include <dlfcn.h>

#include <chrono>
#include <mutex>
#include <thread>

#include "gx_comm.h"

namespace gx {

namespace {

template <typename F>
bool bind(void *h, F &fn, const char *name) {
    fn = reinterpret_cast<F>(dlsym(h, name));
    return fn != nullptr;
}

}  // namespace

const NcclApi *nccl_api() {
    static NcclApi api{};
    static bool ok = false;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        ok = bind(h, api.GetUniqueId, "ncclGetUniqueId") && bind(h, api.CommInitRankConfig, "ncclCommInitRankConfig") &&
             bind(h, api.CommGetAsyncError, "ncclCommGetAsyncError") && bind(h, api.CommAbort, "ncclCommAbort") &&
             bind(h, api.CommDestroy, "ncclCommDestroy") && bind(h, api.GroupStart, "ncclGroupStart") &&
             bind(h, api.GroupEnd, "ncclGroupEnd") && bind(h, api.Send, "ncclSend") && bind(h, api.Recv, "ncclRecv") &&
             bind(h, api.Broadcast, "ncclBroadcast") &&
             bind(h, api.GetErrorString, "ncclGetErrorString") && bind(h, api.GetVersion, "ncclGetVersion");
    });
    return ok ? &api : nullptr;
}

ncclResult_t nccl_settle(const NcclApi *api, ncclComm_t comm, uint32_t timeout_ms) {
    // Enqueueing a group normally settles within microseconds, and the GPU waits for the next
    // launch meanwhile: poll without sleeping for the first 2 ms, then back off.
    const auto start = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        const ncclResult_t r = api->CommGetAsyncError(comm, &st);
        if (r != ncclSuccess) return r;
        if (st != ncclInProgress) return st;
        const auto us =
            std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - start).count();
        if ((uint64_t)us >= (uint64_t)timeout_ms * 1000u) return ncclInProgress;
        if (us < 2000) std::this_thread::yield();
        else std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

}  // namespace gx
