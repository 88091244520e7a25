#include <dlfcn.h>

#include <mutex>

#include "nccl_dyn.cuh"
#include "runtime.cuh"

namespace fg {

const NcclApi &nccl() {
  static NcclApi api;
  static std::once_flag once;
  static std::string err;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // already in the process?
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char *e = dlerror();
      err = e ? e : "dlopen(libnccl.so.2) failed";
      return;
    }
    auto sym = [&](const char *n) { return dlsym(h, n); };
    api.GetUniqueId = (decltype(api.GetUniqueId))sym("ncclGetUniqueId");
    api.CommInitRank = (decltype(api.CommInitRank))sym("ncclCommInitRank");
    api.CommDestroy = (decltype(api.CommDestroy))sym("ncclCommDestroy");
    api.CommAbort = (decltype(api.CommAbort))sym("ncclCommAbort");
    api.CommGetAsyncError = (decltype(api.CommGetAsyncError))sym("ncclCommGetAsyncError");
    api.AllReduce = (decltype(api.AllReduce))sym("ncclAllReduce");
    api.AllGather = (decltype(api.AllGather))sym("ncclAllGather");
    api.GetErrorString = (decltype(api.GetErrorString))sym("ncclGetErrorString");
    if (!api.GetUniqueId || !api.CommInitRank || !api.AllReduce || !api.AllGather || !api.GetErrorString ||
        !api.CommDestroy) {
      err = "libnccl.so.2 lacks a required symbol";
      api = NcclApi();
    }
  });
  FG_REQUIRE(api.AllReduce != nullptr, FG_ERR_UNAVAILABLE, "NCCL unavailable: %s", err.c_str());
  return api;
}

}  // namespace fg
