// tp.cu -- the NCCL entry points tensor parallelism uses, resolved at run
// time from libnccl.so.2 (the one a process has loaded already, e.g. by
// torch.distributed, is reused: same soname).
#include <dlfcn.h>

#include <mutex>

#include "tp.cuh"

namespace ec {

const NcclApi* nccl_api(const char** why) {
  static NcclApi api{};
  static bool ok = false;
  static const char* err = "not loaded";
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      err = "libnccl.so.2 not found";
      return;
    }
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank =
        reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.broadcast = reinterpret_cast<decltype(api.broadcast)>(dlsym(h, "ncclBroadcast"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_gather &&
         api.broadcast && api.error_string;
    if (!ok) err = "libnccl.so.2 lacks an entry point";
  });
  if (why) *why = err;
  return ok ? &api : nullptr;
}

}  // namespace ec
