// NCCL for the tensor-parallel batch, loaded at run time: the library itself has no link-time
// dependency on NCCL (it loads and runs everything else without it), and a process that already
// loaded libnccl.so.2 (PyTorch does) shares that copy.
#include <dlfcn.h>

#include <mutex>
#include <string>

#include "ls_internal.h"

namespace ls {

const NcclApi& nccl_api() {
  static NcclApi api;
  static std::once_flag once;
  static std::string failure;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      failure = std::string("cannot load libnccl.so.2: ") + dlerror();
      return;
    }
    auto sym = [&](const char* name) {
      void* p = dlsym(h, name);
      if (!p && failure.empty()) failure = std::string("libnccl.so.2 lacks ") + name;
      return p;
    };
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
    api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(sym("ncclCommAbort"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
  });
  if (!failure.empty()) LS_THROW(-3, failure);
  return api;
}

void nccl_check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) LS_THROW(-3, std::string(what) + ": " + nccl_api().error_string(r));
}

}  // namespace ls
