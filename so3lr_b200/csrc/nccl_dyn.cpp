#include "nccl_dyn.hpp"

#include <dlfcn.h>

#include <mutex>
#include <string>

#include "model_host.hpp"

namespace so3lr_b200 {

const NcclApi &nccl() {
  static std::mutex mu;
  static NcclApi api{};
  static bool loaded = false;
  std::lock_guard<std::mutex> lock(mu);
  if (loaded) return api;
  void *lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!lib) lib = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!lib) {
    const char *why = dlerror();
    throw Error(std::string("SO3LR: multi-GPU decomposition needs NCCL (libnccl.so.2): ") + (why ? why : "not found"));
  }
  auto sym = [&](const char *name) {
    void *p = dlsym(lib, name);
    if (!p) throw Error(std::string("SO3LR: NCCL library lacks ") + name);
    return p;
  };
  api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
  api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
  api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
  api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
  api.get_error_string = reinterpret_cast<decltype(api.get_error_string)>(sym("ncclGetErrorString"));
  api.send = reinterpret_cast<decltype(api.send)>(sym("ncclSend"));
  api.recv = reinterpret_cast<decltype(api.recv)>(sym("ncclRecv"));
  api.group_start = reinterpret_cast<decltype(api.group_start)>(sym("ncclGroupStart"));
  api.group_end = reinterpret_cast<decltype(api.group_end)>(sym("ncclGroupEnd"));
  loaded = true;
  return api;
}

}  // namespace so3lr_b200
