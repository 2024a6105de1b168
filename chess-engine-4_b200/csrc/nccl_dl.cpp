#include "nccl_dl.h"

#include <dlfcn.h>

#include <mutex>
#include <string>

#include "internal.h"

namespace ce4b {

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  static std::string error;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) {
      const char* e = dlerror();
      error = std::string("cannot load libnccl.so.2: ") + (e != nullptr ? e : "unknown error");
      return;
    }
    auto sym = [&](const char* name) {
      void* p = dlsym(h, name);
      if (p == nullptr && error.empty()) error = std::string("libnccl.so.2 lacks ") + name;
      return p;
    };
    api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(sym("ncclGetUniqueId"));
    api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(sym("ncclCommInitRank"));
    api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(sym("ncclCommDestroy"));
    api.GroupStart = reinterpret_cast<decltype(api.GroupStart)>(sym("ncclGroupStart"));
    api.GroupEnd = reinterpret_cast<decltype(api.GroupEnd)>(sym("ncclGroupEnd"));
    api.Send = reinterpret_cast<decltype(api.Send)>(sym("ncclSend"));
    api.Recv = reinterpret_cast<decltype(api.Recv)>(sym("ncclRecv"));
    api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(sym("ncclGetErrorString"));
  });
  if (!error.empty()) fail(CE4B_ERR_UNSUPPORTED, error);
  return api;
}

void check_nccl(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return;
  const char* msg = nccl().GetErrorString != nullptr ? nccl().GetErrorString(r) : "unknown";
  fail(CE4B_ERR_CUDA, std::string(what) + ": NCCL error " + std::to_string(static_cast<int>(r)) +
                          " (" + msg + ")");
}

}  // namespace ce4b
