// NCCL entry points of libcea.so: communicator set-up and the three transfers of the sequence-parallel
// path (ring step, uneven all-to-all, all-gather) for callers outside PyTorch.
//
// NCCL is resolved at run time (dlopen + dlsym) rather than linked, so libcea.so loads on machines without
// NCCL and shares the NCCL instance a host process has already loaded (PyTorch's, typically): the library
// named by CEA_NCCL_LIBRARY if set, else an already loaded libnccl.so.2, else libnccl.so.2 from the loader
// path.  Only NCCL's stable C API is used; its few types are declared here as the NCCL 2.x headers define
// them (an opaque communicator pointer, a 128-byte unique id, int result and datatype codes).
#pragma once

#include <dlfcn.h>

#include <mutex>
#include <string>

namespace cea {
namespace nccl {

typedef int Result;  // ncclResult_t, ncclSuccess = 0
typedef void* Comm;  // ncclComm_t
struct UniqueId {
  char internal[CEA_NCCL_ID_BYTES];
};
constexpr int kUint8 = 1;  // ncclUint8

struct Api {
  Result (*get_unique_id)(UniqueId*) = nullptr;
  Result (*comm_init_rank)(Comm*, int, UniqueId, int) = nullptr;
  Result (*comm_destroy)(Comm) = nullptr;
  Result (*comm_abort)(Comm) = nullptr;
  Result (*group_start)() = nullptr;
  Result (*group_end)() = nullptr;
  Result (*send)(const void*, size_t, int, int, Comm, cudaStream_t) = nullptr;
  Result (*recv)(void*, size_t, int, int, Comm, cudaStream_t) = nullptr;
  Result (*all_gather)(const void*, void*, size_t, int, Comm, cudaStream_t) = nullptr;
  const char* (*error_string)(Result) = nullptr;
  bool ok = false;
  std::string why;
};

inline const Api& api() {
  static Api a;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = nullptr;
    const char* path = getenv("CEA_NCCL_LIBRARY");
    if (path != nullptr && path[0] != '\0') {
      h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    } else {
      h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the NCCL this process already uses
      if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    }
    if (h == nullptr) {
      const char* e = dlerror();
      a.why = std::string("NCCL library not found: ") + (e ? e : "libnccl.so.2");
      return;
    }
    bool all = true;
    auto get = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      if (fn == nullptr) {
        all = false;
        if (a.why.empty()) a.why = std::string("NCCL library lacks ") + name;
      }
    };
    get(a.get_unique_id, "ncclGetUniqueId");
    get(a.comm_init_rank, "ncclCommInitRank");
    get(a.comm_destroy, "ncclCommDestroy");
    get(a.comm_abort, "ncclCommAbort");
    get(a.group_start, "ncclGroupStart");
    get(a.group_end, "ncclGroupEnd");
    get(a.send, "ncclSend");
    get(a.recv, "ncclRecv");
    get(a.all_gather, "ncclAllGather");
    get(a.error_string, "ncclGetErrorString");
    a.ok = all;
  });
  return a;
}

}  // namespace nccl
}  // namespace cea

struct cea_nccl_comm {
  cea::nccl::Comm comm;
  int rank;
  int nranks;
};
