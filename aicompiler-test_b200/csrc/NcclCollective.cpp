// NCCL collective (see NcclCollective.hpp).
#include "NcclCollective.hpp"

#include <dlfcn.h>

#include <cstring>
#include <mutex>

namespace tensor::runtime {
namespace {

struct NcclApi {
  bool loaded = false;
  std::string error;
  ncclResult_t (*getUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*commInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*allReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*commAbort)(ncclComm_t) = nullptr;
  const char *(*getErrorString)(ncclResult_t) = nullptr;
};

NcclApi &api() {
  static NcclApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      a.error = std::string("NCCL unavailable: ") + dlerror();
      return;
    }
    a.getUniqueId = reinterpret_cast<decltype(a.getUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    a.commInitRank = reinterpret_cast<decltype(a.commInitRank)>(dlsym(h, "ncclCommInitRank"));
    a.allReduce = reinterpret_cast<decltype(a.allReduce)>(dlsym(h, "ncclAllReduce"));
    a.commDestroy = reinterpret_cast<decltype(a.commDestroy)>(dlsym(h, "ncclCommDestroy"));
    a.commAbort = reinterpret_cast<decltype(a.commAbort)>(dlsym(h, "ncclCommAbort"));
    a.getErrorString = reinterpret_cast<decltype(a.getErrorString)>(dlsym(h, "ncclGetErrorString"));
    if (!a.getUniqueId || !a.commInitRank || !a.allReduce || !a.commDestroy || !a.getErrorString) {
      a.error = "NCCL library lacks required symbols";
      return;
    }
    a.loaded = true;
  });
  return a;
}

std::string ncclText(const char *what, ncclResult_t r) {
  return std::string(what) + ": " + (api().getErrorString ? api().getErrorString(r) : "nccl error");
}

}  // namespace

std::string ncclUniqueIdBytes(unsigned char *id) {
  auto &a = api();
  if (!a.loaded) return a.error;
  ncclUniqueId uid;
  const ncclResult_t r = a.getUniqueId(&uid);
  if (r != ncclSuccess) return ncclText("ncclGetUniqueId", r);
  std::memcpy(id, uid.internal, NCCL_UNIQUE_ID_BYTES);
  return {};
}

std::shared_ptr<NcclCollective> NcclCollective::create(const unsigned char *id, int world, int rank,
                                                       std::string *error) {
  auto &a = api();
  if (!a.loaded) {
    if (error) *error = a.error;
    return nullptr;
  }
  ncclUniqueId uid;
  std::memcpy(uid.internal, id, NCCL_UNIQUE_ID_BYTES);
  std::shared_ptr<NcclCollective> c(new NcclCollective());
  const ncclResult_t r = a.commInitRank(&c->comm_, world, uid, rank);
  if (r != ncclSuccess) {
    if (error) *error = ncclText("ncclCommInitRank", r);
    return nullptr;
  }
  return c;
}

NcclCollective::~NcclCollective() {
  if (comm_ && api().loaded) api().commDestroy(comm_);
}

void NcclCollective::abort() {
  if (comm_ && api().loaded && api().commAbort) api().commAbort(comm_);
  comm_ = nullptr;
}

cudaError_t NcclCollective::allReduceSumF32(float *buf, std::size_t count, cudaStream_t s) {
  const ncclResult_t r = api().allReduce(buf, buf, count, ncclFloat32, ncclSum, comm_, s);
  if (r != ncclSuccess) {
    error_ = ncclText("ncclAllReduce(sum)", r);
    return cudaErrorUnknown;
  }
  return cudaSuccess;
}

cudaError_t NcclCollective::allReduceMaxU64(unsigned long long *buf, std::size_t count, cudaStream_t s) {
  const ncclResult_t r = api().allReduce(buf, buf, count, ncclUint64, ncclMax, comm_, s);
  if (r != ncclSuccess) {
    error_ = ncclText("ncclAllReduce(max)", r);
    return cudaErrorUnknown;
  }
  return cudaSuccess;
}

}  // namespace tensor::runtime
