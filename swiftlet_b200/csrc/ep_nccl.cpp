// NCCL entry points resolved with dlopen/dlsym on first use (see ep_nccl.h).
#include "ep_nccl.h"

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>

#include "common.h"

namespace swl {

namespace {

struct Nccl {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*reduce_scatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                                 cudaStream_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  ncclResult_t (*async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  std::string why;
  bool ok = false;
};

Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char* e = dlerror();
      n.why = std::string("cannot load libnccl.so.2: ") + (e ? e : "not found");
      return;
    }
    auto sym = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      if (!fn && n.why.empty()) n.why = std::string("libnccl.so.2 lacks ") + name;
    };
    sym(n.get_unique_id, "ncclGetUniqueId");
    sym(n.comm_init_rank, "ncclCommInitRank");
    sym(n.comm_destroy, "ncclCommDestroy");
    sym(n.all_gather, "ncclAllGather");
    sym(n.reduce_scatter, "ncclReduceScatter");
    sym(n.all_reduce, "ncclAllReduce");
    sym(n.group_start, "ncclGroupStart");
    sym(n.group_end, "ncclGroupEnd");
    sym(n.error_string, "ncclGetErrorString");
    sym(n.async_error, "ncclCommGetAsyncError");
    n.ok = n.why.empty();
  });
  if (!n.ok) throw Error(ERR_UNSUPPORTED, "expert parallelism: " + n.why);
  return n;
}

void check(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return;
  Nccl& n = nccl();
  throw Error(ERR_CUDA, std::string("NCCL ") + what + ": " + (n.error_string ? n.error_string(r) : "error"));
}

}  // namespace

struct EpComm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
};

void ep_unique_id(void* out) {
  ncclUniqueId id;
  check(nccl().get_unique_id(&id), "ncclGetUniqueId");
  memcpy(out, &id, sizeof(id));
}

EpComm* ep_init(int rank, int world, const void* id) {
  if (world < 1 || rank < 0 || rank >= world) throw Error(ERR_INVALID, "expert parallelism: rank outside the world");
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  EpComm* c = new EpComm();
  c->rank = rank;
  c->world = world;
  ncclResult_t r = nccl().comm_init_rank(&c->comm, world, u, rank);
  if (r != ncclSuccess) {
    delete c;
    check(r, "ncclCommInitRank");
  }
  return c;
}

void ep_destroy(EpComm* c) {
  if (!c) return;
  if (c->comm) nccl().comm_destroy(c->comm);
  delete c;
}

bool ep_async_error(EpComm* c, std::string* why) {
  if (!c || !c->comm) return false;
  ncclResult_t r = ncclSuccess;
  if (nccl().async_error(c->comm, &r) != ncclSuccess) return false;
  if (r == ncclSuccess || r == ncclInProgress) return false;
  if (why) *why = nccl().error_string ? nccl().error_string(r) : "error";
  return true;
}

void ep_allgather(EpComm* c, void* buf, size_t bytes, cudaStream_t st) {
  char* b = static_cast<char*>(buf);
  check(nccl().all_gather(b + size_t(c->rank) * bytes, b, bytes, ncclUint8, c->comm, st), "ncclAllGather");
}

void ep_reduce_scatter(EpComm* c, const float* send, float* recv, size_t n, cudaStream_t st) {
  check(nccl().reduce_scatter(send, recv, n, ncclFloat32, ncclSum, c->comm, st), "ncclReduceScatter");
}

void ep_group_start(EpComm*) { check(nccl().group_start(), "ncclGroupStart"); }
void ep_group_end(EpComm*) { check(nccl().group_end(), "ncclGroupEnd"); }

void ep_allreduce_i32_max(EpComm* c, int* buf, size_t n, cudaStream_t st) {
  check(nccl().all_reduce(buf, buf, n, ncclInt32, ncclMax, c->comm, st), "ncclAllReduce");
}

}  // namespace swl
