// comm.cu -- the exchange of a multi-GPU round: all-to-all with per-peer counts
// and a max all-reduce, as NCCL group calls issued straight onto the caller's
// stream (no extra streams or events per call).
//
// NCCL is loaded at run time (the copy a framework already loaded, else
// libnccl.so.2), so the library has no link-time NCCL dependency and single-GPU
// users never load it.  Only NCCL's public C API is used.
#include <dlfcn.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "eps_b200.h"

namespace {

// NCCL public API types (nccl.h): an opaque communicator, a 128-byte unique id,
// and the enum values used here.
typedef struct ncclComm* ncclComm_t;
struct ncclUniqueId { char internal[128]; };
enum NcclResult { kNcclSuccess = 0 };
enum NcclType { kNcclUint8 = 1, kNcclUint32 = 3 };
enum NcclOp { kNcclMax = 2 };

struct Nccl {
  int (*GetUniqueId)(ncclUniqueId*) = nullptr;
  int (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  int (*CommDestroy)(ncclComm_t) = nullptr;
  int (*GroupStart)() = nullptr;
  int (*GroupEnd)() = nullptr;
  int (*Send)(const void*, size_t, int, int, ncclComm_t, cudaStream_t) = nullptr;
  int (*Recv)(void*, size_t, int, int, ncclComm_t, cudaStream_t) = nullptr;
  int (*AllReduce)(const void*, void*, size_t, int, int, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*GetErrorString)(int) = nullptr;
  bool ok = false;
  std::string why;
};

Nccl& Lib() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) { n.why = "libnccl.so.2 could not be loaded"; return; }
    auto sym = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      return fn != nullptr;
    };
    n.ok = sym(n.GetUniqueId, "ncclGetUniqueId") && sym(n.CommInitRank, "ncclCommInitRank") &&
           sym(n.CommDestroy, "ncclCommDestroy") && sym(n.GroupStart, "ncclGroupStart") &&
           sym(n.GroupEnd, "ncclGroupEnd") && sym(n.Send, "ncclSend") && sym(n.Recv, "ncclRecv") &&
           sym(n.AllReduce, "ncclAllReduce") && sym(n.GetErrorString, "ncclGetErrorString");
    if (!n.ok) n.why = "libnccl.so.2 lacks a required entry point";
  });
  return n;
}

struct Fail : std::runtime_error {
  int code;
  Fail(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

void Check(int r, const char* what) {
  if (r != kNcclSuccess) {
    const char* s = Lib().GetErrorString ? Lib().GetErrorString(r) : "error";
    throw Fail(EPS_B200_RUN_FAILED, std::string(what) + ": " + s);
  }
}

template <typename F>
int Guard(EpsB200Status* status, F fn) noexcept {
  if (status) { status->code = 0; status->message[0] = 0; }
  auto fail = [&](int code, const char* m) {
    if (status) {
      status->code = code;
      std::strncpy(status->message, m, sizeof(status->message) - 1);
      status->message[sizeof(status->message) - 1] = 0;
    }
    return code;
  };
  try { fn(); return 0; }
  catch (const Fail& e) { return fail(e.code, e.what()); }
  catch (const std::exception& e) { return fail(EPS_B200_RUN_FAILED, e.what()); }
  catch (...) { return fail(EPS_B200_RUN_FAILED, "unknown communicator failure"); }
}

Nccl& Need() {
  Nccl& n = Lib();
  if (!n.ok) throw Fail(EPS_B200_UNAVAILABLE, n.why);
  return n;
}

}  // namespace

struct EpsB200Comm {
  ncclComm_t comm = nullptr;
  int device = 0;
  unsigned rank = 0, world = 1;
  std::mutex mutex;
};

extern "C" {

int eps_b200_comm_unique_id(uint8_t* id, EpsB200Status* status) {
  return Guard(status, [&] {
    if (!id) throw Fail(EPS_B200_INVALID_ARGUMENT, "null unique id buffer");
    ncclUniqueId u;
    Check(Need().GetUniqueId(&u), "ncclGetUniqueId");
    std::memcpy(id, u.internal, sizeof(u.internal));
  });
}

int eps_b200_comm_create(int32_t device, uint32_t rank, uint32_t world, const uint8_t* id,
                         EpsB200Comm** out, EpsB200Status* status) {
  return Guard(status, [&] {
    if (!id || !out || world == 0 || rank >= world)
      throw Fail(EPS_B200_INVALID_ARGUMENT, "invalid communicator arguments");
    Nccl& n = Need();
    if (cudaSetDevice(device) != cudaSuccess) throw Fail(EPS_B200_INVALID_ARGUMENT, "invalid device");
    auto* c = new EpsB200Comm;
    c->device = device;
    c->rank = rank;
    c->world = world;
    ncclUniqueId u;
    std::memcpy(u.internal, id, sizeof(u.internal));
    const int r = n.CommInitRank(&c->comm, (int)world, u, (int)rank);
    if (r != kNcclSuccess) { delete c; Check(r, "ncclCommInitRank"); }
    *out = c;
  });
}

void eps_b200_comm_destroy(EpsB200Comm* c) {
  if (!c) return;
  if (c->comm && Lib().ok) {
    cudaSetDevice(c->device);
    Lib().CommDestroy(c->comm);
  }
  delete c;
}

int eps_b200_comm_alltoallv(EpsB200Comm* c, const void* send, const uint64_t* send_counts,
                            void* recv, const uint64_t* recv_counts, uint32_t elem_bytes,
                            void* stream, EpsB200Status* status) {
  return Guard(status, [&] {
    if (!c || !send_counts || !recv_counts || elem_bytes == 0)
      throw Fail(EPS_B200_INVALID_ARGUMENT, "invalid all-to-all arguments");
    Nccl& n = Need();
    std::lock_guard lock(c->mutex);
    if (cudaSetDevice(c->device) != cudaSuccess) throw Fail(EPS_B200_RUN_FAILED, "cudaSetDevice");
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const char* sp = static_cast<const char*>(send);
    char* rp = static_cast<char*>(recv);
    Check(n.GroupStart(), "ncclGroupStart");
    size_t so = 0, ro = 0;
    int err = kNcclSuccess;
    for (unsigned p = 0; p < c->world && err == kNcclSuccess; ++p) {
      const size_t sb = send_counts[p] * elem_bytes, rb = recv_counts[p] * elem_bytes;
      if (sb) err = n.Send(sp + so, sb, kNcclUint8, (int)p, c->comm, s);
      if (err == kNcclSuccess && rb) err = n.Recv(rp + ro, rb, kNcclUint8, (int)p, c->comm, s);
      so += sb;
      ro += rb;
    }
    const int end = n.GroupEnd();
    Check(err, "ncclSend/ncclRecv");
    Check(end, "ncclGroupEnd");
  });
}

int eps_b200_comm_allreduce_max(EpsB200Comm* c, uint32_t* buf, uint64_t count, void* stream,
                                EpsB200Status* status) {
  return Guard(status, [&] {
    if (!c || (!buf && count)) throw Fail(EPS_B200_INVALID_ARGUMENT, "invalid all-reduce arguments");
    Nccl& n = Need();
    std::lock_guard lock(c->mutex);
    if (cudaSetDevice(c->device) != cudaSuccess) throw Fail(EPS_B200_RUN_FAILED, "cudaSetDevice");
    Check(n.AllReduce(buf, buf, count, kNcclUint32, kNcclMax, c->comm,
                      static_cast<cudaStream_t>(stream)), "ncclAllReduce");
  });
}

}  // extern "C"

namespace eps_b200 {
// Internal queries for the sharded client (client.cu).
unsigned comm_rank(const EpsB200Comm* c) { return c->rank; }
unsigned comm_world(const EpsB200Comm* c) { return c->world; }
int comm_device(const EpsB200Comm* c) { return c->device; }
}  // namespace eps_b200
