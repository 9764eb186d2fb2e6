// client.cu -- the host side of a multi-GPU round in C++: the reference's
// DistributedClient (include/eps/distributed_client.hpp:32-70) over one shard
// per GPU, with every rank both a client of its own batch and the shard of the
// keys k with k % n == rank.
//
//   prepare   route (partition by key % n, src/access/prepared_lookup.cpp:47-83)
//             -> count rows all-to-all -> ONE wait for the counts -> payload
//             (keys, kept-bag offsets, valid lengths) all-to-all; on the input
//             stream and the input communicator, so the next batch can be
//             prepared while the current round's push runs
//   lookup    shard lookup over every requester's part (eps_b200_serve) ->
//             partial all-to-all -> shard-ordered merge and mean
//             (src/client/distributed_client.cpp:173-188,227-232)
//   push      gradient gather with the client finiteness check
//             (src/client/distributed_client.cpp:249) -> max all-reduce of the
//             flag -> gradient all-to-all -> one push per shard that rejects on
//             the device if any rank saw a non-finite value (eps_b200_serve_push)
//
// One round of n ranks is what a reference shard serves for ONE combined
// request: the features of every rank, rank-major (ids r * F + f).  Input
// errors travel in the count rows, so every rank raises the same error before
// any data moves.  Exchange buffers come from the stream-ordered allocator.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "eps_b200.h"

namespace eps_b200 {
bool store_table_dimension(EpsB200Store* s, unsigned table, unsigned* dim);
int store_device(EpsB200Store* s);
unsigned store_shard(EpsB200Store* s, unsigned* count);
unsigned comm_rank(const EpsB200Comm* c);
unsigned comm_world(const EpsB200Comm* c);
int comm_device(const EpsB200Comm* c);
}  // namespace eps_b200

namespace {

struct Fail : std::runtime_error {
  int code;
  Fail(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

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
  catch (const std::bad_alloc&) { return fail(EPS_B200_CAPACITY_EXCEEDED, "client allocation failed"); }
  catch (const std::exception& e) { return fail(EPS_B200_RUN_FAILED, e.what()); }
  catch (...) { return fail(EPS_B200_RUN_FAILED, "unknown client failure"); }
}

void Cu(cudaError_t e) {
  if (e != cudaSuccess)
    throw Fail(e == cudaErrorMemoryAllocation ? EPS_B200_CAPACITY_EXCEEDED : EPS_B200_RUN_FAILED,
               cudaGetErrorString(e));
}
void Call(int rc, const EpsB200Status& st) {
  if (rc) throw Fail(rc, st.message);
}
void Require(bool ok, const char* m, int code = EPS_B200_INVALID_ARGUMENT) {
  if (!ok) throw Fail(code, m);
}

std::string InputMessage(long long bits) {
  std::string m = "invalid lookup inputs:";
  if (bits & 1) m += " bag offsets must rise from 0 to the key count;";
  if (bits & 4) m += " valid lengths must equal the bag sizes;";
  if (bits & 2) m += " key outside the table's key space;";
  return m;
}

struct Prepared {
  uint64_t route = 0;
  unsigned F = 0;
  std::vector<unsigned> dims, pools, tables;
  std::vector<uint64_t> mine;       // [n][F][2] keys, kept bags of this rank's batch per owner
  std::vector<uint64_t> peer;       // [n][F][2] of every requester's part on this shard
  uint64_t* rpay = nullptr;         // received payload (device)
  cudaEvent_t ready = nullptr;      // on the input stream, after the payload exchange
};

struct Round {
  uint64_t route = 0, ticket = 0;
  unsigned F = 0;
  std::vector<unsigned> dims, pools, tables;
  std::vector<uint64_t> peer;
  std::vector<uint64_t> send_f, recv_f;   // floats of partials sent to requester r / from owner o
};

template <typename T>
T* DevAlloc(size_t count, cudaStream_t s) {
  void* p = nullptr;
  Cu(cudaMallocAsync(&p, std::max<size_t>(count * sizeof(T), 16), s));
  return static_cast<T*>(p);
}

}  // namespace

struct EpsB200Client {
  EpsB200Store* store = nullptr;
  EpsB200Comm* comm = nullptr;
  EpsB200Comm* input_comm = nullptr;
  unsigned rank = 0, n = 1;
  int device = 0;
  std::mutex mutex;
  std::map<uint64_t, Prepared> prepared;
  std::map<uint64_t, Round> rounds;
  uint64_t next = 1;
  long long* pinned = nullptr;
  size_t pinned_words = 0;
  std::vector<cudaEvent_t> events;

  cudaEvent_t Event() {
    if (!events.empty()) { cudaEvent_t e = events.back(); events.pop_back(); return e; }
    cudaEvent_t e;
    Cu(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    return e;
  }
  void Pinned(size_t words) {
    if (pinned_words >= words) return;
    if (pinned) Cu(cudaFreeHost(pinned));
    pinned = nullptr;
    pinned_words = 0;
    Cu(cudaMallocHost(reinterpret_cast<void**>(&pinned), words * sizeof(long long)));
    pinned_words = words;
  }
  void Alltoall(EpsB200Comm* c, const void* send, const std::vector<uint64_t>& sc, void* recv,
                const std::vector<uint64_t>& rc, unsigned elem, cudaStream_t s) {
    EpsB200Status st;
    Call(eps_b200_comm_alltoallv(c, send, sc.data(), recv, rc.data(), elem, s, &st), st);
  }
};

extern "C" {

int eps_b200_client_create(EpsB200Store* store, EpsB200Comm* comm, EpsB200Comm* input_comm,
                           EpsB200Client** out, EpsB200Status* status) {
  return Guard(status, [&] {
    Require(store && comm && out, "invalid client arguments");
    if (!input_comm) input_comm = comm;
    unsigned count = 0;
    const unsigned shard = eps_b200::store_shard(store, &count);
    Require(eps_b200::comm_rank(comm) == shard && eps_b200::comm_world(comm) == count &&
            eps_b200::comm_rank(input_comm) == shard && eps_b200::comm_world(input_comm) == count,
            "the store's shard id / count must be the communicators' rank / size");
    Require(eps_b200::comm_device(comm) == eps_b200::store_device(store) &&
            eps_b200::comm_device(input_comm) == eps_b200::store_device(store),
            "the communicators must be on the store's device");
    auto* c = new EpsB200Client;
    c->store = store;
    c->comm = comm;
    c->input_comm = input_comm;
    c->rank = shard;
    c->n = count;
    c->device = eps_b200::store_device(store);
    *out = c;
  });
}

void eps_b200_client_destroy(EpsB200Client* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  EpsB200Status st;
  for (auto& [id, p] : c->prepared) {
    eps_b200_route_release(c->store, p.route, &st);
    if (p.rpay) cudaFree(p.rpay);
    if (p.ready) cudaEventDestroy(p.ready);
  }
  for (auto& [id, r] : c->rounds) {
    if (r.route) eps_b200_route_release(c->store, r.route, &st);
    if (r.ticket) eps_b200_release(c->store, r.ticket, &st);
  }
  for (auto e : c->events) cudaEventDestroy(e);
  if (c->pinned) cudaFreeHost(c->pinned);
  delete c;
}

int eps_b200_client_prepare(EpsB200Client* c, const EpsB200Feature* features, uint64_t count,
                            void* input_stream, uint64_t* prepared_out, EpsB200Status* status) {
  return Guard(status, [&] {
    Require(c && features && prepared_out && count > 0 && count <= 1024, "invalid client prepare");
    std::lock_guard lock(c->mutex);
    Cu(cudaSetDevice(c->device));
    const unsigned n = c->n, F = (unsigned)count, width = 4 * F + 1;
    const cudaStream_t in = static_cast<cudaStream_t>(input_stream);
    Prepared P;
    P.F = F;
    for (unsigned f = 0; f < F; ++f) {
      unsigned d = 0;
      if (!eps_b200::store_table_dimension(c->store, features[f].table, &d)) d = 0;
      P.dims.push_back(d);
      P.pools.push_back(features[f].pooling);
      P.tables.push_back(features[f].table);
    }
    // ---- 1./2. partition and count rows [send | recv], one row per peer
    int64_t* rows = DevAlloc<int64_t>(2ull * n * width, in);
    std::string host_error;
    int host_code = 0;
    {
      EpsB200Status st;
      const int rc = eps_b200_route(c->store, features, count, n, in, &P.route, rows, &st);
      if (rc) {                      // shape error found on the host: still exchange
        host_code = rc;
        host_error = st.message;
        P.route = 0;
        std::vector<int64_t> h((size_t)n * width, 0);
        for (unsigned o = 0; o < n; ++o) {
          for (unsigned f = 0; f < F; ++f) {
            h[(size_t)o * width + 2 * F + f] = P.tables[f];
            h[(size_t)o * width + 3 * F + f] = P.pools[f];
          }
          h[(size_t)o * width + 4 * F] = -1;
        }
        Cu(cudaMemcpyAsync(rows, h.data(), h.size() * 8, cudaMemcpyHostToDevice, in));
      }
    }
    try {
      c->Alltoall(c->input_comm, rows, std::vector<uint64_t>(n, width), rows + (size_t)n * width,
                  std::vector<uint64_t>(n, width), 8, in);
      c->Pinned(2ull * n * width);
      Cu(cudaMemcpyAsync(c->pinned, rows, 2ull * n * width * 8, cudaMemcpyDeviceToHost, in));
      Cu(cudaStreamSynchronize(in));            // the one wait of a round
    } catch (...) {
      EpsB200Status st;
      if (P.route) eps_b200_route_release(c->store, P.route, &st);
      cudaFreeAsync(rows, in);
      throw;
    }
    Cu(cudaFreeAsync(rows, in));
    const long long* mine = c->pinned;
    const long long* recv = c->pinned + (size_t)n * width;
    bool peer_error = false, bad_schema = false;
    for (unsigned r = 0; r < n; ++r) {
      peer_error |= recv[(size_t)r * width + 4 * F] != 0;
      for (unsigned f = 0; f < F; ++f)
        bad_schema |= recv[(size_t)r * width + 2 * F + f] != P.tables[f] ||
                      recv[(size_t)r * width + 3 * F + f] != P.pools[f];
    }
    const long long own_bits = mine[4 * F];
    if (host_code || own_bits || peer_error || bad_schema) {
      EpsB200Status st;
      if (P.route) eps_b200_route_release(c->store, P.route, &st);
      if (host_code) throw Fail(host_code, host_error);
      if (own_bits) throw Fail(EPS_B200_INVALID_ARGUMENT, InputMessage(own_bits));
      throw Fail(EPS_B200_INVALID_ARGUMENT, bad_schema ? "ranks disagree on the feature schema"
                                                      : "a peer rank rejected its lookup inputs");
    }
    P.mine.resize((size_t)n * F * 2);
    P.peer.resize((size_t)n * F * 2);
    std::vector<uint64_t> send_words(n, 0), recv_words(n, 0);
    for (unsigned o = 0; o < n; ++o)
      for (unsigned f = 0; f < F; ++f)
        for (unsigned k = 0; k < 2; ++k) {
          P.mine[((size_t)o * F + f) * 2 + k] = (uint64_t)mine[(size_t)o * width + 2 * f + k];
          P.peer[((size_t)o * F + f) * 2 + k] = (uint64_t)recv[(size_t)o * width + 2 * f + k];
        }
    for (unsigned o = 0; o < n; ++o)
      for (unsigned f = 0; f < F; ++f) {
        send_words[o] += P.mine[((size_t)o * F + f) * 2] + 2 * P.mine[((size_t)o * F + f) * 2 + 1] + 1;
        recv_words[o] += P.peer[((size_t)o * F + f) * 2] + 2 * P.peer[((size_t)o * F + f) * 2 + 1] + 1;
      }
    // ---- 3. payload: keys / kept-bag offsets / valid lengths per owner
    uint64_t total_send = 0, total_recv = 0;
    for (unsigned o = 0; o < n; ++o) { total_send += send_words[o]; total_recv += recv_words[o]; }
    uint64_t* pay = nullptr;
    try {
      pay = DevAlloc<uint64_t>(total_send, in);
      P.rpay = DevAlloc<uint64_t>(total_recv, in);
      EpsB200Status st;
      Call(eps_b200_route_scatter(c->store, P.route, pay, in, &st), st);
      c->Alltoall(c->input_comm, pay, send_words, P.rpay, recv_words, 8, in);
      Cu(cudaFreeAsync(pay, in));
      pay = nullptr;
      P.ready = c->Event();
      Cu(cudaEventRecord(P.ready, in));
    } catch (...) {
      EpsB200Status st;
      eps_b200_route_release(c->store, P.route, &st);
      if (pay) cudaFreeAsync(pay, in);
      if (P.rpay) cudaFreeAsync(P.rpay, in);
      throw;
    }
    const uint64_t id = c->next++;
    c->prepared.emplace(id, std::move(P));
    *prepared_out = id;
  });
}

int eps_b200_client_lookup(EpsB200Client* c, uint64_t prepared, EpsB200Buffer* outputs,
                           int32_t read_only, void* stream_arg, uint64_t* round_out,
                           EpsB200Status* status) {
  return Guard(status, [&] {
    Require(c && outputs && (read_only || round_out), "invalid client lookup");
    std::lock_guard lock(c->mutex);
    Cu(cudaSetDevice(c->device));
    auto it = c->prepared.find(prepared);
    Require(it != c->prepared.end(), "unknown prepared batch");
    Prepared P = std::move(it->second);
    c->prepared.erase(it);
    const unsigned n = c->n, F = P.F;
    const cudaStream_t s = static_cast<cudaStream_t>(stream_arg);
    Cu(cudaStreamWaitEvent(s, P.ready, 0));
    c->events.push_back(P.ready);
    Round R;
    R.route = P.route;
    R.F = F;
    R.dims = P.dims;
    R.pools = P.pools;
    R.tables = P.tables;
    R.peer = P.peer;
    R.send_f.assign(n, 0);
    R.recv_f.assign(n, 0);
    for (unsigned o = 0; o < n; ++o)
      for (unsigned f = 0; f < F; ++f) {
        const size_t i = ((size_t)o * F + f) * 2 + (P.pools[f] == 2 ? 0 : 1);
        R.send_f[o] += P.peer[i] * P.dims[f];     // partials this shard returns to requester o
        R.recv_f[o] += P.mine[i] * P.dims[f];     // partials owner o returns to this rank
      }
    uint64_t ts = 0, tr = 0;
    for (unsigned o = 0; o < n; ++o) { ts += R.send_f[o]; tr += R.recv_f[o]; }
    float* part_send = nullptr;
    float* part_recv = nullptr;
    bool have_ticket = false;
    try {
      part_send = DevAlloc<float>(ts, s);
      part_recv = DevAlloc<float>(tr, s);
      EpsB200Status st;
      Call(eps_b200_serve(c->store, P.rpay, P.peer.data(), P.tables.data(), P.pools.data(), n, F,
                          read_only, part_send, s, &R.ticket, &st), st);
      have_ticket = !read_only;
      c->Alltoall(c->comm, part_send, R.send_f, part_recv, R.recv_f, 4, s);
      Call(eps_b200_route_merge(c->store, R.route, part_recv, outputs, s, &st), st);
    } catch (...) {
      EpsB200Status st;
      eps_b200_route_release(c->store, R.route, &st);
      if (have_ticket) eps_b200_release(c->store, R.ticket, &st);
      if (part_send) cudaFreeAsync(part_send, s);
      if (part_recv) cudaFreeAsync(part_recv, s);
      cudaFreeAsync(P.rpay, s);
      throw;
    }
    Cu(cudaFreeAsync(part_send, s));
    Cu(cudaFreeAsync(part_recv, s));
    Cu(cudaFreeAsync(P.rpay, s));
    if (read_only) {
      EpsB200Status st;
      Call(eps_b200_route_release(c->store, R.route, &st), st);
      if (round_out) *round_out = 0;
      return;
    }
    const uint64_t id = c->next++;
    c->rounds.emplace(id, std::move(R));
    *round_out = id;
  });
}

int eps_b200_client_push(EpsB200Client* c, uint64_t round, const EpsB200Buffer* gradients,
                         void* stream_arg, int32_t wait, EpsB200Status* status) {
  return Guard(status, [&] {
    Require(c && gradients, "invalid client push");
    std::lock_guard lock(c->mutex);
    Cu(cudaSetDevice(c->device));
    auto it = c->rounds.find(round);
    Require(it != c->rounds.end(), "unknown round");
    Round& R = it->second;
    const unsigned n = c->n;
    const cudaStream_t s = static_cast<cudaStream_t>(stream_arg);
    uint64_t ts = 0, tr = 0;
    for (unsigned o = 0; o < n; ++o) { ts += R.recv_f[o]; tr += R.send_f[o]; }
    float* send = DevAlloc<float>(ts, s);
    float* recv = DevAlloc<float>(tr, s);
    uint32_t* flag = DevAlloc<uint32_t>(1, s);
    int rc = 0;
    EpsB200Status st;
    try {
      Cu(cudaMemsetAsync(flag, 0, sizeof(uint32_t), s));
      Call(eps_b200_route_gather(c->store, R.route, gradients, send, flag, s, &st), st);
      Call(eps_b200_comm_allreduce_max(c->comm, flag, 1, s, &st), st);
      // gradient rows travel in the layout the partials came back in
      c->Alltoall(c->comm, send, R.recv_f, recv, R.send_f, 4, s);
      rc = eps_b200_serve_push(c->store, R.ticket, recv, R.peer.data(), R.tables.data(),
                               R.pools.data(), n, R.F, flag, s, wait, &st);
    } catch (...) {
      cudaFreeAsync(send, s); cudaFreeAsync(recv, s); cudaFreeAsync(flag, s);
      throw;
    }
    Cu(cudaFreeAsync(send, s));
    Cu(cudaFreeAsync(recv, s));
    Cu(cudaFreeAsync(flag, s));
    // a push rejected while waiting keeps the round (push again, or release)
    if (rc) throw Fail(rc, st.message);
    EpsB200Status st2;
    Call(eps_b200_route_release(c->store, R.route, &st2), st2);
    c->rounds.erase(it);
  });
}

int eps_b200_client_release(EpsB200Client* c, uint64_t handle, EpsB200Status* status) {
  return Guard(status, [&] {
    Require(c != nullptr, "invalid client");
    std::lock_guard lock(c->mutex);
    Cu(cudaSetDevice(c->device));
    EpsB200Status st;
    if (auto it = c->prepared.find(handle); it != c->prepared.end()) {
      Call(eps_b200_route_release(c->store, it->second.route, &st), st);
      Cu(cudaStreamWaitEvent(nullptr, it->second.ready, 0));
      Cu(cudaFreeAsync(it->second.rpay, nullptr));
      c->events.push_back(it->second.ready);
      c->prepared.erase(it);
      return;
    }
    auto it = c->rounds.find(handle);
    Require(it != c->rounds.end(), "unknown prepared batch or round");
    Call(eps_b200_route_release(c->store, it->second.route, &st), st);
    Call(eps_b200_release(c->store, it->second.ticket, &st), st);
    c->rounds.erase(it);
  });
}

}  // extern "C"
