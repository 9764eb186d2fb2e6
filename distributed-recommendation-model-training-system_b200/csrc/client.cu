// client.cu -- the host side of a multi-GPU round in C++: the reference's
// DistributedClient (include/eps/distributed_client.hpp:32-70) over one shard
// per GPU, with every rank both a client of its own batch and the shard of the
// keys k with k % n == rank.
//
//   prepare   route (partition by key % n, src/access/prepared_lookup.cpp:47-83)
//             -> count rows all-to-all -> an asynchronous copy of the counts to
//             the host; on the input stream and the input communicator, so the
//             next batch can be prepared while the current round's push runs.
//             The prepare returns at once: the batch's payload exchange (keys,
//             kept-bag offsets, valid lengths), which needs its counts on the
//             host, is issued by the NEXT prepare call (for every earlier batch
//             still pending) or by the batch's own lookup, whichever comes
//             first.  Both points are the same on every rank, so every rank
//             issues the same collectives in the same order; a caller that
//             prepares two batches ahead finds the counts long arrived and the
//             host never waits on fresh device work.
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
// errors travel in the count rows, so every rank sees the same error, at the
// batch's payload exchange, before any of its data moves; it is reported by
// the batch's lookup.  Exchange buffers come from the stream-ordered allocator.
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
  // first phase (prepare): the count rows, on their way to the host
  long long* counts = nullptr;      // pinned [2][n][5F + 1]: rows sent | rows received
  size_t counts_words = 0;
  cudaEvent_t counts_ready = nullptr;
  cudaStream_t in = nullptr;        // the input stream of the first phase
  int host_code = 0;                // this rank's shape error found on the host
  std::string host_error;
  // second phase (payload exchange)
  bool exchanged = false;
  int fail_code = 0;                // the batch's input error, reported by its lookup
  std::string fail_message;
  std::vector<uint64_t> mine;       // [n][F][3] keys, kept bags, distinct keys of this rank's batch per owner
  std::vector<uint64_t> peer;       // [n][F][3] of every requester's part on this shard
  uint64_t* rpay = nullptr;         // received payload (device)
  cudaEvent_t ready = nullptr;      // on the input stream, after the payload exchange
};

struct Round {
  uint64_t route = 0, ticket = 0;
  unsigned F = 0;
  std::vector<unsigned> dims, pools, tables;
  std::vector<uint64_t> peer;
  std::vector<uint64_t> send_f, recv_f;   // floats of partials sent to requester r / from owner o
  std::vector<uint64_t> gsend_f, grecv_f; // floats of gradients sent to owner o / from requester r
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
  std::vector<std::pair<long long*, size_t>> pinned;   // free pinned count buffers
  std::vector<cudaEvent_t> events;

  cudaEvent_t Event() {
    if (!events.empty()) { cudaEvent_t e = events.back(); events.pop_back(); return e; }
    cudaEvent_t e;
    Cu(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    return e;
  }
  // A pinned buffer of at least `words` (reused: allocating pinned memory is slow).
  std::pair<long long*, size_t> TakePinned(size_t words) {
    for (size_t i = 0; i < pinned.size(); ++i)
      if (pinned[i].second >= words) {
        auto b = pinned[i];
        pinned.erase(pinned.begin() + (long)i);
        return b;
      }
    long long* p = nullptr;
    Cu(cudaMallocHost(reinterpret_cast<void**>(&p), words * sizeof(long long)));
    return {p, words};
  }
  void GivePinned(Prepared& P) {
    if (P.counts) pinned.push_back({P.counts, P.counts_words});
    P.counts = nullptr;
    if (P.counts_ready) { events.push_back(P.counts_ready); P.counts_ready = nullptr; }
  }
  // The second phase of a prepared batch on `s` (which the count copy is
  // ordered before): read its counts, check the inputs of every rank, then the
  // payload exchange.  An input error is kept for the batch's lookup.
  void Exchange(Prepared& P, cudaStream_t s);
  // ---- exchange profile: CUDA events around every all-to-all on its stream,
  // and the bytes this rank sends to other ranks (EPS_B200_EXCHANGE_*)
  bool profiling = false;
  struct Pending { int kind; cudaEvent_t a, b; };
  std::vector<Pending> pending;
  std::vector<cudaEvent_t> timing_events;
  double ex_ms[EPS_B200_EXCHANGES] = {};
  uint64_t ex_bytes[EPS_B200_EXCHANGES] = {}, ex_calls[EPS_B200_EXCHANGES] = {};
  cudaEvent_t TimingEvent() {
    if (!timing_events.empty()) { cudaEvent_t e = timing_events.back(); timing_events.pop_back(); return e; }
    cudaEvent_t e;
    Cu(cudaEventCreate(&e));
    return e;
  }
  void Collect() {
    for (auto& x : pending) {
      Cu(cudaEventSynchronize(x.b));
      float ms = 0;
      Cu(cudaEventElapsedTime(&ms, x.a, x.b));
      ex_ms[x.kind] += ms;
      timing_events.push_back(x.a);
      timing_events.push_back(x.b);
    }
    pending.clear();
  }
  void Alltoall(EpsB200Comm* c, const void* send, const std::vector<uint64_t>& sc, void* recv,
                const std::vector<uint64_t>& rc, unsigned elem, cudaStream_t s, int kind) {
    EpsB200Status st;
    cudaEvent_t a = nullptr;
    if (profiling) { a = TimingEvent(); Cu(cudaEventRecord(a, s)); }
    Call(eps_b200_comm_alltoallv(c, send, sc.data(), recv, rc.data(), elem, s, &st), st);
    uint64_t out = 0;
    for (unsigned o = 0; o < sc.size(); ++o)
      if (o != rank) out += sc[o] * elem;
    ex_bytes[kind] += out;
    ++ex_calls[kind];
    if (a) {
      cudaEvent_t b = TimingEvent();
      Cu(cudaEventRecord(b, s));
      pending.push_back({kind, a, b});
    }
  }
};

void EpsB200Client::Exchange(Prepared& P, cudaStream_t s) {
  P.exchanged = true;
  Cu(cudaEventSynchronize(P.counts_ready));   // recorded a call ago: normally long done
  const unsigned F = P.F, width = 5 * F + 1;
  const long long* mine = P.counts;
  const long long* recv = P.counts + (size_t)n * width;
  bool peer_error = false, bad_schema = false;
  for (unsigned r = 0; r < n; ++r) {
    peer_error |= recv[(size_t)r * width + 5 * F] != 0;
    for (unsigned f = 0; f < F; ++f)
      bad_schema |= recv[(size_t)r * width + 2 * F + f] != P.tables[f] ||
                    recv[(size_t)r * width + 3 * F + f] != P.pools[f];
  }
  const long long own_bits = mine[5 * F];
  if (P.host_code || own_bits || peer_error || bad_schema) {
    EpsB200Status st;
    if (P.route) eps_b200_route_release(store, P.route, &st);
    P.route = 0;
    if (P.host_code) { P.fail_code = P.host_code; P.fail_message = P.host_error; }
    else if (own_bits) { P.fail_code = EPS_B200_INVALID_ARGUMENT; P.fail_message = InputMessage(own_bits); }
    else {
      P.fail_code = EPS_B200_INVALID_ARGUMENT;
      P.fail_message = bad_schema ? "ranks disagree on the feature schema"
                                  : "a peer rank rejected its lookup inputs";
    }
    GivePinned(P);
    return;
  }
  P.mine.resize((size_t)n * F * 3);
  P.peer.resize((size_t)n * F * 3);
  std::vector<uint64_t> send_words(n, 0), recv_words(n, 0);
  for (unsigned o = 0; o < n; ++o)
    for (unsigned f = 0; f < F; ++f) {
      for (unsigned k = 0; k < 2; ++k) {
        P.mine[((size_t)o * F + f) * 3 + k] = (uint64_t)mine[(size_t)o * width + 2 * f + k];
        P.peer[((size_t)o * F + f) * 3 + k] = (uint64_t)recv[(size_t)o * width + 2 * f + k];
      }
      P.mine[((size_t)o * F + f) * 3 + 2] = (uint64_t)mine[(size_t)o * width + 4 * F + f];
      P.peer[((size_t)o * F + f) * 3 + 2] = (uint64_t)recv[(size_t)o * width + 4 * F + f];
    }
  GivePinned(P);
  // payload words per (owner, feature): keys, kept-bag offsets (+1), lengths, and
  // [0, U, U distinct keys] for a deduplicated group
  auto words = [](const uint64_t* c) { return c[0] + 2 * c[1] + 1 + (c[2] ? c[2] + 2 : 0); };
  for (unsigned o = 0; o < n; ++o)
    for (unsigned f = 0; f < F; ++f) {
      send_words[o] += words(&P.mine[((size_t)o * F + f) * 3]);
      recv_words[o] += words(&P.peer[((size_t)o * F + f) * 3]);
    }
  // ---- 3. payload: keys / kept-bag offsets / valid lengths per owner
  uint64_t total_send = 0, total_recv = 0;
  for (unsigned o = 0; o < n; ++o) { total_send += send_words[o]; total_recv += recv_words[o]; }
  uint64_t* pay = nullptr;
  try {
    pay = DevAlloc<uint64_t>(total_send, s);
    P.rpay = DevAlloc<uint64_t>(total_recv, s);
    EpsB200Status st;
    Call(eps_b200_route_scatter(store, P.route, pay, s, &st), st);
    Alltoall(input_comm, pay, send_words, P.rpay, recv_words, 8, s, EPS_B200_EXCHANGE_KEYS);
    Cu(cudaFreeAsync(pay, s));
    pay = nullptr;
    P.ready = Event();
    Cu(cudaEventRecord(P.ready, s));
  } catch (...) {
    EpsB200Status st;
    eps_b200_route_release(store, P.route, &st);
    P.route = 0;
    if (pay) cudaFreeAsync(pay, s);
    if (P.rpay) cudaFreeAsync(P.rpay, s);
    P.rpay = nullptr;
    throw;
  }
}

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
    if (p.counts_ready) cudaEventSynchronize(p.counts_ready);
    if (p.route) eps_b200_route_release(c->store, p.route, &st);
    if (p.rpay) cudaFree(p.rpay);
    if (p.ready) cudaEventDestroy(p.ready);
    if (p.counts_ready) cudaEventDestroy(p.counts_ready);
    if (p.counts) cudaFreeHost(p.counts);
  }
  for (auto& [id, r] : c->rounds) {
    if (r.route) eps_b200_route_release(c->store, r.route, &st);
    if (r.ticket) eps_b200_release(c->store, r.ticket, &st);
  }
  for (auto e : c->events) cudaEventDestroy(e);
  for (auto& x : c->pending) { cudaEventDestroy(x.a); cudaEventDestroy(x.b); }
  for (auto e : c->timing_events) cudaEventDestroy(e);
  for (auto& b : c->pinned) cudaFreeHost(b.first);
  delete c;
}

int eps_b200_client_prepare(EpsB200Client* c, const EpsB200Feature* features, uint64_t count,
                            void* input_stream, uint64_t* prepared_out, EpsB200Status* status) {
  return Guard(status, [&] {
    Require(c && features && prepared_out && count > 0 && count <= 1024, "invalid client prepare");
    std::lock_guard lock(c->mutex);
    Cu(cudaSetDevice(c->device));
    const unsigned n = c->n, F = (unsigned)count, width = 5 * F + 1;
    const cudaStream_t in = static_cast<cudaStream_t>(input_stream);
    // first the payload exchanges of earlier batches still pending, oldest first
    // (their counts arrived a call ago): queued ahead of this batch's partition
    // and count exchange, so that the next lookup, which waits for its batch's
    // payload, does not also wait behind this batch's count all-to-all
    for (auto& [pid, Q] : c->prepared)
      if (!Q.exchanged) c->Exchange(Q, in);
    Prepared P;
    P.F = F;
    P.in = in;
    for (unsigned f = 0; f < F; ++f) {
      unsigned d = 0;
      if (!eps_b200::store_table_dimension(c->store, features[f].table, &d)) d = 0;
      P.dims.push_back(d);
      P.pools.push_back(features[f].pooling);
      P.tables.push_back(features[f].table);
    }
    // ---- 1./2. partition and count rows [send | recv], one row per peer
    int64_t* rows = DevAlloc<int64_t>(2ull * n * width, in);
    {
      EpsB200Status st;
      const int rc = eps_b200_route(c->store, features, count, n, in, &P.route, rows, &st);
      if (rc) {                      // shape error found on the host: still exchange
        P.host_code = rc;
        P.host_error = st.message;
        P.route = 0;
        std::vector<int64_t> h((size_t)n * width, 0);
        for (unsigned o = 0; o < n; ++o) {
          for (unsigned f = 0; f < F; ++f) {
            h[(size_t)o * width + 2 * F + f] = P.tables[f];
            h[(size_t)o * width + 3 * F + f] = P.pools[f];
          }
          h[(size_t)o * width + 5 * F] = -1;
        }
        Cu(cudaMemcpyAsync(rows, h.data(), h.size() * 8, cudaMemcpyHostToDevice, in));
        Cu(cudaStreamSynchronize(in));          // h is pageable and local
      }
    }
    try {
      c->Alltoall(c->input_comm, rows, std::vector<uint64_t>(n, width), rows + (size_t)n * width,
                  std::vector<uint64_t>(n, width), 8, in, EPS_B200_EXCHANGE_COUNTS);
      auto buf = c->TakePinned(2ull * n * width);
      P.counts = buf.first;
      P.counts_words = buf.second;
      Cu(cudaMemcpyAsync(P.counts, rows, 2ull * n * width * 8, cudaMemcpyDeviceToHost, in));
      P.counts_ready = c->Event();
      Cu(cudaEventRecord(P.counts_ready, in));
    } catch (...) {
      EpsB200Status st;
      if (P.route) eps_b200_route_release(c->store, P.route, &st);
      cudaFreeAsync(rows, in);
      throw;
    }
    Cu(cudaFreeAsync(rows, in));
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
    if (!it->second.exchanged) c->Exchange(it->second, it->second.in);
    Prepared P = std::move(it->second);
    c->prepared.erase(it);
    if (P.fail_code) throw Fail(P.fail_code, P.fail_message);
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
    R.gsend_f.assign(n, 0);
    R.grecv_f.assign(n, 0);
    for (unsigned o = 0; o < n; ++o)
      for (unsigned f = 0; f < F; ++f) {
        // rows of a (shard, feature) block: its keys (sequence) or kept bags;
        // the partials of a deduplicated group: its distinct keys
        const uint64_t* pe = &P.peer[((size_t)o * F + f) * 3];
        const uint64_t* mi = &P.mine[((size_t)o * F + f) * 3];
        const unsigned k = P.pools[f] == 2 ? 0 : 1;
        R.send_f[o] += (pe[2] ? pe[2] : pe[k]) * P.dims[f];   // partials returned to requester o
        R.recv_f[o] += (mi[2] ? mi[2] : mi[k]) * P.dims[f];   // partials owner o returns here
        R.gsend_f[o] += mi[k] * P.dims[f];                    // gradients sent to owner o
        R.grecv_f[o] += pe[k] * P.dims[f];                    // gradients received from requester o
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
      c->Alltoall(c->comm, part_send, R.send_f, part_recv, R.recv_f, 4, s, EPS_B200_EXCHANGE_PARTIALS);
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
    for (unsigned o = 0; o < n; ++o) { ts += R.gsend_f[o]; tr += R.grecv_f[o]; }
    float* send = DevAlloc<float>(ts, s);
    float* recv = DevAlloc<float>(tr, s);
    uint32_t* flag = DevAlloc<uint32_t>(2, s);       // non-finite flag, max |g| bits
    int rc = 0;
    EpsB200Status st;
    try {
      Cu(cudaMemsetAsync(flag, 0, 2 * sizeof(uint32_t), s));
      Call(eps_b200_route_gather(c->store, R.route, gradients, send, flag, s, &st), st);
      Call(eps_b200_comm_allreduce_max(c->comm, flag, 2, s, &st), st);
      // gradient rows: one per kept bag (or key) of every (shard, feature) block
      c->Alltoall(c->comm, send, R.gsend_f, recv, R.grecv_f, 4, s, EPS_B200_EXCHANGE_GRADIENTS);
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

int eps_b200_client_profile(EpsB200Client* c, int32_t mode, double* exchange_ms,
                            uint64_t* exchange_bytes, uint64_t* exchange_calls,
                            EpsB200Status* status) {
  return Guard(status, [&] {
    Require(c != nullptr, "invalid client");
    std::lock_guard lock(c->mutex);
    Cu(cudaSetDevice(c->device));
    c->Collect();
    for (int k = 0; k < EPS_B200_EXCHANGES; ++k) {
      if (exchange_ms) exchange_ms[k] = c->ex_ms[k];
      if (exchange_bytes) exchange_bytes[k] = c->ex_bytes[k];
      if (exchange_calls) exchange_calls[k] = c->ex_calls[k];
    }
    if (mode == 1) {
      for (int k = 0; k < EPS_B200_EXCHANGES; ++k) { c->ex_ms[k] = 0; c->ex_bytes[k] = 0; c->ex_calls[k] = 0; }
      c->profiling = true;
    } else if (mode == 0) {
      c->profiling = false;
    }
  });
}

int eps_b200_client_release(EpsB200Client* c, uint64_t handle, EpsB200Status* status) {
  return Guard(status, [&] {
    Require(c != nullptr, "invalid client");
    std::lock_guard lock(c->mutex);
    Cu(cudaSetDevice(c->device));
    EpsB200Status st;
    if (auto it = c->prepared.find(handle); it != c->prepared.end()) {
      Prepared& P = it->second;
      if (P.counts_ready) Cu(cudaEventSynchronize(P.counts_ready));
      if (P.route) Call(eps_b200_route_release(c->store, P.route, &st), st);
      if (P.ready) {
        Cu(cudaStreamWaitEvent(nullptr, P.ready, 0));
        c->events.push_back(P.ready);
      }
      if (P.rpay) Cu(cudaFreeAsync(P.rpay, nullptr));
      c->GivePinned(P);
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
