// runtime.cu -- host side of the B200 parameter store and its C ABI (eps_b200.h).
//
// Mirrors the shard contract of the reference (include/eps/parameter_service.hpp,
// src/server/service.cpp Lookup/Push/Release) and its C-ABI error convention
// (adapters/entropy/runtime_c.cpp:21-30): every call returns 0 or
// eps::Error::Code + 1 with a message.  All device work of one store is ordered
// on one stream at a time; switching streams inserts an event dependency.
//
// Lookup tickets (LookupReply::ticket, include/eps/types.hpp:151-156) own one
// stream-ordered device slab holding the occurrence list emitted by the lookup
// kernel and already sorted for the Push, the mean scales of every gradient row,
// and the Push scratch.  A rejected Push keeps its ticket (retryable, as
// tests/core_tests.cpp:98-105 of the reference requires); an accepted one retires
// it into a bounded completed history so a repeated Push is acknowledged
// without effect (src/server/service.cpp:241-245).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <unistd.h>
#include <cstring>
#include <deque>
#include <map>
#include <mutex>
#include <new>
#include <stdexcept>
#include <string>
#include <unordered_set>
#include <vector>

#include "eps_b200.h"
#include "kernels.cuh"

namespace eps_b200 {
namespace {

struct Failure : std::runtime_error {
  int code;
  Failure(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};
void Require(bool ok, const char* message, int code = EPS_B200_INVALID_ARGUMENT) {
  if (!ok) throw Failure(code, message);
}
// CUDA errors map as in the reference backend (src/cuda/cache_backend.cu:19-24).
void Cuda(cudaError_t e) {
  if (e != cudaSuccess)
    throw Failure(e == cudaErrorMemoryAllocation ? EPS_B200_CAPACITY_EXCEEDED : EPS_B200_RUN_FAILED,
                  cudaGetErrorString(e));
}

template <typename F>
int Boundary(EpsB200Status* status, F fn) noexcept {
  if (status) { status->code = 0; status->message[0] = 0; }
  auto fail = [&](int code, const char* message) {
    if (status) {
      status->code = code;
      std::strncpy(status->message, message, sizeof(status->message) - 1);
      status->message[sizeof(status->message) - 1] = 0;
    }
    return code;
  };
  try { fn(); return 0; }
  catch (const Failure& e) { return fail(e.code, e.what()); }
  catch (const std::bad_alloc&) { return fail(EPS_B200_CAPACITY_EXCEEDED, "native runtime allocation failed"); }
  catch (const std::exception& e) { return fail(EPS_B200_RUN_FAILED, e.what()); }
  catch (...) { return fail(EPS_B200_RUN_FAILED, "unknown native runtime failure"); }
}

unsigned bits_for(unsigned long long max_value) {
  unsigned b = 0;
  while (b < 64 && (max_value >> b)) ++b;
  return b;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct Table {
  EpsB200Table def{};
  float* state = nullptr;
  unsigned long long* updates = nullptr;
  DeviceTable* dtable = nullptr;
  unsigned long long rows = 0;      // slots (dense: of the key space; hashed: the capacity)
  unsigned long long bytes = 0;
  // hashed tables (def.key_space == 0): the id -> slot index
  bool hashed = false;
  HashIndex index{};                // host copy; its pointers are device memory
  HashIndex* dindex = nullptr;      // device copy, for the lookup kernels
  unsigned long long entries = 0;   // index entries (power of two)

  // Frees the table's device memory.
  void Free() {
    cudaFree(state); cudaFree(updates); cudaFree(dtable);
    if (hashed) {
      cudaFree(index.keys); cudaFree(index.slots); cudaFree(index.slot_keys);
      cudaFree(index.used); cudaFree(dindex);
    }
  }
  // Empties a hashed table's index (no key, no slot used); stream-ordered.
  void ClearIndex(cudaStream_t stream) const {
    if (!hashed) return;
    Cuda(cudaMemsetAsync(index.keys, 0xFF, entries * 8, stream));
    Cuda(cudaMemsetAsync(index.slots, 0xFF, (entries + 1) * 4, stream));
    Cuda(cudaMemsetAsync(index.used, 0, 16, stream));      // used + top
  }
};

// Per-ticket status block, laid out identically in the device slab and in the
// pinned host mirror so that one copy transfers it: the lookup-error word (set
// by the lookup / sort kernels) and the push control block.
struct StatusBlock {
  unsigned lookup_error;
  unsigned pad[63];
  PushControl control;
};
using HostStatus = StatusBlock;

struct Ticket {
  bool read_only = false;
  void* slab = nullptr;
  int slot = -1;
  bool push_in_flight = false;
  bool lookup_checked = false;
  cudaEvent_t done = nullptr;       // recorded after an enqueued push's status copy
  cudaEvent_t sorted = nullptr;     // recorded on the side stream after the coalescing sort
  // layout
  std::vector<unsigned> feature_ids, feature_tables, dims, ranks;
  std::vector<unsigned long long> grad_rows, scale_base;
  std::vector<unsigned> table_ids;
  std::vector<unsigned long long> table_occ;
  unsigned long long n = 0;
  unsigned slot_bits = 0, dim_max = 0;
  int key64 = 0;
  void* keys = nullptr;
  unsigned* srcs = nullptr;
  float* row_scale = nullptr;
  RowRec* rows = nullptr;          // the push's row plan (built after the sort)
  RowPlan* plan = nullptr;
  unsigned* seg_start = nullptr;
  unsigned* seg_total = nullptr;
  uint2* pieces = nullptr;
  unsigned max_pieces = 0;
  LongRecord* records = nullptr;
  PushControl* control = nullptr;
  unsigned* lookup_error = nullptr;
  StatusBlock* status = nullptr;
  PushTable* push_tables = nullptr;
  PushFeature* push_features = nullptr;
  unsigned long long* grad_prefix = nullptr;
  char* stage_end = nullptr;        // end of the span staged by a push
};

// A shard partition of one lookup (multi-GPU round), see eps_b200_route.
struct Route {
  char* slab = nullptr;
  cudaStream_t last = nullptr;          // stream of the latest call that used the route
  unsigned n = 0, F = 0;
  unsigned long long B = 0, N = 0, cells = 0;
  unsigned tiles = 0;
  std::vector<unsigned> dims, pooling;
  std::vector<unsigned long long> rows;           // [F] output rows (bags or keys)
  unsigned long long* row_total = nullptr;   // device: rows of all (shard, feature) blocks
  int has_sequence = 0;
  LookupFeature* desc = nullptr;
  unsigned *cnt = nullptr, *pk = nullptr, *pb = nullptr, *tile_k = nullptr, *tile_b = nullptr,
           *bounds = nullptr, *error = nullptr, *bag_map = nullptr, *pos_map = nullptr;
  unsigned long long *part_off = nullptr, *row_pre = nullptr;
  float** outs = nullptr;
  const float** grads = nullptr;
  // distinct rows of one-key groups (see RouteLaunch::dd_*)
  unsigned long long* dd_keys = nullptr;
  unsigned* dd_rank = nullptr;
  unsigned long long dd_mask = 0;
  unsigned *dd_count = nullptr, *dd_used = nullptr, *dd_idx = nullptr;
  unsigned long long *dd_off = nullptr, *dd_words = nullptr;
};

// Slab carve-out helper.
struct Carver {
  size_t offset = 0;
  template <typename T> size_t take(size_t count) {
    const size_t at = offset;
    offset = align256(offset + count * sizeof(T));
    return at;
  }
};

void choose_vec(const std::vector<unsigned>& dims, bool align16, bool /*align8*/, int* vec,
                int* group, int* iters) {
  unsigned dmax = 1;
  bool all4 = true;
  for (unsigned d : dims) { dmax = std::max(dmax, d); all4 &= d % 4 == 0; }
  Shape sh;
  Require(choose_shape(dmax, all4, align16, &sh),
          "embedding dimension/alignment not supported by this build", EPS_B200_CAPACITY_EXCEEDED);
  *vec = sh.vec;
  *group = sh.group;
  *iters = sh.iters;
}

}  // namespace
}  // namespace eps_b200

using namespace eps_b200;

struct EpsB200Store {
  EpsB200Options opt{};
  std::mutex mutex;
  cudaStream_t own = nullptr;
  // the coalescing sort of a lookup runs on `side`, concurrently with the
  // gather on the caller's stream: fork after the occurrence list; the ticket's
  // `sorted` event orders the push (and every call that reads the ticket) after it
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr;
  // a push's piece sums run on `side` concurrently with its prescan
  cudaEvent_t push_fork = nullptr, push_join = nullptr;
  cudaStream_t last = nullptr;
  cudaEvent_t last_done = nullptr;
  std::map<unsigned, Table> tables;
  std::map<unsigned long long, Ticket> tickets;
  std::map<unsigned long long, Route> routes;
  unsigned long long next_route = 1;
  std::deque<unsigned long long> completed_order;
  std::unordered_set<unsigned long long> completed;
  unsigned long long next_ticket = 1;
  HostStatus* host_status = nullptr;
  std::vector<int> free_slots;
  unsigned* sticky_error = nullptr;     // device: errors of read-only device lookups
  std::deque<unsigned long long> inflight;   // tickets whose push is enqueued, in order
  std::string deferred;                     // first error of a push settled by Poll
  std::vector<cudaEvent_t> sync_pool;       // timing-disabled events for completion checks
  unsigned long long allocated_state = 0;
  EpsB200Stats stats{};
  // ---- per-phase device timing (CUDA events on the launching stream)
  struct Pending { int phase; cudaEvent_t a, b; };
  bool profiling = false;
  std::vector<cudaEvent_t> event_pool;
  std::vector<Pending> pending;
  double phase_ms[EPS_B200_PHASES] = {};
  unsigned long long phase_launches[EPS_B200_PHASES] = {}, phase_calls[EPS_B200_PHASES] = {};

  cudaEvent_t Event() {
    if (!event_pool.empty()) { cudaEvent_t e = event_pool.back(); event_pool.pop_back(); return e; }
    cudaEvent_t e;
    Cuda(cudaEventCreate(&e));
    return e;
  }
  cudaEvent_t SyncEvent() {
    if (!sync_pool.empty()) { cudaEvent_t e = sync_pool.back(); sync_pool.pop_back(); return e; }
    cudaEvent_t e;
    Cuda(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    return e;
  }
  cudaEvent_t Begin(cudaStream_t stream) {
    if (!profiling) return nullptr;
    cudaEvent_t a = Event();
    Cuda(cudaEventRecord(a, stream));
    return a;
  }
  void End(int phase, cudaEvent_t a, cudaStream_t stream, unsigned launches) {
    stats.kernel_launches += launches;
    phase_launches[phase] += launches;
    ++phase_calls[phase];
    if (!a) return;
    cudaEvent_t b = Event();
    Cuda(cudaEventRecord(b, stream));
    pending.push_back({phase, a, b});
  }
  void Collect() {
    for (auto& x : pending) {
      Cuda(cudaEventSynchronize(x.b));
      float ms = 0;
      Cuda(cudaEventElapsedTime(&ms, x.a, x.b));
      phase_ms[x.phase] += ms;
      event_pool.push_back(x.a);
      event_pool.push_back(x.b);
    }
    pending.clear();
  }

  // ---- pinned staging ring for small host->device descriptor copies, so that
  // enqueueing a lookup/push never waits for the device (pageable copies would).
  static constexpr size_t kRing = 8u << 20;
  char* ring = nullptr;
  size_t ring_head = 0;
  struct Fence { size_t begin, end; cudaEvent_t done; };
  std::deque<Fence> fences;

  // Copies `bytes` from host `src` to device `dst` on `stream` through the ring.
  void Stage(void* dst, const void* src, size_t bytes, cudaStream_t stream) {
    if (!bytes) return;
    if (!ring || bytes > kRing / 4) {
      Cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, stream));
      return;
    }
    const size_t need = (bytes + 255) & ~size_t(255);
    if (ring_head + need > kRing) ring_head = 0;
    const size_t a = ring_head, b = ring_head + need;
    // wait for earlier copies that still read [a, b)
    while (!fences.empty()) {
      const Fence& f = fences.front();
      const bool overlap = f.begin < b && a < f.end;
      if (!overlap && cudaEventQuery(f.done) != cudaSuccess) break;
      Cuda(cudaEventSynchronize(f.done));
      event_pool.push_back(f.done);
      fences.pop_front();
    }
    std::memcpy(ring + a, src, bytes);
    Cuda(cudaMemcpyAsync(dst, ring + a, bytes, cudaMemcpyHostToDevice, stream));
    cudaEvent_t e = Event();
    Cuda(cudaEventRecord(e, stream));
    fences.push_back({a, b, e});
    ring_head = b;
  }

  void Activate() {
    Cuda(cudaSetDevice(opt.device));
    (void)cudaGetLastError();   // a launch check below must not see an older error
  }

  cudaStream_t Use(void* s) {
    cudaStream_t stream = s ? static_cast<cudaStream_t>(s) : own;
    if (last && last != stream) Cuda(cudaStreamWaitEvent(stream, last_done, 0));
    last = stream;
    return stream;
  }
  void Done(cudaStream_t stream) { Cuda(cudaEventRecord(last_done, stream)); }
  // Route calls touch no table state, only their inputs and their own slab, so
  // they run on the caller's stream without joining the store's stream order
  // (the partition of the next round can then overlap this round's push).
  cudaStream_t RouteStream(void* s) { return s ? static_cast<cudaStream_t>(s) : own; }
  void Sync(cudaStream_t stream) { Cuda(cudaStreamSynchronize(stream)); }

  Table& Get(unsigned id) {
    auto it = tables.find(id);
    Require(it != tables.end(), "unknown table");
    return it->second;
  }

  void FreeTicket(std::map<unsigned long long, Ticket>::iterator it, cudaStream_t stream) {
    if (it->second.sorted) {
      // the sort on the side stream writes the slab: release it after the sort
      cudaStreamWaitEvent(stream, it->second.sorted, 0);
      sync_pool.push_back(it->second.sorted);
      it->second.sorted = nullptr;
    }
    if (it->second.slab) cudaFreeAsync(it->second.slab, stream);
    if (it->second.slot >= 0) free_slots.push_back(it->second.slot);
    tickets.erase(it);
    stats.live_tickets = tickets.size();
  }

  void Complete(unsigned long long id) {
    completed.insert(id);
    completed_order.push_back(id);
    while (completed_order.size() > 4096) {
      completed.erase(completed_order.front());
      completed_order.pop_front();
    }
  }

  // Lookup-input errors recorded by the lookup kernel (LookupErrorBits).
  static std::string LookupMessage(unsigned bits) {
    if (bits & kLookupSortFailed) return "coalescing sort did not complete";
    if (bits & kLookupCapacity) return "hashed table capacity exceeded";
    if (bits & kLookupBadOffsets) return "invalid bag offsets";
    if (bits & kLookupShortLength) return "original bag length is smaller than shard contribution";
    return "key routed to wrong shard or outside the table";
  }
  // Push rejection reasons in the reference's order of checks.
  static std::string PushMessage(unsigned bits, unsigned lookup) {
    if (bits & 16u) return LookupMessage(lookup);
    if (bits & kRejectNonFiniteInput) return "non-finite gradient";
    if (bits & kRejectReduction) return "gradient reduction overflow";
    if (bits & kRejectLearningRate) return "optimizer learning-rate overflow";
    return "optimizer state would overflow";
  }

  // After the stream finished: settle an in-flight push of ticket `it`.
  // Returns an empty string when the push was accepted.
  std::string Resolve(std::map<unsigned long long, Ticket>::iterator it, cudaStream_t stream) {
    Ticket& t = it->second;
    const HostStatus& h = host_status[t.slot];
    t.push_in_flight = false;
    if (t.done) { sync_pool.push_back(t.done); t.done = nullptr; }
    if (h.control.accepted) {
      ++stats.updates;
      Complete(it->first);
      FreeTicket(it, stream);
      return {};
    }
    ++stats.rejected_updates;
    if (h.control.reject_bits & 16u) {
      // the lookup itself was invalid: the reference never issued a ticket
      const std::string m = LookupMessage(h.lookup_error);
      FreeTicket(it, stream);
      return m;
    }
    return PushMessage(h.control.reject_bits, h.lookup_error);
  }
  // Back-pressure for callers that enqueue rounds faster than the device runs
  // them: with kMaxInflight asynchronous pushes still enqueued, the host waits
  // for the oldest before the next lookup allocates its ticket, so that the
  // ticket memory of a steady stream of rounds stays bounded (and the
  // stream-ordered pool stops growing after the first rounds).
  static constexpr size_t kMaxInflight = 16;   // default of max_enqueued_pushes
  void Throttle(cudaStream_t stream) {
    const size_t limit = opt.max_enqueued_pushes ? opt.max_enqueued_pushes : kMaxInflight;
    while (inflight.size() >= limit) {
      auto it = tickets.find(inflight.front());
      if (it == tickets.end() || !it->second.push_in_flight) { inflight.pop_front(); continue; }
      Cuda(cudaEventSynchronize(it->second.done));
      Poll(stream);
    }
  }
  // Settles, without waiting, every enqueued push that the device has finished
  // (in enqueue order), so tickets of asynchronous pushes release their device
  // memory as soon as possible.  Rejections are reported by the next
  // eps_b200_synchronize.
  void Poll(cudaStream_t stream) {
    while (!inflight.empty()) {
      auto it = tickets.find(inflight.front());
      if (it == tickets.end() || !it->second.push_in_flight) { inflight.pop_front(); continue; }
      if (cudaEventQuery(it->second.done) != cudaSuccess) break;
      inflight.pop_front();
      const std::string m = Resolve(it, stream);
      if (!m.empty() && deferred.empty()) deferred = m;
    }
  }
};

namespace {

EpsB200Store* Checked(EpsB200Store* s) {
  Require(s != nullptr, "null native store");
  return s;
}

void ValidateTable(const EpsB200Store& s, const EpsB200Table& d) {
  Require(d.dimension > 0 && d.dimension <= 65536, "invalid embedding dimension");
  Require(d.dimension <= 128 || (d.dimension <= 512 && d.dimension % 4 == 0),
          "embedding dimension not supported by this build", EPS_B200_CAPACITY_EXCEEDED);
  Require(d.shard_count == s.opt.shard_count && d.partition_epoch == s.opt.partition_epoch,
          "table partition does not match server");
  if (d.has_weight_bounds)
    Require(std::isfinite(d.weight_min) && std::isfinite(d.weight_max) &&
                d.weight_min <= d.weight_max,
            "invalid optimizer weight bounds");
  Require(std::isfinite(d.learning_rate) && d.learning_rate > 0 && d.beta1 >= 0 && d.beta1 < 1 &&
              d.beta2 >= 0 && d.beta2 < 1 && std::isfinite(d.epsilon) && d.epsilon > 0 &&
              d.initial_beta1_power >= 0 && d.initial_beta1_power < 1 &&
              d.initial_beta2_power >= 0 && d.initial_beta2_power < 1,
          "invalid sparse LazyAdam configuration");
  Require(std::isfinite(d.initialization_min) && std::isfinite(d.initialization_max) &&
              d.initialization_min <= d.initialization_max,
          "invalid initializer bounds");
  Require(d.key_space > 0 || (d.capacity > 0 && d.capacity < 0xFFFFFFF0ull),
          "invalid key space (a hashed table, key space 0, needs a capacity below 2^32 - 16)");
}

bool SameTable(const EpsB200Table& a, const EpsB200Table& b) {
  return a.id == b.id && a.dimension == b.dimension && a.shard_count == b.shard_count &&
         a.partition_epoch == b.partition_epoch && a.learning_rate == b.learning_rate &&
         a.beta1 == b.beta1 && a.beta2 == b.beta2 && a.epsilon == b.epsilon &&
         a.initial_beta1_power == b.initial_beta1_power &&
         a.initial_beta2_power == b.initial_beta2_power &&
         a.has_weight_bounds == b.has_weight_bounds &&
         (!a.has_weight_bounds || (a.weight_min == b.weight_min && a.weight_max == b.weight_max)) &&
         a.initialization_min == b.initialization_min &&
         a.initialization_max == b.initialization_max &&
         a.initialization_seed == b.initialization_seed && a.key_space == b.key_space &&
         (a.key_space != 0 || a.capacity == b.capacity);
}

// Per-feature shape checks shared by every lookup entry point: the host half of
// ValidateFeature (src/access/batch_access.cpp:10-23); the keys and offsets
// themselves are checked by the kernels.  Returns the feature's output rows.
unsigned long long CheckFeatureShape(const EpsB200Feature& f) {
  Require(f.pooling <= 2, "unsupported pooling mode");
  Require(f.offset_count >= 1 && f.offsets, "invalid bag offsets");
  Require(f.offset_count > 1 || f.key_count == 0, "invalid bag offsets");
  Require(!f.key_count || f.keys, "null feature keys");
  Require(!f.has_padding || !f.valid_lengths,
          "valid lengths are derived from the padding key; pass one or the other");
  const unsigned long long rows = f.pooling == 2 ? f.key_count : f.offset_count - 1;
  Require(rows < (1ull << kRowBits) && f.key_count < (1ull << 31),
          "feature exceeds the per-feature row limit", EPS_B200_CAPACITY_EXCEEDED);
  return rows;
}

}  // namespace

extern "C" {

uint32_t eps_b200_abi_version(void) { return EPS_B200_ABI; }

int eps_b200_create(const EpsB200Options* options, EpsB200Store** out, EpsB200Status* status) {
  if (out) *out = nullptr;
  return Boundary(status, [&] {
    Require(options && out, "null store options/output");
    Require(options->shard_count > 0 && options->shard_count <= 1024 &&
                options->shard_id < options->shard_count,
            "invalid shard topology");
    int devices = 0;
    Cuda(cudaGetDeviceCount(&devices));
    Require(options->device >= 0 && options->device < devices, "invalid CUDA device",
            EPS_B200_UNAVAILABLE);
    auto s = new EpsB200Store();
    try {
      s->opt = *options;
      if (!s->opt.max_live_tickets) s->opt.max_live_tickets = 1024;
      s->Activate();
      // a blocking stream: work the caller queued on the legacy default stream
      // (e.g. framework tensor copies) is ordered before the store's own work
      Cuda(cudaStreamCreateWithFlags(&s->own, cudaStreamDefault));
      Cuda(cudaEventCreateWithFlags(&s->last_done, cudaEventDisableTiming));
      {
        // highest priority: the sort's blocks are scheduled ahead of the gather's
        int lowest = 0, greatest = 0;
        Cuda(cudaDeviceGetStreamPriorityRange(&lowest, &greatest));
        Cuda(cudaStreamCreateWithPriority(&s->side, cudaStreamNonBlocking, greatest));
      }
      Cuda(cudaEventCreateWithFlags(&s->fork, cudaEventDisableTiming));
      Cuda(cudaEventCreateWithFlags(&s->push_fork, cudaEventDisableTiming));
      Cuda(cudaEventCreateWithFlags(&s->push_join, cudaEventDisableTiming));
      // one status slot per live ticket plus a scratch slot (index max_live_tickets)
      Cuda(cudaMallocHost(&s->host_status, sizeof(HostStatus) * (s->opt.max_live_tickets + 1)));
      std::memset(s->host_status, 0, sizeof(HostStatus) * (s->opt.max_live_tickets + 1));
      for (int i = (int)s->opt.max_live_tickets - 1; i >= 0; --i) s->free_slots.push_back(i);
      Cuda(cudaMallocHost(&s->ring, EpsB200Store::kRing));
      Cuda(cudaMalloc(&s->sticky_error, sizeof(unsigned)));
      Cuda(cudaMemset(s->sticky_error, 0, sizeof(unsigned)));
      // keep freed ticket slabs in the stream-ordered pool for reuse
      cudaMemPool_t pool;
      Cuda(cudaDeviceGetDefaultMemPool(&pool, s->opt.device));
      unsigned long long threshold = ~0ull;
      Cuda(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold));
    } catch (...) {
      eps_b200_destroy(s);
      throw;
    }
    *out = s;
  });
}

void eps_b200_destroy(EpsB200Store* s) {
  if (!s) return;
  try {
    cudaSetDevice(s->opt.device);
    // the store's own completion event (recorded after every call's work, on
    // whatever stream the caller passed) and the store's own streams: no caller
    // stream is touched, so callers may destroy theirs first
    if (s->last && s->last_done) cudaEventSynchronize(s->last_done);
    if (s->side) cudaStreamSynchronize(s->side);
    if (s->own) cudaStreamSynchronize(s->own);
    for (auto& [id, t] : s->tickets) if (t.slab) cudaFree(t.slab);
    for (auto& [id, r] : s->routes) if (r.slab) cudaFree(r.slab);
    for (auto& [id, t] : s->tables) t.Free();
    for (auto& f : s->fences) cudaEventDestroy(f.done);
    if (s->ring) cudaFreeHost(s->ring);
    for (auto& x : s->pending) { cudaEventDestroy(x.a); cudaEventDestroy(x.b); }
    for (auto e : s->event_pool) cudaEventDestroy(e);
    for (auto e : s->sync_pool) cudaEventDestroy(e);
    for (auto& [id, t] : s->tickets) {
      if (t.done) cudaEventDestroy(t.done);
      if (t.sorted) cudaEventDestroy(t.sorted);
    }
    if (s->sticky_error) cudaFree(s->sticky_error);
    if (s->host_status) cudaFreeHost(s->host_status);
    if (s->last_done) cudaEventDestroy(s->last_done);
    if (s->side) cudaStreamDestroy(s->side);
    if (s->fork) cudaEventDestroy(s->fork);
    if (s->push_fork) cudaEventDestroy(s->push_fork);
    if (s->push_join) cudaEventDestroy(s->push_join);
    if (s->own) cudaStreamDestroy(s->own);
  } catch (...) {
  }
  delete s;
}

int eps_b200_create_table(EpsB200Store* store, const EpsB200Table* table, EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    Require(table != nullptr, "null table definition");
    std::lock_guard lock(s.mutex);
    s.Activate();
    const EpsB200Table d = *table;
    ValidateTable(s, d);
    if (auto it = s.tables.find(d.id); it != s.tables.end()) {
      Require(SameTable(it->second.def, d), "table already exists with different configuration");
      return;
    }
    Require(s.tables.size() < 1024, "table count exceeds limit", EPS_B200_CAPACITY_EXCEEDED);
    const unsigned long long shard = s.opt.shard_id, n = s.opt.shard_count;
    const bool hashed = d.key_space == 0;
    const unsigned long long rows =
        hashed ? d.capacity : d.key_space > shard ? (d.key_space - 1 - shard) / n + 1 : 0;
    Require(rows < 0xffffffffull, "key space exceeds the per-shard slot limit (2^32 - 1)",
            EPS_B200_CAPACITY_EXCEEDED);
    unsigned long long entries = 0;
    if (hashed) {
      entries = 1;
      while (entries < 2 * rows) entries <<= 1;        // at most half full
    }
    const unsigned long long bytes = rows * (12ull * d.dimension + 8) + entries * 12 + rows * 8;
    Require(s.opt.state_bytes >= s.allocated_state && bytes <= s.opt.state_bytes - s.allocated_state,
            "parameter-state budget exhausted", EPS_B200_CAPACITY_EXCEEDED);
    Table t;
    t.def = d;
    t.rows = rows;
    t.bytes = bytes;
    t.hashed = hashed;
    t.entries = entries;
    if (hashed) {
      try {
        Cuda(cudaMalloc(&t.state, std::max<size_t>(rows * 12ull * d.dimension, 16)));
        Cuda(cudaMalloc(&t.updates, std::max<size_t>(((rows + 1ull) & ~1ull) * 8ull, 16)));
        Cuda(cudaMalloc(&t.dtable, sizeof(DeviceTable)));
        HashIndex& h = t.index;
        Cuda(cudaMalloc(&h.keys, entries * 8));
        Cuda(cudaMalloc(&h.slots, (entries + 1) * 4));
        Cuda(cudaMalloc(&h.slot_keys, std::max<size_t>(rows * 8, 8)));
        Cuda(cudaMalloc(&h.used, 16));               // used (u64) | top (u32)
        h.top = reinterpret_cast<unsigned*>(h.used + 1);
        h.mask = entries - 1;
        h.capacity = rows;
        h.state = t.state;
        h.updates = t.updates;
        h.dim = d.dimension;
        h.table_id = d.id;
        h.seed = d.initialization_seed;
        h.init_min = d.initialization_min;
        h.init_max = d.initialization_max;
        h.has_bounds = d.has_weight_bounds;
        h.bound_min = d.weight_min;
        h.bound_max = d.weight_max;
        Cuda(cudaMalloc(&t.dindex, sizeof(HashIndex)));
        Cuda(cudaMemcpy(t.dindex, &h, sizeof(HashIndex), cudaMemcpyHostToDevice));
        t.ClearIndex(s.own);
        DeviceTable dt{};
        dt.beta1_power = d.initial_beta1_power;
        dt.beta2_power = d.initial_beta2_power;
        float bound = std::max(std::fabs(d.initialization_min), std::fabs(d.initialization_max));
        if (d.has_weight_bounds)
          bound = std::max(bound, std::max(std::fabs(d.weight_min), std::fabs(d.weight_max)));
        std::memcpy(&dt.state_absmax_bits, &bound, sizeof(bound));
        Cuda(cudaMemcpy(t.dtable, &dt, sizeof(dt), cudaMemcpyHostToDevice));
        Cuda(cudaStreamSynchronize(s.own));
      } catch (...) {
        t.Free();
        throw;
      }
      s.allocated_state += bytes;
      s.stats.state_bytes = s.allocated_state;
      s.stats.rows += rows;
      s.stats.tables = s.tables.size() + 1;
      s.tables.emplace(d.id, t);
      return;
    }
    try {
      Cuda(cudaMalloc(&t.state, std::max<size_t>(rows * 12ull * d.dimension, 16)));
      // an even number of counters: the ring push reads the 16-byte block of two
      Cuda(cudaMalloc(&t.updates, std::max<size_t>(((rows + 1ull) & ~1ull) * 8ull, 16)));
      Cuda(cudaMalloc(&t.dtable, sizeof(DeviceTable)));
      DeviceTable dt{};
      dt.beta1_power = d.initial_beta1_power;
      dt.beta2_power = d.initial_beta2_power;
      dt.optimizer_sequence = 0;
      float bound = std::max(std::fabs(d.initialization_min), std::fabs(d.initialization_max));
      if (d.has_weight_bounds)
        bound = std::max(bound, std::max(std::fabs(d.weight_min), std::fabs(d.weight_max)));
      std::memcpy(&dt.state_absmax_bits, &bound, sizeof(bound));
      Cuda(cudaMemcpy(t.dtable, &dt, sizeof(dt), cudaMemcpyHostToDevice));
      InitLaunch p{t.state, t.updates, rows, d.dimension, s.opt.shard_count, s.opt.shard_id,
                   d.id, d.initialization_seed, d.initialization_min, d.initialization_max,
                   d.has_weight_bounds, d.weight_min, d.weight_max};
      Cuda(launch_init(p, s.own));
      Cuda(cudaStreamSynchronize(s.own));
    } catch (...) {
      t.Free();
      throw;
    }
    s.allocated_state += bytes;
    s.stats.state_bytes = s.allocated_state;
    s.stats.rows += rows;
    s.stats.tables = s.tables.size() + 1;
    s.tables.emplace(d.id, t);
  });
}

int eps_b200_lookup(EpsB200Store* store, const EpsB200Feature* features, uint64_t count,
                    int32_t input_on_device, int32_t read_only, int32_t shard_partial,
                    EpsB200Buffer* outputs, void* stream_arg, uint64_t* ticket_out,
                    EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    Require(features && count > 0 && count <= kMaxFeatures, "invalid native feature count");
    // no outputs: a push-only lookup (the occurrence list and its coalescing
    // sort, no gather) for a caller that pushes gradients of rows it already holds
    const bool gather = outputs != nullptr;
    Require(gather || !read_only, "a read-only lookup needs output buffers");
    Require(read_only || ticket_out, "null ticket output");
    std::lock_guard lock(s.mutex);
    s.Activate();
    if (!read_only)
      Require(s.tickets.size() < s.opt.max_live_tickets && !s.free_slots.empty(),
              "live ticket limit reached", EPS_B200_CAPACITY_EXCEEDED);
    Require(shard_partial || s.opt.shard_count == 1,
            "a client-level lookup needs a single-shard store");

    // ---- host-side validation of shapes (O(features)); keys/offsets are
    // validated by the lookup kernel itself.
    std::map<unsigned, unsigned> ranks;   // table id -> rank (ascending id)
    std::unordered_set<unsigned> ids;
    unsigned long long total_keys = 0, total_offsets = 0, total_lengths = 0, total_rows = 0,
                       host_out_values = 0, bags = 0;
    std::vector<unsigned> dims;
    bool out16 = true, out8 = true, any_host_out = false, any_padding = false, any_hashed = false;
    for (uint64_t i = 0; i < count; ++i) {
      const auto& f = features[i];
      Require(ids.insert(f.feature).second, "duplicate feature ID");
      const Table& t = s.Get(f.table);
      const unsigned long long rows = CheckFeatureShape(f);
      any_padding |= f.has_padding != 0;
      any_hashed |= t.hashed;
      if (gather) {
        const auto& o = outputs[i];
        Require(o.feature == f.feature && o.rows == rows && o.columns == t.def.dimension,
                "output buffer layout mismatch");
        // a null buffer in a lookup that will be pushed makes that feature
        // push-only (its occurrences are listed, nothing is gathered)
        Require(!rows || o.data || !read_only, "null output buffer");
        Require(o.device < 0 || o.device == s.opt.device, "output device mismatch");
        if (!o.data) {
        } else if (o.device < 0) { any_host_out = true; host_out_values += rows * t.def.dimension; }
        else {
          out16 &= (reinterpret_cast<uintptr_t>(o.data) & 15) == 0;
          out8 &= (reinterpret_cast<uintptr_t>(o.data) & 7) == 0;
        }
      }
      ranks.emplace(f.table, 0);
      total_keys += f.key_count;
      total_offsets += f.offset_count;
      if (f.valid_lengths) total_lengths += f.offset_count - 1;
      total_rows += rows;
      bags += f.offset_count - 1;
      dims.push_back(t.def.dimension);
    }
    Require(total_keys < (1ull << 32), "lookup exceeds the occurrence limit",
            EPS_B200_CAPACITY_EXCEEDED);
    {
      unsigned r = 0;
      for (auto& [id, rank] : ranks) rank = r++;
    }
    unsigned long long max_rows = 1;
    unsigned dim_max = 1;
    for (auto& [id, rank] : ranks) {
      max_rows = std::max(max_rows, s.Get(id).rows);
      dim_max = std::max(dim_max, s.Get(id).def.dimension);
    }
    const unsigned slot_bits = std::max(1u, bits_for(max_rows - 1));
    const unsigned table_bits = bits_for(ranks.size() - 1);
    // padding occurrences get the composite key (table rank = 2^table_bits, slot 0):
    // one more bit, sorted after every row key, skipped by the push
    const unsigned key_bits = slot_bits + table_bits + (any_padding ? 1u : 0u);
    const int key64 = key_bits > 32;
    const size_t key_bytes = key64 ? 8 : 4;
    int vec, group, iters;
    choose_vec(dims, out16, out8, &vec, &group, &iters);

    // ---- slab layout
    Carver c;
    const size_t at_desc = c.take<LookupFeature>(count);
    size_t at_keys = 0, at_offsets = 0, at_lengths = 0, at_hostout = 0;
    if (!input_on_device) {
      at_keys = c.take<unsigned long long>(total_keys);
      at_offsets = c.take<unsigned long long>(total_offsets);
      at_lengths = c.take<unsigned long long>(total_lengths);
    }
    if (any_host_out) at_hostout = c.take<float>(host_out_values);
    // the resolved slots of hashed features' occurrences
    const size_t at_slots = any_hashed ? c.take<unsigned>(total_keys) : 0;
    const unsigned stiles = sort_tiles(total_keys);
    // pieces: one per row with 2..kLongRun occurrences (at most total_keys / 2
    // rows) and ceil(len / kPiece) per longer row
    const unsigned long long max_long = total_keys / (kLongRun + 1) + 1;
    const unsigned long long max_pieces = (total_keys + kPiece - 1) / kPiece + max_long + total_keys / 2;
    size_t at_k0 = 0, at_k1 = 0, at_s0 = 0, at_s1 = 0, at_scale = 0, at_hist = 0, at_seg = 0,
           at_segtot = 0, at_segscr = 0, at_pieces = 0, at_rec = 0, at_rows = 0,
           at_plan = 0,
           at_ptab = 0, at_pfeat = 0, at_gpre = 0, at_end = 0;
    size_t at_zero = 0;   // start of the region zeroed by the lookup's single memset
    if (!read_only) {
      at_k0 = c.take<char>(total_keys * key_bytes);
      at_k1 = c.take<char>(total_keys * key_bytes);
      at_s0 = c.take<unsigned>(total_keys);
      at_s1 = c.take<unsigned>(total_keys);
      at_scale = c.take<float>(total_rows);
      at_seg = c.take<unsigned>(total_keys + 1);
      at_segtot = c.take<unsigned>(1);
      at_pieces = c.take<uint2>(max_pieces);
      at_rec = c.take<LongRecord>(max_long);
      at_rows = c.take<RowRec>(total_keys);
      // [sort scratch | segment scratch | row plan counts | status] zeroed together
      at_zero = at_hist = c.take<char>(sort_scratch_bytes(total_keys, key_bits));
      at_segscr = c.take<char>(segment_scratch_bytes(total_keys));
      at_plan = c.take<RowPlan>(1);
    }
    const size_t at_status = c.take<StatusBlock>(1);
    if (read_only) at_zero = at_status;
    const size_t zero_bytes = c.offset - at_zero;
    if (!read_only) {
      // [status.control | push tables | push features | gradient prefix] staged by one copy
      at_ptab = c.take<PushTable>(ranks.size());
      at_pfeat = c.take<PushFeature>(count);
      at_gpre = c.take<unsigned long long>(count + 1);
      at_end = c.offset;
    }
    cudaStream_t stream = s.Use(stream_arg);
    s.Poll(stream);
    s.Throttle(stream);
    char* slab = nullptr;
    Cuda(cudaMallocAsync(reinterpret_cast<void**>(&slab), std::max<size_t>(c.offset, 256), stream));
    auto P = [&](size_t at) { return slab + at; };
    try {
      StatusBlock* status_block = reinterpret_cast<StatusBlock*>(P(at_status));
      unsigned* err = &status_block->lookup_error;
      Cuda(cudaMemsetAsync(P(at_zero), 0, zero_bytes, stream));
      // ---- descriptors (and staging of host inputs)
      std::vector<LookupFeature> desc(count);
      Ticket t;
      t.read_only = read_only != 0;
      unsigned long long bag_base = 0, occ_base = 0, scale_base = 0, koff = 0,
                         ooff = 0, loff = 0, hoff = 0, unit_base = 0, emit_base = 0;
      t.table_ids.resize(ranks.size());
      t.table_occ.assign(ranks.size(), 0);
      for (auto& [id, rank] : ranks) t.table_ids[rank] = id;
      for (uint64_t i = 0; i < count; ++i) {
        const auto& f = features[i];
        const Table& tab = s.Get(f.table);
        const unsigned D = tab.def.dimension;
        LookupFeature& L = desc[i];
        const unsigned long long rows = f.pooling == 2 ? f.key_count : f.offset_count - 1;
        if (input_on_device) {
          L.keys = reinterpret_cast<const unsigned long long*>(f.keys);
          L.offsets = reinterpret_cast<const unsigned long long*>(f.offsets);
          L.lengths = reinterpret_cast<const unsigned long long*>(f.valid_lengths);
        } else {
          auto* kd = reinterpret_cast<unsigned long long*>(P(at_keys)) + koff;
          auto* od = reinterpret_cast<unsigned long long*>(P(at_offsets)) + ooff;
          if (f.key_count) Cuda(cudaMemcpyAsync(kd, f.keys, f.key_count * 8, cudaMemcpyHostToDevice, stream));
          Cuda(cudaMemcpyAsync(od, f.offsets, f.offset_count * 8, cudaMemcpyHostToDevice, stream));
          L.keys = kd; L.offsets = od; L.lengths = nullptr;
          if (f.valid_lengths) {
            auto* ld = reinterpret_cast<unsigned long long*>(P(at_lengths)) + loff;
            if (f.offset_count > 1)
              Cuda(cudaMemcpyAsync(ld, f.valid_lengths, (f.offset_count - 1) * 8,
                                   cudaMemcpyHostToDevice, stream));
            L.lengths = ld;
            loff += f.offset_count - 1;
          }
          koff += f.key_count;
          ooff += f.offset_count;
        }
        if (!gather || !outputs[i].data) {
          L.out = nullptr;
        } else if (outputs[i].device < 0) {
          L.out = reinterpret_cast<float*>(P(at_hostout)) + hoff;
          hoff += rows * D;
        } else {
          L.out = static_cast<float*>(outputs[i].data);
        }
        L.state = tab.state;
        L.rows = tab.rows;
        L.key_count = f.key_count;
        L.bag_count = f.offset_count - 1;
        L.bag_base = bag_base;
        L.occ_base = occ_base;
        L.scale_base = scale_base;
        L.dim = D;
        L.pooling = f.pooling;
        L.table_rank = ranks.at(f.table);
        L.feature_index = (unsigned)i;
        L.has_padding = f.has_padding ? 1u : 0u;
        L.padding_key = f.padding_key;
        L.hash = tab.hashed ? tab.dindex : nullptr;
        L.slots = tab.hashed ? reinterpret_cast<unsigned*>(P(at_slots)) + occ_base : nullptr;
        L.unit_bags = feature_unit_bags(f.pooling, f.key_count, L.bag_count, (unsigned)group);
        L.unit_base = unit_base;
        L.units = L.out ? feature_units(f.pooling, f.key_count, L.bag_count, L.unit_bags) : 0;
        unit_base += L.units;
        L.emit_base = emit_base;
        L.emit_units = feature_units(f.pooling, f.key_count, L.bag_count,
                                     emit_unit_bags(f.key_count, L.bag_count));
        emit_base += L.emit_units;
        bag_base += L.bag_count;
        occ_base += f.key_count;
        scale_base += rows;
        t.feature_ids.push_back(f.feature);
        t.feature_tables.push_back(f.table);
        t.dims.push_back(D);
        t.ranks.push_back(L.table_rank);
        t.grad_rows.push_back(rows);
        t.scale_base.push_back(L.scale_base);
        t.table_occ[L.table_rank] += f.key_count;
      }
      s.Stage(P(at_desc), desc.data(), count * sizeof(LookupFeature), stream);
      LookupLaunch lp{};
      lp.features = reinterpret_cast<const LookupFeature*>(P(at_desc));
      lp.feature_count = (unsigned)count;
      lp.bag_total = bag_base;
      lp.unit_total = unit_base;
      lp.emit_total = emit_base;
      lp.shard_count = s.opt.shard_count;
      lp.shard_id = s.opt.shard_id;
      lp.client = shard_partial ? 0 : 1;
      lp.slot_bits = slot_bits;
      lp.key64 = key64;
      lp.pad_key = 1ull << (slot_bits + table_bits);
      lp.error = read_only && input_on_device && !any_host_out ? s.sticky_error : err;
      lp.vec = vec;
      lp.group = group;
      lp.iters = iters;
      if (any_hashed) {
        // keys of hashed tables -> slots, creating the rows of unseen keys
        ResolveLaunch rp{lp.features, (unsigned)count, total_keys, s.opt.shard_count,
                         s.opt.shard_id, reinterpret_cast<unsigned*>(P(at_slots)), lp.error};
        Cuda(launch_resolve(rp, stream));
        s.stats.kernel_launches += total_keys ? 2 : 0;
      }
      if (!read_only) {
        lp.occ_key = P(at_k0);
        lp.occ_src = reinterpret_cast<unsigned*>(P(at_s0));
        lp.row_scale = reinterpret_cast<float*>(P(at_scale));
        // the sort's digit histograms are counted by the emit kernel (the sort
        // scratch they start was zeroed above)
        lp.digit_hist = reinterpret_cast<unsigned*>(P(at_hist));
        lp.digit_passes = (key_bits + 7) / 8;
      }
      cudaEvent_t ev = nullptr;
      if (!read_only) {
        // the occurrence list first; the gather below does not emit, and the
        // sort (histograms, digit passes, segment compaction) runs on the side
        // stream concurrently with the gather
        ev = s.Begin(stream);
        Cuda(launch_emit(lp, stream));
        s.End(EPS_B200_PHASE_EMIT, ev, stream, emit_base ? 1u : 0u);
        Cuda(cudaEventRecord(s.fork, stream));
      }
      if (gather) {
        ev = s.Begin(stream);
        Cuda(launch_lookup(lp, stream));
        s.End(EPS_B200_PHASE_LOOKUP, ev, stream, unit_base ? 1u : 0u);
      }
      // ---- host outputs: final once the gather ends; their copies overlap the
      // sort, which runs on the side stream
      hoff = 0;
      for (uint64_t i = 0; gather && i < count; ++i) {
        if (outputs[i].device >= 0 || !outputs[i].data) continue;
        const unsigned long long n = outputs[i].rows * outputs[i].columns;
        if (n)
          Cuda(cudaMemcpyAsync(outputs[i].data, reinterpret_cast<float*>(P(at_hostout)) + hoff,
                               n * 4, cudaMemcpyDeviceToHost, stream));
        hoff += n;
      }
      if (!read_only) {
        cudaStream_t sort_stream = s.side;
        Cuda(cudaStreamWaitEvent(s.side, s.fork, 0));
        SortLaunch sp{P(at_k0), P(at_k1), reinterpret_cast<unsigned*>(P(at_s0)),
                      reinterpret_cast<unsigned*>(P(at_s1)), total_keys, key_bits,
                      key64, reinterpret_cast<unsigned*>(P(at_hist)), stiles, err, 1};
        int swapped = 0;
        ev = s.Begin(sort_stream);
        Cuda(launch_sort(sp, sort_stream, &swapped));
        SegmentLaunch gl{swapped ? P(at_k1) : P(at_k0), total_keys, key64,
                         reinterpret_cast<unsigned*>(P(at_seg)),
                         reinterpret_cast<unsigned*>(P(at_segtot)),
                         reinterpret_cast<unsigned*>(P(at_segscr)), err};
        Cuda(launch_segments(gl, sort_stream));
        PlanLaunch pp{};
        pp.keys = swapped ? P(at_k1) : P(at_k0);
        pp.srcs = reinterpret_cast<const unsigned*>(swapped ? P(at_s1) : P(at_s0));
        pp.seg_start = reinterpret_cast<const unsigned*>(P(at_seg));
        pp.seg_total = reinterpret_cast<const unsigned*>(P(at_segtot));
        pp.features = lp.features;
        pp.feature_count = (unsigned)count;
        pp.row_scale = reinterpret_cast<const float*>(P(at_scale));
        pp.n = total_keys;
        pp.key64 = key64;
        pp.slot_bits = slot_bits;
        pp.table_count = (unsigned)ranks.size();
        pp.long_run = (s.opt.flags & EPS_B200_FLAG_REFERENCE_ORDER) ? ~0ull : (unsigned long long)kLongRun;
        pp.rows = reinterpret_cast<RowRec*>(P(at_rows));
        pp.plan = reinterpret_cast<RowPlan*>(P(at_plan));
        pp.pieces = reinterpret_cast<uint2*>(P(at_pieces));
        pp.longs = reinterpret_cast<LongRecord*>(P(at_rec));
        Cuda(launch_row_plan(pp, sort_stream));
        s.End(EPS_B200_PHASE_SORT, ev, sort_stream,
              sort_launch_count(sp) + segment_launch_count(total_keys) + (total_keys ? 1u : 0u));
        // the caller's stream does not wait for the sort: the lookup's outputs
        // are final when the gather ends; the push (and every call that reads
        // the ticket) waits for this event
        t.sorted = s.SyncEvent();
        Cuda(cudaEventRecord(t.sorted, s.side));
        t.keys = swapped ? P(at_k1) : P(at_k0);
        t.srcs = reinterpret_cast<unsigned*>(swapped ? P(at_s1) : P(at_s0));
        t.n = total_keys;
        t.slot_bits = slot_bits;
        t.key64 = key64;
        t.dim_max = dim_max;
        t.row_scale = reinterpret_cast<float*>(P(at_scale));
        t.seg_start = reinterpret_cast<unsigned*>(P(at_seg));
        t.seg_total = reinterpret_cast<unsigned*>(P(at_segtot));
        t.pieces = reinterpret_cast<uint2*>(P(at_pieces));
        t.max_pieces = (unsigned)max_pieces;
        t.records = reinterpret_cast<LongRecord*>(P(at_rec));
        t.rows = reinterpret_cast<RowRec*>(P(at_rows));
        t.plan = reinterpret_cast<RowPlan*>(P(at_plan));
        t.status = status_block;
        t.control = &status_block->control;
        t.lookup_error = err;
        t.push_tables = reinterpret_cast<PushTable*>(P(at_ptab));
        t.push_features = reinterpret_cast<PushFeature*>(P(at_pfeat));
        t.grad_prefix = reinterpret_cast<unsigned long long*>(P(at_gpre));
        t.stage_end = P(at_end);
      }
      const bool synchronous = !input_on_device || any_host_out;
      int slot = -1;
      if (!read_only) {
        slot = s.free_slots.back();
        s.free_slots.pop_back();
        std::memset(&s.host_status[slot], 0, sizeof(HostStatus));
        if (synchronous)
          Cuda(cudaMemcpyAsync(&s.host_status[slot].lookup_error, err, sizeof(unsigned),
                               cudaMemcpyDeviceToHost, stream));
      }
      unsigned sync_err = 0;
      if (synchronous && t.sorted) Cuda(cudaStreamWaitEvent(stream, t.sorted, 0));
      if (synchronous) {
        HostStatus& scratch = s.host_status[s.opt.max_live_tickets];
        if (read_only)
          Cuda(cudaMemcpyAsync(&scratch.lookup_error, err, sizeof(unsigned),
                               cudaMemcpyDeviceToHost, stream));
        s.Sync(stream);
        sync_err = read_only ? scratch.lookup_error : s.host_status[slot].lookup_error;
      }
      ++s.stats.lookups;
      if (read_only || sync_err) {
        if (slot >= 0) s.free_slots.push_back(slot);
        if (t.sorted) { s.sync_pool.push_back(t.sorted); t.sorted = nullptr; }
        char* owned = slab;
        slab = nullptr;                 // freed exactly once, here
        Cuda(cudaFreeAsync(owned, stream));
        s.Done(stream);
        Require(!sync_err, EpsB200Store::LookupMessage(sync_err).c_str(),
                (sync_err & kLookupCapacity) ? EPS_B200_CAPACITY_EXCEEDED
                                             : EPS_B200_INVALID_ARGUMENT);
        return;
      }
      t.slab = slab;
      t.slot = slot;
      t.lookup_checked = synchronous;
      const unsigned long long id = s.next_ticket++;
      s.tickets.emplace(id, std::move(t));
      s.stats.live_tickets = s.tickets.size();
      slab = nullptr;                   // owned by the ticket now
      *ticket_out = id;
      s.Done(stream);
    } catch (...) {
      cudaStreamSynchronize(stream);
      cudaStreamSynchronize(s.side);
      if (slab) cudaFreeAsync(slab, stream);
      throw;
    }
  });
}

// Read-only pooled lookup that allocates nothing: see eps_b200.h.  Same kernel
// and same results as eps_b200_lookup(read_only=1, shard_partial=0) with device
// inputs and outputs; only the feature descriptors live elsewhere (noalloc.cu).
int eps_b200_lookup_noalloc(EpsB200Store* store, const EpsB200Feature* features, uint64_t count,
                            EpsB200Buffer* outputs, void* stream_arg, EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    Require(features && outputs, "null features or outputs");
    Require(count >= 1 && count <= kNoAllocFeatures,
            "the allocation-free lookup takes 1 to 256 features per call",
            EPS_B200_CAPACITY_EXCEEDED);
    std::lock_guard lock(s.mutex);
    s.Activate();
    Require(s.opt.shard_count == 1, "a client-level lookup needs a single-shard store");
    LookupFeature desc[kNoAllocFeatures];
    unsigned long long bag_base = 0, unit_base = 0;
    unsigned dmax = 1;
    bool all4 = true, all2 = true, out16 = true, out8 = true;
    for (uint64_t i = 0; i < count; ++i) {
      const auto& f = features[i];
      for (uint64_t j = 0; j < i; ++j) Require(features[j].feature != f.feature, "duplicate feature ID");
      const Table& t = s.Get(f.table);
      Require(!t.hashed, "the allocation-free lookup serves dense tables (key_space > 0)");
      const unsigned long long rows = CheckFeatureShape(f);
      const unsigned D = t.def.dimension;
      const auto& o = outputs[i];
      Require(o.feature == f.feature && o.rows == rows && o.columns == D,
              "output buffer layout mismatch");
      Require(o.device == s.opt.device, "the allocation-free lookup writes device outputs only");
      Require(!rows || o.data, "null output buffer");
      dmax = std::max(dmax, D);
      all4 &= D % 4 == 0;
      all2 &= D % 2 == 0;
      out16 &= (reinterpret_cast<uintptr_t>(o.data) & 15) == 0;
      out8 &= (reinterpret_cast<uintptr_t>(o.data) & 7) == 0;
      // value-initialised: every field this path does not set (hash index,
      // slot list, emit units) must read as null / zero in the kernel
      LookupFeature& L = desc[i];
      L = LookupFeature{};
      L.keys = reinterpret_cast<const unsigned long long*>(f.keys);
      L.offsets = reinterpret_cast<const unsigned long long*>(f.offsets);
      L.lengths = reinterpret_cast<const unsigned long long*>(f.valid_lengths);
      L.out = static_cast<float*>(o.data);
      L.state = t.state;
      L.rows = t.rows;
      L.key_count = f.key_count;
      L.bag_count = f.offset_count - 1;
      L.bag_base = bag_base;
      L.occ_base = 0;
      L.scale_base = 0;
      L.dim = D;
      L.pooling = f.pooling;
      L.table_rank = 0;
      L.feature_index = (unsigned)i;
      L.has_padding = f.has_padding ? 1u : 0u;
      L.padding_key = f.padding_key;
      bag_base += L.bag_count;
    }
    // launch shape as in the regular lookup (no heap use here), then the work
    // units, whose size for short bags follows the shape's group
    Shape sh;
    Require(choose_shape(dmax, all4, out16, &sh),
            "embedding dimension/alignment not supported by this build", EPS_B200_CAPACITY_EXCEEDED);
    for (uint64_t i = 0; i < count; ++i) {
      LookupFeature& L = desc[i];
      L.unit_bags = feature_unit_bags(L.pooling, L.key_count, L.bag_count, (unsigned)sh.group);
      L.unit_base = unit_base;
      L.units = feature_units(L.pooling, L.key_count, L.bag_count, L.unit_bags);
      unit_base += L.units;
    }
    (void)all2;
    (void)out8;
    LookupFeature* table = nullptr;
    Cuda(noalloc_feature_table(s.opt.device, &table));
    cudaStream_t stream = s.Use(stream_arg);
    unsigned stores = 0;
    Cuda(noalloc_store_features(desc, (unsigned)count, stream, &stores));
    s.stats.kernel_launches += stores;
    LookupLaunch lp{};
    lp.features = table;
    lp.feature_count = (unsigned)count;
    lp.bag_total = bag_base;
    lp.unit_total = unit_base;
    lp.shard_count = 1;
    lp.shard_id = 0;
    lp.client = 1;
    lp.slot_bits = 1;
    lp.key64 = 0;
    lp.error = s.sticky_error;      // reported by eps_b200_synchronize
    lp.vec = sh.vec;
    lp.group = sh.group;
    lp.iters = sh.iters;
    Cuda(launch_lookup(lp, stream));
    ++s.stats.lookups;
    if (unit_base) ++s.stats.kernel_launches;
    s.Done(stream);
  });
}

}  // extern "C"

namespace {
// eps_b200_push with an optional device reject word (sharded rounds).
int PushEntry(EpsB200Store* store, uint64_t ticket, const EpsB200Buffer* gradients,
              uint64_t count, void* stream_arg, int32_t wait, const unsigned* external_reject,
              EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    std::lock_guard lock(s.mutex);
    s.Activate();
    cudaStream_t stream = s.Use(stream_arg);
    s.Poll(stream);
    auto it = s.tickets.find(ticket);
    if (it == s.tickets.end()) {
      // src/server/service.cpp:241-245: a completed Push is acknowledged again
      Require(s.completed.count(ticket) != 0, "unknown lookup ticket");
      ++s.stats.duplicate_requests;
      return;
    }
    if (it->second.push_in_flight) {
      s.Sync(stream);
      const std::string m = s.Resolve(it, stream);
      if (m.empty()) { ++s.stats.duplicate_requests; return; }
      it = s.tickets.find(ticket);
      Require(it != s.tickets.end(), m.c_str());
    }
    Ticket& t = it->second;
    Require(!t.read_only, "ticket does not belong to update");
    // the push reads the ticket's coalesced occurrence list
    if (t.sorted) Cuda(cudaStreamWaitEvent(stream, t.sorted, 0));
    const size_t nf = t.feature_ids.size();
    Require(gradients && count == nf, "gradient feature count mismatch");
    // gradient index by feature id (src/access/batch_access.cpp:86-96)
    std::map<unsigned, const EpsB200Buffer*> by_id;
    for (uint64_t i = 0; i < count; ++i)
      Require(by_id.emplace(gradients[i].feature, &gradients[i]).second, "duplicate gradient feature");
    unsigned long long host_values = 0, total_values = 0;
    bool g16 = true, g8 = true;
    std::vector<const EpsB200Buffer*> ordered(nf);
    for (size_t i = 0; i < nf; ++i) {
      auto f = by_id.find(t.feature_ids[i]);
      Require(f != by_id.end(), "missing feature gradient");
      const EpsB200Buffer& g = *f->second;
      Require(g.rows == t.grad_rows[i] && g.columns == t.dims[i], "gradient tensor layout mismatch");
      const unsigned long long n = g.rows * g.columns;
      Require(!n || g.data, "native gradient budget/pointer invalid");
      Require(g.device < 0 || g.device == s.opt.device, "gradient device mismatch");
      if (g.device < 0) host_values += n;
      else {
        g16 &= (reinterpret_cast<uintptr_t>(g.data) & 15) == 0;
        g8 &= (reinterpret_cast<uintptr_t>(g.data) & 7) == 0;
      }
      total_values += n;
      ordered[i] = &g;
    }
    int vec, group, iters;
    choose_vec(t.dims, g16, g8, &vec, &group, &iters);
    float* stage = nullptr;
    if (host_values)
      Cuda(cudaMallocAsync(reinterpret_cast<void**>(&stage), host_values * 4, stream));
    // the piece sums live only for the push's kernels: one stream-ordered block
    // per push, released right after them, so consecutive pushes reuse it
    float* part = nullptr;
    try {
      Cuda(cudaMallocAsync(reinterpret_cast<void**>(&part),
                           std::max<size_t>((size_t)t.max_pieces * t.dim_max * 4, 256), stream));
    } catch (...) {
      if (stage) cudaFreeAsync(stage, stream);
      throw;
    }
    try {
      std::vector<PushFeature> pf(nf);
      std::vector<unsigned long long> prefix(nf + 1, 0);
      unsigned long long hoff = 0;
      for (size_t i = 0; i < nf; ++i) {
        const EpsB200Buffer& g = *ordered[i];
        const unsigned long long n = g.rows * g.columns;
        const float* dev = static_cast<const float*>(g.data);
        if (g.device < 0) {
          if (n) Cuda(cudaMemcpyAsync(stage + hoff, g.data, n * 4, cudaMemcpyHostToDevice, stream));
          dev = stage + hoff;
          hoff += n;
        }
        pf[i] = PushFeature{dev, g.rows, t.scale_base[i], t.dims[i], t.ranks[i]};
        prefix[i + 1] = prefix[i] + n;
      }
      std::vector<PushTable> pt(t.table_ids.size());
      for (size_t r = 0; r < pt.size(); ++r) {
        const Table& tab = s.Get(t.table_ids[r]);
        const auto& d = tab.def;
        PushTable& x = pt[r];
        x.state = tab.state;
        x.updates = tab.updates;
        x.dtable = tab.dtable;
        x.rows = tab.rows;
        x.occurrences = t.table_occ[r];
        x.learning_rate = d.learning_rate;
        x.beta1 = d.beta1;
        x.beta2 = d.beta2;
        x.epsilon = d.epsilon;
        x.one_minus_beta1 = 1.0f - d.beta1;   // exact (Sterbenz), as (1 - o.beta1) in the reference
        x.one_minus_beta2 = 1.0f - d.beta2;
        x.has_bounds = d.has_weight_bounds;
        x.bound_min = d.weight_min;
        x.bound_max = d.weight_max;
        x.dim = d.dimension;
        x.lr_t = 0.0f;
      }
      {
        // one host image of [control (zeroed) | tables | features | prefix]
        char* first = reinterpret_cast<char*>(t.control);
        const size_t span = t.stage_end - first;
        std::vector<char> image(span, 0);
        std::memcpy(image.data() + (reinterpret_cast<char*>(t.push_tables) - first), pt.data(),
                    pt.size() * sizeof(PushTable));
        std::memcpy(image.data() + (reinterpret_cast<char*>(t.push_features) - first), pf.data(),
                    nf * sizeof(PushFeature));
        std::memcpy(image.data() + (reinterpret_cast<char*>(t.grad_prefix) - first), prefix.data(),
                    (nf + 1) * 8);
        s.Stage(first, image.data(), span, stream);
      }
      PushLaunch pl{};
      pl.tables = t.push_tables;
      pl.table_count = (unsigned)pt.size();
      pl.features = t.push_features;
      pl.feature_count = (unsigned)nf;
      pl.row_scale = t.row_scale;
      pl.keys = t.keys;
      pl.srcs = t.srcs;
      pl.n = t.n;
      pl.slot_bits = t.slot_bits;
      pl.key64 = t.key64;
      pl.grad_values = total_values;
      {
        unsigned long long mx = 0;
        bool v4 = true;
        for (size_t i = 0; i < nf; ++i) {
          const unsigned long long nv = pf[i].rows * (unsigned long long)pf[i].dim;
          mx = std::max(mx, nv);
          v4 &= nv % 4 == 0 && (reinterpret_cast<uintptr_t>(pf[i].grad) & 15) == 0;
        }
        pl.grad_max_values = mx;
        pl.grad_vec4 = v4 ? 1 : 0;
      }
      pl.grad_prefix = t.grad_prefix;
      pl.seg_start = t.seg_start;
      pl.seg_total = t.seg_total;
      pl.rows = t.rows;
      pl.plan = t.plan;
      pl.pieces = t.pieces;
      pl.max_pieces = t.max_pieces;
      pl.part = part;
      pl.records = t.records;
      pl.dim_max = t.dim_max;
      pl.control = t.control;
      pl.lookup_error = t.lookup_error;
      pl.external_reject = external_reject;
      pl.long_run = (s.opt.flags & EPS_B200_FLAG_REFERENCE_ORDER) ? ~0ull : (unsigned long long)kLongRun;
      pl.vec = vec;
      pl.group = group;
      pl.iters = iters;
      {
        // the async ring row path: one dimension in {32, 64, 128}, aligned gradients
        const unsigned d0 = t.dims.empty() ? 0u : t.dims[0];
        bool same = d0 == 32 || d0 == 64 || d0 == 128;
        for (unsigned d : t.dims) same &= d == d0;
        pl.ring_dim = (same && pl.grad_vec4 && t.dim_max == d0 && !(s.opt.flags & EPS_B200_FLAG_REGISTER_ROWS))
                          ? (int)d0 : 0;
      }
      // the piece sums (uniform shape) write only the push's scratch, so they
      // run on the side stream concurrently with the prescan; the row updates
      // wait for both
      const unsigned piece_launches = launch_push_apply_count(pl, 0);
      if (piece_launches) {
        Cuda(cudaEventRecord(s.push_fork, stream));
        Cuda(cudaStreamWaitEvent(s.side, s.push_fork, 0));
        cudaEvent_t evp = s.Begin(s.side);
        Cuda(launch_push_apply(pl, s.side, 0));
        s.End(EPS_B200_PHASE_PIECES, evp, s.side, piece_launches);
        Cuda(cudaEventRecord(s.push_join, s.side));
      }
      cudaEvent_t ev = s.Begin(stream);
      Cuda(launch_push_prescan(pl, stream));
      s.End(EPS_B200_PHASE_PRESCAN, ev, stream, 1);
      if (piece_launches) Cuda(cudaStreamWaitEvent(stream, s.push_join, 0));
      ev = s.Begin(stream);
      Cuda(launch_push_apply(pl, stream, 1));
      s.End(EPS_B200_PHASE_APPLY, ev, stream, launch_push_apply_count(pl, 1));
      ev = s.Begin(stream);
      Cuda(launch_push_apply(pl, stream, 2));
      s.End(EPS_B200_PHASE_LONG, ev, stream, launch_push_apply_count(pl, 2));
      ev = s.Begin(stream);
      Cuda(launch_push_finalize(pl, stream));
      s.End(EPS_B200_PHASE_FINALIZE, ev, stream, launch_push_finalize_count(pl));
      Cuda(cudaMemcpyAsync(&s.host_status[t.slot], t.status, sizeof(StatusBlock),
                           cudaMemcpyDeviceToHost, stream));
      { float* owned = part; part = nullptr; Cuda(cudaFreeAsync(owned, stream)); }
      if (stage) { float* owned = stage; stage = nullptr; Cuda(cudaFreeAsync(owned, stream)); }
      t.done = s.SyncEvent();
      Cuda(cudaEventRecord(t.done, stream));
      s.inflight.push_back(ticket);
      t.push_in_flight = true;
      s.Done(stream);
    } catch (...) {
      cudaStreamSynchronize(stream);
      if (part) cudaFreeAsync(part, stream);
      if (stage) cudaFreeAsync(stage, stream);
      throw;
    }
    if (wait || host_values) {
      s.Sync(stream);
      const std::string m = s.Resolve(it, stream);
      Require(m.empty(), m.c_str());
    }
  });
}
}  // namespace

extern "C" {

int eps_b200_push(EpsB200Store* store, uint64_t ticket, const EpsB200Buffer* gradients,
                  uint64_t count, void* stream_arg, int32_t wait, EpsB200Status* status) {
  return PushEntry(store, ticket, gradients, count, stream_arg, wait, nullptr, status);
}

int eps_b200_release(EpsB200Store* store, uint64_t ticket, EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    std::lock_guard lock(s.mutex);
    s.Activate();
    cudaStream_t stream = s.Use(nullptr);
    auto it = s.tickets.find(ticket);
    if (it == s.tickets.end()) {
      Require(s.completed.count(ticket) != 0, "unknown lookup ticket");
      return;
    }
    if (it->second.push_in_flight) {
      s.Sync(stream);
      const std::string m = s.Resolve(it, stream);
      it = s.tickets.find(ticket);
      if (it == s.tickets.end()) { if (!m.empty()) Require(false, m.c_str()); return; }
    }
    s.FreeTicket(it, stream);
    s.Done(stream);
  });
}

int eps_b200_ticket_coalesced(EpsB200Store* store, uint64_t ticket, uint32_t* tables,
                              uint64_t* keys, uint64_t* row_offsets, uint32_t* features,
                              uint64_t* sources, float* scales, uint64_t row_capacity,
                              uint64_t reference_capacity, uint64_t* rows_out,
                              uint64_t* references_out, EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    Require(rows_out && references_out, "null count outputs");
    std::lock_guard lock(s.mutex);
    s.Activate();
    auto it = s.tickets.find(ticket);
    Require(it != s.tickets.end(), "unknown lookup ticket");
    const Ticket& t = it->second;
    Require(!t.read_only, "ticket does not belong to update");
    // the ticket's lookup ended before the store's latest call did; its sort
    // (side stream) is waited for separately
    Cuda(cudaEventSynchronize(s.last_done));
    if (t.sorted) Cuda(cudaEventSynchronize(t.sorted));
    unsigned lookup_error = 0, seg_total = 0;
    Cuda(cudaMemcpy(&lookup_error, t.lookup_error, sizeof(unsigned), cudaMemcpyDeviceToHost));
    Require(!lookup_error, EpsB200Store::LookupMessage(lookup_error).c_str());
    Cuda(cudaMemcpy(&seg_total, t.seg_total, sizeof(unsigned), cudaMemcpyDeviceToHost));
    const unsigned long long n = t.n;
    std::vector<unsigned long long> ck(n);
    if (t.key64) {
      Cuda(cudaMemcpy(ck.data(), t.keys, n * 8, cudaMemcpyDeviceToHost));
    } else {
      std::vector<unsigned> k32(n);
      Cuda(cudaMemcpy(k32.data(), t.keys, n * 4, cudaMemcpyDeviceToHost));
      for (unsigned long long i = 0; i < n; ++i) ck[i] = k32[i];
    }
    std::vector<unsigned> src(n), seg(seg_total + 1ull);
    Cuda(cudaMemcpy(src.data(), t.srcs, n * 4, cudaMemcpyDeviceToHost));
    Cuda(cudaMemcpy(seg.data(), t.seg_start, seg.size() * 4, cudaMemcpyDeviceToHost));
    const unsigned long long grad_rows =
        t.scale_base.empty() ? 0 : t.scale_base.back() + t.grad_rows.back();
    std::vector<float> scale(grad_rows);
    if (grad_rows)
      Cuda(cudaMemcpy(scale.data(), t.row_scale, grad_rows * 4, cudaMemcpyDeviceToHost));
    // runs of padding occurrences (table rank past the lookup's tables) are not rows
    const unsigned long long slot_mask = (1ull << t.slot_bits) - 1ull;
    unsigned long long rows = 0, refs = 0;
    for (unsigned u = 0; u < seg_total; ++u)
      if ((ck[seg[u]] >> t.slot_bits) < t.table_ids.size()) { ++rows; refs += seg[u + 1] - seg[u]; }
    *rows_out = rows;
    *references_out = refs;
    if (!tables) return;
    Require(keys && row_offsets && features && sources && scales, "null coalesced outputs");
    Require(row_capacity >= rows && reference_capacity >= refs, "coalesced output capacity too small",
            EPS_B200_CAPACITY_EXCEEDED);
    // a row's key: slot * shards + shard in a dense table; in a hashed table the
    // key its slot was created for (the index's slot -> key array, read once)
    std::vector<std::vector<unsigned long long>> slot_keys(t.table_ids.size());
    auto key_of = [&](unsigned long long rank, unsigned long long slot) {
      const Table& tab = s.Get(t.table_ids[rank]);
      if (!tab.hashed) return slot * s.opt.shard_count + s.opt.shard_id;
      auto& v = slot_keys[rank];
      if (v.empty()) {
        unsigned long long used = 0;
        Cuda(cudaMemcpy(&used, tab.index.used, 8, cudaMemcpyDeviceToHost));
        v.resize(std::max(1ull, std::min(used, tab.rows)));
        Cuda(cudaMemcpy(v.data(), tab.index.slot_keys, v.size() * 8, cudaMemcpyDeviceToHost));
      }
      Require(slot < v.size(), "corrupt occurrence list", EPS_B200_RUN_FAILED);
      return v[slot];
    };
    unsigned long long r = 0, q = 0;
    row_offsets[0] = 0;
    for (unsigned u = 0; u < seg_total; ++u) {
      const unsigned long long rank = ck[seg[u]] >> t.slot_bits;
      if (rank >= t.table_ids.size()) continue;
      tables[r] = t.table_ids[rank];
      keys[r] = key_of(rank, ck[seg[u]] & slot_mask);
      for (unsigned i = seg[u]; i < seg[u + 1]; ++i, ++q) {
        const unsigned f = src[i] >> kRowBits, row = src[i] & ((1u << kRowBits) - 1u);
        Require(f < t.feature_ids.size() && row < t.grad_rows[f], "corrupt occurrence list",
                EPS_B200_RUN_FAILED);
        features[q] = t.feature_ids[f];
        sources[q] = row;
        scales[q] = scale[t.scale_base[f] + row];
      }
      row_offsets[++r] = q;
    }
  });
}

int eps_b200_synchronize(EpsB200Store* store, EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    std::lock_guard lock(s.mutex);
    s.Activate();
    cudaStream_t stream = s.Use(nullptr);
    s.Sync(stream);
    Cuda(cudaStreamSynchronize(s.side));      // lookups' sorts set their error words too
    std::string first = s.deferred;
    s.deferred.clear();
    s.inflight.clear();
    for (auto it = s.tickets.begin(); it != s.tickets.end();) {
      auto next = std::next(it);
      if (it->second.push_in_flight) {
        const std::string m = s.Resolve(it, stream);
        if (first.empty()) first = m;
      } else if (!it->second.lookup_checked) {
        unsigned e = 0;
        Cuda(cudaMemcpy(&e, it->second.lookup_error, sizeof(unsigned), cudaMemcpyDeviceToHost));
        it->second.lookup_checked = true;
        if (e) {
          if (first.empty()) first = EpsB200Store::LookupMessage(e);
          s.FreeTicket(it, stream);
        }
      }
      it = next;
    }
    unsigned sticky = 0;
    Cuda(cudaMemcpy(&sticky, s.sticky_error, sizeof(unsigned), cudaMemcpyDeviceToHost));
    if (sticky) {
      Cuda(cudaMemset(s.sticky_error, 0, sizeof(unsigned)));
      if (first.empty()) first = EpsB200Store::LookupMessage(sticky);
    }
    s.Done(stream);
    Require(first.empty(), first.c_str());
  });
}

namespace {
std::vector<unsigned long long> CheckedKeys(const EpsB200Store& s, const Table& t,
                                            const uint64_t* keys, uint64_t count) {
  Require(!count || keys, "null keys");
  std::vector<unsigned long long> out(keys, keys + count);
  std::unordered_set<unsigned long long> seen;
  for (auto k : out) {
    Require(k % s.opt.shard_count == s.opt.shard_id, "key belongs to another shard");
    Require(t.hashed || k / s.opt.shard_count < t.rows, "unknown parameter row");
    Require(seen.insert(k).second, "duplicate row");
  }
  return out;
}

// A hashed table's keys (on the device) -> slots (on the device), creating the
// rows of unseen keys; `scratch` holds n u32.  Errors land in *err.
void ResolveKeys(const Table& t, const unsigned long long* keys, unsigned long long n,
                 unsigned* scratch, unsigned* slots, unsigned* err, cudaStream_t stream) {
  Cuda(launch_resolve_keys(&t.index, keys, n, scratch, slots, err, stream));
}
}  // namespace

int eps_b200_read_state(EpsB200Store* store, uint32_t table, const uint64_t* keys,
                        uint64_t count, float* weights, float* first, float* second,
                        uint64_t* row_updates, EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    std::lock_guard lock(s.mutex);
    s.Activate();
    const Table& t = s.Get(table);
    auto k = CheckedKeys(s, t, keys, count);
    if (!count) return;
    const unsigned D = t.def.dimension;
    cudaStream_t stream = s.Use(nullptr);
    char* buf = nullptr;
    const size_t kb = align256(count * 8), pb = align256(count * 12ull * D), ub = align256(count * 8);
    const size_t hb = t.hashed ? align256(count * 4) : 0;      // entries, slots (hashed)
    Cuda(cudaMallocAsync(reinterpret_cast<void**>(&buf), kb + pb + ub + 2 * hb + 256, stream));
    std::vector<float> packed(count * 3ull * D);
    std::vector<unsigned long long> upd(count);
    unsigned* err = reinterpret_cast<unsigned*>(buf + kb + pb + ub + 2 * hb);
    unsigned herr = 0;
    try {
      Cuda(cudaMemsetAsync(err, 0, 4, stream));
      Cuda(cudaMemcpyAsync(buf, k.data(), count * 8, cudaMemcpyHostToDevice, stream));
      const auto* dkeys = reinterpret_cast<unsigned long long*>(buf);
      if (t.hashed) {
        auto* slots = reinterpret_cast<unsigned*>(buf + kb + pb + ub + hb);
        ResolveKeys(t, dkeys, count, reinterpret_cast<unsigned*>(buf + kb + pb + ub), slots, err, stream);
        Cuda(launch_read_slots(t.state, t.updates, D, slots, count, reinterpret_cast<float*>(buf + kb),
                               reinterpret_cast<unsigned long long*>(buf + kb + pb), err, stream));
      } else {
        Cuda(launch_read_rows(t.state, t.updates, D, t.rows, s.opt.shard_count, dkeys, count,
                              reinterpret_cast<float*>(buf + kb),
                              reinterpret_cast<unsigned long long*>(buf + kb + pb), err, stream));
      }
      Cuda(cudaMemcpyAsync(packed.data(), buf + kb, count * 12ull * D, cudaMemcpyDeviceToHost, stream));
      Cuda(cudaMemcpyAsync(upd.data(), buf + kb + pb, count * 8, cudaMemcpyDeviceToHost, stream));
      Cuda(cudaMemcpyAsync(&herr, err, 4, cudaMemcpyDeviceToHost, stream));
      char* owned = buf;
      buf = nullptr;
      Cuda(cudaFreeAsync(owned, stream));
      s.Sync(stream);
    } catch (...) {
      cudaStreamSynchronize(stream);
      if (buf) cudaFreeAsync(buf, stream);
      throw;
    }
    s.Done(stream);
    Require(!(herr & kLookupCapacity), "hashed table capacity exceeded", EPS_B200_CAPACITY_EXCEEDED);
    for (uint64_t r = 0; r < count; ++r) {
      const float* row = packed.data() + r * 3ull * D;
      if (weights) std::memcpy(weights + r * D, row, D * 4);
      if (first) std::memcpy(first + r * D, row + D, D * 4);
      if (second) std::memcpy(second + r * D, row + 2 * D, D * 4);
      if (row_updates) row_updates[r] = upd[r];
    }
  });
}

int eps_b200_load_state(EpsB200Store* store, uint32_t table, const uint64_t* keys,
                        uint64_t count, const float* weights, const float* first,
                        const float* second, const uint64_t* row_updates,
                        EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    std::lock_guard lock(s.mutex);
    s.Activate();
    const Table& t = s.Get(table);
    auto k = CheckedKeys(s, t, keys, count);
    if (!count) return;
    Require(weights && first && second, "null row state");
    const unsigned D = t.def.dimension;
    std::vector<float> packed(count * 3ull * D);
    std::vector<unsigned long long> upd(count, 0);
    for (uint64_t r = 0; r < count; ++r) {
      float* row = packed.data() + r * 3ull * D;
      std::memcpy(row, weights + r * D, D * 4);
      std::memcpy(row + D, first + r * D, D * 4);
      std::memcpy(row + 2 * D, second + r * D, D * 4);
      for (unsigned d = 0; d < 3 * D; ++d) Require(std::isfinite(row[d]), "non-finite cache state");
      for (unsigned d = 0; d < D; ++d) Require(row[2 * D + d] >= 0, "negative second moment");
      if (row_updates) upd[r] = row_updates[r];
    }
    cudaStream_t stream = s.Use(nullptr);
    char* buf = nullptr;
    const size_t kb = align256(count * 8), pb = align256(count * 12ull * D), ub = align256(count * 8);
    const size_t hb = t.hashed ? align256(count * 4) : 0;      // entries, slots (hashed)
    Cuda(cudaMallocAsync(reinterpret_cast<void**>(&buf), kb + pb + ub + 2 * hb + 256, stream));
    unsigned* err = reinterpret_cast<unsigned*>(buf + kb + pb + ub + 2 * hb);
    unsigned herr = 0;
    try {
      Cuda(cudaMemsetAsync(err, 0, 4, stream));
      Cuda(cudaMemcpyAsync(buf, k.data(), count * 8, cudaMemcpyHostToDevice, stream));
      Cuda(cudaMemcpyAsync(buf + kb, packed.data(), count * 12ull * D, cudaMemcpyHostToDevice, stream));
      Cuda(cudaMemcpyAsync(buf + kb + pb, upd.data(), count * 8, cudaMemcpyHostToDevice, stream));
      const auto* dkeys = reinterpret_cast<unsigned long long*>(buf);
      if (t.hashed) {
        auto* slots = reinterpret_cast<unsigned*>(buf + kb + pb + ub + hb);
        ResolveKeys(t, dkeys, count, reinterpret_cast<unsigned*>(buf + kb + pb + ub), slots, err, stream);
        Cuda(launch_write_slots(t.state, t.updates, D, slots, count, reinterpret_cast<float*>(buf + kb),
                                reinterpret_cast<unsigned long long*>(buf + kb + pb), t.dtable, stream));
      } else {
        Cuda(launch_write_rows(t.state, t.updates, D, t.rows, s.opt.shard_count, dkeys, count,
                               reinterpret_cast<float*>(buf + kb),
                               reinterpret_cast<unsigned long long*>(buf + kb + pb), t.dtable, stream));
      }
      Cuda(cudaMemcpyAsync(&herr, err, 4, cudaMemcpyDeviceToHost, stream));
      char* owned = buf;
      buf = nullptr;
      Cuda(cudaFreeAsync(owned, stream));
      s.Sync(stream);
    } catch (...) {
      cudaStreamSynchronize(stream);
      if (buf) cudaFreeAsync(buf, stream);
      throw;
    }
    s.Done(stream);
    Require(!(herr & kLookupCapacity), "hashed table capacity exceeded", EPS_B200_CAPACITY_EXCEEDED);
  });
}

int eps_b200_optimizer_state(EpsB200Store* store, uint32_t table, uint64_t* optimizer_sequence,
                             float* beta1_power, float* beta2_power, EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    std::lock_guard lock(s.mutex);
    s.Activate();
    const Table& t = s.Get(table);
    cudaStream_t stream = s.Use(nullptr);
    DeviceTable d{};
    Cuda(cudaMemcpyAsync(&d, t.dtable, sizeof(d), cudaMemcpyDeviceToHost, stream));
    s.Sync(stream);
    s.Done(stream);
    if (optimizer_sequence) *optimizer_sequence = d.optimizer_sequence;
    if (beta1_power) *beta1_power = d.beta1_power;
    if (beta2_power) *beta2_power = d.beta2_power;
  });
}

int eps_b200_profile(EpsB200Store* store, int32_t mode, double* phase_ms,
                     uint64_t* phase_launches, uint64_t* phase_calls, EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    std::lock_guard lock(s.mutex);
    s.Activate();
    s.Collect();
    for (int i = 0; i < EPS_B200_PHASES; ++i) {
      if (phase_ms) phase_ms[i] = s.phase_ms[i];
      if (phase_launches) phase_launches[i] = s.phase_launches[i];
      if (phase_calls) phase_calls[i] = s.phase_calls[i];
    }
    if (mode == 1) {
      for (int i = 0; i < EPS_B200_PHASES; ++i) {
        s.phase_ms[i] = 0; s.phase_launches[i] = 0; s.phase_calls[i] = 0;
      }
      s.profiling = true;
    } else if (mode == 0) {
      s.profiling = false;
    }
  });
}

namespace {
Route& GetRoute(EpsB200Store& s, uint64_t id) {
  auto it = s.routes.find(id);
  Require(it != s.routes.end(), "unknown route");
  return it->second;
}
RouteLaunch RouteParams(const Route& r) {
  RouteLaunch lp{};
  lp.features = r.desc;
  lp.feature_count = r.F;
  lp.shard_count = r.n;
  lp.bag_total = r.B;
  lp.key_total = r.N;
  lp.cells = r.cells;
  lp.tiles = r.tiles;
  lp.cnt = r.cnt; lp.pk = r.pk; lp.pb = r.pb;
  lp.bounds = r.bounds;
  lp.error = r.error;
  lp.bag_map = r.bag_map;
  lp.pos_map = r.pos_map;
  lp.part_off = r.part_off;
  lp.row_pre = r.row_pre;
  lp.row_total_dev = r.row_total;
  lp.dd_keys = r.dd_keys;
  lp.dd_rank = r.dd_rank;
  lp.dd_mask = r.dd_mask;
  lp.dd_count = r.dd_count;
  lp.dd_used = r.dd_used;
  lp.dd_off = r.dd_off;
  lp.dd_words = r.dd_words;
  lp.dd_idx = r.dd_idx;
  lp.has_sequence = r.has_sequence;
  return lp;
}
bool Aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
}  // namespace

int eps_b200_route(EpsB200Store* store, const EpsB200Feature* features, uint64_t count,
                   uint32_t shard_count, void* stream_arg, uint64_t* route_out, int64_t* counts,
                   EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    Require(features && route_out && counts && count > 0 && count <= kMaxFeatures,
            "invalid native feature count");
    Require(shard_count >= 1 && shard_count <= 32 && shard_count * count <= kMaxFeatures,
            "route shard count must be 1 .. 32, with shards x features <= 1024");
    std::lock_guard lock(s.mutex);
    s.Activate();
    Route r;
    r.n = shard_count;
    r.F = (unsigned)count;
    std::vector<LookupFeature> desc(count);
    std::unordered_set<unsigned> ids;
    unsigned dim_max = 1;
    for (uint64_t i = 0; i < count; ++i) {
      const auto& f = features[i];
      Require(ids.insert(f.feature).second, "duplicate feature ID");
      const Table& t = s.Get(f.table);
      Require(f.pooling <= 2, "unsupported pooling mode");
      Require(f.offset_count >= 1 && f.offsets, "invalid bag offsets");
      Require(f.offset_count > 1 || f.key_count == 0, "invalid bag offsets");
      Require(!f.key_count || f.keys, "null feature keys");
      Require(!f.has_padding || !f.valid_lengths,
              "valid lengths are derived from the padding key; pass one or the other");
      const unsigned long long rows = f.pooling == 2 ? f.key_count : f.offset_count - 1;
      Require(rows < (1ull << kRowBits) && f.key_count < (1ull << 31),
              "feature exceeds the per-feature row limit", EPS_B200_CAPACITY_EXCEEDED);
      LookupFeature& L = desc[i];
      L.keys = reinterpret_cast<const unsigned long long*>(f.keys);
      L.offsets = reinterpret_cast<const unsigned long long*>(f.offsets);
      L.lengths = reinterpret_cast<const unsigned long long*>(f.valid_lengths);
      L.rows = t.hashed ? ~0ull : t.def.key_space;   // route checks keys against it
      L.key_count = f.key_count;
      L.bag_count = f.offset_count - 1;
      L.bag_base = r.B;
      L.dim = t.def.dimension;
      L.pooling = f.pooling;
      L.table_rank = f.table;            // a route's descriptors carry the table id
      L.feature_index = (unsigned)i;
      L.has_padding = f.has_padding ? 1u : 0u;
      L.padding_key = f.padding_key;
      r.B += L.bag_count;
      r.N += f.key_count;
      r.dims.push_back(t.def.dimension);
      r.pooling.push_back(f.pooling);
      r.rows.push_back(rows);
      r.has_sequence |= f.pooling == 2;
      dim_max = std::max(dim_max, t.def.dimension);
    }
    r.cells = (unsigned long long)r.n * r.B;
    Require(r.N < (1ull << 32) && r.cells < (1ull << 32) &&
            (r.N + r.B) * (unsigned long long)dim_max < (1ull << 32),
            "route exceeds the occurrence limit", EPS_B200_CAPACITY_EXCEEDED);
    r.tiles = route_tiles(r.cells);
    const size_t nb = (size_t)r.n * (r.F + 1) * 2;
    Carver c;
    const size_t at_desc = c.take<LookupFeature>(count);
    const size_t at_cnt = c.take<unsigned>(r.cells);
    const size_t at_pk = c.take<unsigned>(r.cells + 1);
    const size_t at_pb = c.take<unsigned>(r.cells + 1);
    const size_t at_tk = c.take<unsigned>(r.tiles);
    const size_t at_tb = c.take<unsigned>(r.tiles);
    const size_t at_bounds = c.take<unsigned>(nb + 1);   // + error word
    const size_t at_bag = c.take<unsigned>(r.cells);
    const size_t at_pos = c.take<unsigned>(r.N);
    const size_t at_poff = c.take<unsigned long long>((size_t)r.n * r.F);
    const size_t at_rpre = c.take<unsigned long long>((size_t)r.n * r.F + 1);   // + row total
    const size_t at_outs = c.take<float*>(count);
    const size_t at_grads = c.take<float*>(count);
    // the distinct-key set: a power of two of at least 2N entries (half full at most)
    unsigned long long dd_cap = 0;
    if (r.N) { dd_cap = 2; while (dd_cap < 2 * r.N) dd_cap <<= 1; }
    const size_t groups = (size_t)r.n * r.F;
    const size_t at_ddk = c.take<unsigned long long>(dd_cap);
    const size_t at_ddr = c.take<unsigned>(dd_cap);
    const size_t at_ddc = c.take<unsigned>(groups);
    const size_t at_ddu = c.take<unsigned>(groups);
    const size_t at_ddo = c.take<unsigned long long>(groups);
    const size_t at_ddw = c.take<unsigned long long>(groups + 1);
    const size_t at_ddi = c.take<unsigned>(r.N);
    cudaStream_t stream = s.RouteStream(stream_arg);
    Cuda(cudaMallocAsync(reinterpret_cast<void**>(&r.slab), std::max<size_t>(c.offset, 256), stream));
    try {
      auto P = [&](size_t at) { return r.slab + at; };
      r.desc = reinterpret_cast<LookupFeature*>(P(at_desc));
      r.cnt = reinterpret_cast<unsigned*>(P(at_cnt));
      r.pk = reinterpret_cast<unsigned*>(P(at_pk));
      r.pb = reinterpret_cast<unsigned*>(P(at_pb));
      r.tile_k = reinterpret_cast<unsigned*>(P(at_tk));
      r.tile_b = reinterpret_cast<unsigned*>(P(at_tb));
      r.bounds = reinterpret_cast<unsigned*>(P(at_bounds));
      r.error = r.bounds + nb;
      r.bag_map = reinterpret_cast<unsigned*>(P(at_bag));
      r.pos_map = reinterpret_cast<unsigned*>(P(at_pos));
      r.part_off = reinterpret_cast<unsigned long long*>(P(at_poff));
      r.row_pre = reinterpret_cast<unsigned long long*>(P(at_rpre));
      r.row_total = r.row_pre + (size_t)r.n * r.F;
      r.outs = reinterpret_cast<float**>(P(at_outs));
      r.grads = reinterpret_cast<const float**>(P(at_grads));
      r.dd_keys = reinterpret_cast<unsigned long long*>(P(at_ddk));
      r.dd_rank = reinterpret_cast<unsigned*>(P(at_ddr));
      r.dd_mask = dd_cap ? dd_cap - 1 : 0;
      r.dd_count = reinterpret_cast<unsigned*>(P(at_ddc));
      r.dd_used = reinterpret_cast<unsigned*>(P(at_ddu));
      r.dd_off = reinterpret_cast<unsigned long long*>(P(at_ddo));
      r.dd_words = reinterpret_cast<unsigned long long*>(P(at_ddw));
      r.dd_idx = reinterpret_cast<unsigned*>(P(at_ddi));
      Cuda(cudaMemsetAsync(r.error, 0, sizeof(unsigned), stream));
      if (dd_cap) Cuda(cudaMemsetAsync(r.dd_keys, 0xFF, dd_cap * 8, stream));
      Cuda(cudaMemsetAsync(r.dd_count, 0, groups * 4, stream));
      s.Stage(r.desc, desc.data(), count * sizeof(LookupFeature), stream);
      RouteLaunch lp = RouteParams(r);
      lp.tile_k = r.tile_k;
      lp.tile_b = r.tile_b;
      lp.counts_out = reinterpret_cast<long long*>(counts);
      Cuda(launch_route_count(lp, stream));
      s.stats.kernel_launches += route_count_launches(lp);
    } catch (...) {
      cudaFreeAsync(r.slab, stream);
      throw;
    }
    r.last = stream;
    const unsigned long long id = s.next_route++;
    s.routes.emplace(id, std::move(r));
    *route_out = id;
  });
}


int eps_b200_route_scatter(EpsB200Store* store, uint64_t route, uint64_t* payload, void* stream_arg,
                           EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    std::lock_guard lock(s.mutex);
    s.Activate();
    Route& r = GetRoute(s, route);
    Require(payload != nullptr, "null route payload");
    Require((reinterpret_cast<uintptr_t>(payload) & 7) == 0, "misaligned route payload");
    cudaStream_t stream = s.RouteStream(stream_arg);
    RouteLaunch lp = RouteParams(r);
    lp.payload = reinterpret_cast<unsigned long long*>(payload);
    Cuda(launch_route_scatter(lp, stream));
    s.stats.kernel_launches += 1;
    r.last = stream;
  });
}

int eps_b200_route_merge(EpsB200Store* store, uint64_t route, const float* partials,
                         const EpsB200Buffer* outputs, void* stream_arg, EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    std::lock_guard lock(s.mutex);
    s.Activate();
    Route& r = GetRoute(s, route);
    Require(outputs != nullptr, "null route outputs");
    Require(partials != nullptr, "null route partials");
    std::vector<float*> outs(r.F);
    bool a16 = Aligned16(partials);
    for (unsigned f = 0; f < r.F; ++f) {
      const auto& o = outputs[f];
      Require(o.rows == r.rows[f] && o.columns == r.dims[f], "output buffer layout mismatch");
      Require(!o.rows || o.data, "null output buffer");
      Require(o.device == s.opt.device, "route outputs must be on the store's device");
      outs[f] = static_cast<float*>(o.data);
      a16 &= Aligned16(o.data);
    }
    cudaStream_t stream = s.RouteStream(stream_arg);
    s.Stage(r.outs, outs.data(), r.F * sizeof(float*), stream);
    RouteLaunch lp = RouteParams(r);
    lp.partials = partials;
    lp.outs = r.outs;
    choose_vec(r.dims, a16, false, &lp.vec, &lp.group, &lp.iters);
    if (r.B || (r.has_sequence && r.N)) {
      Cuda(launch_route_merge(lp, stream));
      s.stats.kernel_launches += 1;
    }
    r.last = stream;
  });
}

int eps_b200_route_gather(EpsB200Store* store, uint64_t route, const EpsB200Buffer* gradients,
                          float* send, uint32_t* nonfinite, void* stream_arg, EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    std::lock_guard lock(s.mutex);
    s.Activate();
    Route& r = GetRoute(s, route);
    Require(gradients != nullptr, "null route gradients");
    Require(send != nullptr, "null route send buffer");
    std::vector<const float*> grads(r.F);
    bool a16 = Aligned16(send);
    for (unsigned f = 0; f < r.F; ++f) {
      const auto& g = gradients[f];
      Require(g.rows == r.rows[f] && g.columns == r.dims[f], "gradient tensor layout mismatch");
      Require(!g.rows || g.data, "null gradient buffer");
      Require(g.device == s.opt.device, "route gradients must be on the store's device");
      grads[f] = static_cast<const float*>(g.data);
      a16 &= Aligned16(g.data);
    }
    cudaStream_t stream = s.RouteStream(stream_arg);
    s.Stage(r.grads, grads.data(), r.F * sizeof(float*), stream);
    RouteLaunch lp = RouteParams(r);
    lp.grads = r.grads;
    lp.send = send;
    lp.nonfinite = nonfinite;
    choose_vec(r.dims, a16, false, &lp.vec, &lp.group, &lp.iters);
    {
      Cuda(launch_route_gather(lp, stream));
      s.stats.kernel_launches += 1;
    }
    r.last = stream;
  });
}

int eps_b200_route_release(EpsB200Store* store, uint64_t route, EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    std::lock_guard lock(s.mutex);
    s.Activate();
    auto it = s.routes.find(route);
    Require(it != s.routes.end(), "unknown route");
    char* slab = it->second.slab;
    cudaStream_t last = it->second.last;
    s.routes.erase(it);
    Cuda(cudaFreeAsync(slab, last ? last : s.own));
  });
}

namespace {
// Owner-side layout of a sharded round: requester r's payload region and the
// (requester, feature) row blocks of the partial / gradient buffers.  Peer
// counts are [requester][feature][keys, kept bags, distinct keys]; a group with
// distinct keys U > 0 is deduplicated: its payload ends with [0, U, U keys] and
// its partial block holds U rows (its gradient block, as any other, one row per
// kept bag or key).
struct ServeLayout {
  std::vector<EpsB200Feature> feats;
  std::vector<EpsB200Buffer> blocks;     // rows x dim views
  std::vector<EpsB200Feature> uniq;      // deduplicated groups: their distinct keys
  std::vector<EpsB200Buffer> uniq_blocks;
};
ServeLayout MakeServeLayout(EpsB200Store& s, const uint64_t* payload, const uint64_t* peer_counts,
                            const uint32_t* tables, const uint32_t* poolings, uint32_t n,
                            uint32_t F, const float* rows_base, bool partials) {
  Require(peer_counts && tables && poolings && n >= 1 && n <= 32 && F >= 1 &&
          (uint64_t)n * F <= kMaxFeatures, "invalid sharded round layout");
  std::vector<unsigned> dims(F);
  {
    std::lock_guard lock(s.mutex);
    for (uint32_t f = 0; f < F; ++f) {
      Require(poolings[f] <= 2, "unsupported pooling mode");
      dims[f] = s.Get(tables[f]).def.dimension;
    }
  }
  ServeLayout L;
  L.feats.resize((size_t)n * F);
  L.blocks.resize((size_t)n * F);
  unsigned long long base = 0, floats = 0;
  for (uint32_t r = 0; r < n; ++r) {
    const uint64_t* c = peer_counts + (size_t)r * F * 3;
    unsigned long long NK = 0, KB = 0, UW = 0;
    for (uint32_t f = 0; f < F; ++f) {
      NK += c[3 * f]; KB += c[3 * f + 1];
      UW += c[3 * f + 2] ? c[3 * f + 2] + 2 : 0;
    }
    unsigned long long ko = 0, oo = 0, lo = 0, uo = 0;
    for (uint32_t f = 0; f < F; ++f) {
      const unsigned long long nk = c[3 * f], kb = c[3 * f + 1], U = c[3 * f + 2];
      Require(U <= nk, "invalid sharded round layout");
      EpsB200Feature& x = L.feats[(size_t)r * F + f];
      x.table = tables[f];
      x.feature = r * F + f;
      x.pooling = poolings[f];
      x.has_padding = 0;
      x.padding_key = 0;
      x.keys = payload + base + ko;
      x.key_count = nk;
      x.offsets = payload + base + NK + oo;
      x.offset_count = kb + 1;
      x.valid_lengths = payload + base + NK + KB + F + lo;
      ko += nk; oo += kb + 1; lo += kb;
      const unsigned long long rows = poolings[f] == 2 ? nk : kb;
      const unsigned long long block_rows = partials && U ? U : rows;
      EpsB200Buffer& b = L.blocks[(size_t)r * F + f];
      b.feature = r * F + f;
      b.reserved = 0;
      b.rows = rows;
      b.columns = dims[f];
      b.data = const_cast<float*>(rows_base) + floats;
      b.device = s.opt.device;
      b.reserved2 = 0;
      if (partials && U) {
        // the group's distinct rows: a sequence feature over its unique keys,
        // gathered into the partial block; the per-bag feature gathers nothing
        EpsB200Feature u{};
        u.table = tables[f];
        u.feature = r * F + f;
        u.pooling = 2;
        u.keys = payload + base + NK + 2 * KB + F + uo + 2;
        u.key_count = U;
        u.offsets = payload + base + NK + 2 * KB + F + uo;
        u.offset_count = 2;
        L.uniq.push_back(u);
        EpsB200Buffer ub = b;
        ub.rows = U;
        L.uniq_blocks.push_back(ub);
        b.data = nullptr;
        uo += U + 2;
      }
      floats += block_rows * dims[f];
    }
    base += NK + 2 * KB + F + UW;
  }
  return L;
}
}  // namespace

int eps_b200_serve(EpsB200Store* store, const uint64_t* payload, const uint64_t* peer_counts,
                   const uint32_t* tables, const uint32_t* poolings, uint32_t requesters,
                   uint32_t feature_count, int32_t read_only, float* partials, void* stream,
                   uint64_t* ticket, EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    Require(payload != nullptr && partials != nullptr, "null sharded round buffer");
    ServeLayout L = MakeServeLayout(s, payload, peer_counts, tables, poolings, requesters,
                                    feature_count, partials, true);
    EpsB200Status inner;
    if (!read_only) {
      // every occurrence joins the ticket (the push sums them in order)
      const int rc = eps_b200_lookup(store, L.feats.data(), L.feats.size(), 1, 0, 1,
                                     L.blocks.data(), stream, ticket, &inner);
      if (rc) throw Failure(rc, inner.message);
    } else {
      // a read-only round gathers only the groups that are not deduplicated
      std::vector<EpsB200Feature> fs;
      std::vector<EpsB200Buffer> bs;
      for (size_t i = 0; i < L.feats.size(); ++i)
        if (L.blocks[i].data) { fs.push_back(L.feats[i]); bs.push_back(L.blocks[i]); }
      if (!fs.empty()) {
        const int rc = eps_b200_lookup(store, fs.data(), fs.size(), 1, 1, 1, bs.data(), stream,
                                       ticket, &inner);
        if (rc) throw Failure(rc, inner.message);
      }
    }
    if (!L.uniq.empty()) {
      uint64_t none = 0;
      const int rc = eps_b200_lookup(store, L.uniq.data(), L.uniq.size(), 1, 1, 1,
                                     L.uniq_blocks.data(), stream, &none, &inner);
      if (rc) {
        if (!read_only) { EpsB200Status st; eps_b200_release(store, *ticket, &st); }
        throw Failure(rc, inner.message);
      }
    }
  });
}

int eps_b200_serve_push(EpsB200Store* store, uint64_t ticket, const float* gradients,
                        const uint64_t* peer_counts, const uint32_t* tables,
                        const uint32_t* poolings, uint32_t requesters, uint32_t feature_count,
                        const uint32_t* reject, void* stream, int32_t wait, EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    Require(gradients != nullptr, "null sharded round buffer");
    static const uint64_t kNoPayload = 0;
    ServeLayout L = MakeServeLayout(s, &kNoPayload, peer_counts, tables, poolings, requesters,
                                    feature_count, gradients, false);
    EpsB200Status inner;
    const int rc = PushEntry(store, ticket, L.blocks.data(), L.blocks.size(), stream, wait,
                             reject, &inner);
    if (rc) throw Failure(rc, inner.message);
  });
}

namespace {
// Shared body of eps_b200_apply_rows / eps_b200_apply_compact.
void ApplyWithContext(EpsB200Store& s, const EpsB200UpdateContext& c, const uint64_t* keys,
                      uint64_t rows, const float* values, bool values_on_device,
                      const EpsB200CompactGradients* compact, void* stream_arg) {
  // src/cache/host_backend.cpp:122-125: a usable optimizer context
  Require(c.beta1_power >= 0 && c.beta1_power < 1 && c.beta2_power >= 0 && c.beta2_power < 1 &&
          std::isfinite(c.learning_rate) && c.learning_rate > 0, "invalid cache optimizer context");
  std::lock_guard lock(s.mutex);
  s.Activate();
  const Table& t = s.Get(c.table);
  Require(!t.hashed, "cache updates address slots of a dense table (key_space > 0)");
  const auto& d = t.def;
  const unsigned D = d.dimension;
  Require(rows == 0 || keys, "null gradient rows");
  std::vector<unsigned long long> slots(rows);
  {
    std::unordered_set<uint64_t> unique;
    unique.reserve(rows * 2);
    for (uint64_t i = 0; i < rows; ++i) {
      Require(unique.insert(keys[i]).second, "duplicate cached gradient row");
      Require(keys[i] < d.key_space && keys[i] % s.opt.shard_count == s.opt.shard_id,
              "cached gradient routed to wrong owner");
      slots[i] = keys[i] / s.opt.shard_count;
    }
  }
  unsigned long long sources = 0, refs = 0;
  if (compact) {
    // src/access/compact_gradients.cpp:10-22 (ValidateCompactGradients)
    const auto& p = *compact;
    Require(p.dimension == D, "compact CUDA table dimension mismatch");
    Require(p.row_offsets && p.row_offsets[0] == 0, "invalid compact gradient offsets");
    for (uint64_t i = 0; i < rows; ++i)
      Require(p.row_offsets[i] <= p.row_offsets[i + 1], "invalid compact gradient offsets");
    refs = p.row_offsets[rows];
    Require(refs == p.refs && (!refs || (p.source_rows && p.scales)), "invalid compact gradient offsets");
    sources = p.sources;
    Require(!sources || p.source_values, "null compact gradient values");
    for (uint64_t j = 0; j < refs; ++j) {
      Require(p.source_rows[j] < sources, "compact gradient source out of range");
      Require(std::isfinite(p.scales[j]) && p.scales[j] >= 0, "invalid compact gradient scale");
    }
    for (uint64_t j = 0; j < sources * D; ++j)
      Require(std::isfinite(p.source_values[j]), "non-finite compact gradient value");
  }
  cudaStream_t stream = s.Use(stream_arg);
  if (rows == 0) return;
  Carver cv;
  const size_t at_slots = cv.take<unsigned long long>(rows);
  const size_t at_vals = cv.take<float>(compact ? sources * D : (values_on_device ? 0 : rows * D));
  const size_t at_off = cv.take<unsigned long long>(compact ? rows + 1 : 0);
  const size_t at_src = cv.take<unsigned long long>(refs);
  const size_t at_sc = cv.take<float>(refs);
  const size_t at_rej = cv.take<unsigned>(1);
  char* slab = nullptr;
  Cuda(cudaMallocAsync(reinterpret_cast<void**>(&slab), cv.offset, stream));
  try {
    auto P = [&](size_t at) { return slab + at; };
    auto H2D = [&](size_t at, const void* src, size_t bytes) {
      if (bytes) Cuda(cudaMemcpyAsync(P(at), src, bytes, cudaMemcpyHostToDevice, stream));
    };
    H2D(at_slots, slots.data(), rows * 8);
    ApplyLaunch lp{};
    if (compact) {
      H2D(at_vals, compact->source_values, sources * D * 4);
      H2D(at_off, compact->row_offsets, (rows + 1) * 8);
      H2D(at_src, compact->source_rows, refs * 8);
      H2D(at_sc, compact->scales, refs * 4);
      lp.source_values = reinterpret_cast<const float*>(P(at_vals));
      lp.row_offsets = reinterpret_cast<const unsigned long long*>(P(at_off));
      lp.source_rows = reinterpret_cast<const unsigned long long*>(P(at_src));
      lp.scales = reinterpret_cast<const float*>(P(at_sc));
      lp.compact = 1;
    } else if (values_on_device) {
      lp.values = values;
    } else {
      H2D(at_vals, values, rows * D * 4);
      lp.values = reinterpret_cast<const float*>(P(at_vals));
    }
    Cuda(cudaMemsetAsync(P(at_rej), 0, sizeof(unsigned), stream));
    PushTable& x = lp.table;
    x.state = t.state;
    x.updates = t.updates;
    x.dtable = t.dtable;
    x.rows = t.rows;
    x.learning_rate = d.learning_rate;
    x.beta1 = d.beta1;
    x.beta2 = d.beta2;
    x.epsilon = d.epsilon;
    x.one_minus_beta1 = 1.0f - d.beta1;
    x.one_minus_beta2 = 1.0f - d.beta2;
    x.has_bounds = d.has_weight_bounds;
    x.bound_min = d.weight_min;
    x.bound_max = d.weight_max;
    x.dim = D;
    // src/cache/host_backend.cpp:127 -- (lr * sqrt(1 - b2p)) / (1 - b1p) in float
    volatile float one_b2 = 1.0f - c.beta2_power, one_b1 = 1.0f - c.beta1_power;
    volatile float num = c.learning_rate * std::sqrt((float)one_b2);
    x.lr_t = num / one_b1;
    lp.slots = reinterpret_cast<const unsigned long long*>(P(at_slots));
    lp.rows = rows;
    lp.reject = reinterpret_cast<unsigned*>(P(at_rej));
    std::vector<unsigned> dims{D};
    const bool a16 = !lp.values || (reinterpret_cast<uintptr_t>(lp.values) & 15) == 0;
    choose_vec(dims, a16, false, &lp.vec, &lp.group, &lp.iters);
    Cuda(launch_apply_rows(lp, stream));
    s.stats.kernel_launches += 2;
    unsigned rej = 0;
    Cuda(cudaMemcpyAsync(&s.host_status[s.opt.max_live_tickets].lookup_error, P(at_rej),
                         sizeof(unsigned), cudaMemcpyDeviceToHost, stream));
    s.Sync(stream);
    rej = s.host_status[s.opt.max_live_tickets].lookup_error;
    char* owned = slab;
    slab = nullptr;
    Cuda(cudaFreeAsync(owned, stream));
    s.Done(stream);
    if (rej) {
      ++s.stats.rejected_updates;
      Require(!(compact && (rej & kRejectReduction)), "compact gradient reduction overflow");
      Require(false, "cached optimizer overflow");
    }
    ++s.stats.updates;
  } catch (...) {
    if (slab) cudaFreeAsync(slab, stream);
    throw;
  }
}
}  // namespace

int eps_b200_apply_rows(EpsB200Store* store, const EpsB200UpdateContext* context,
                        const uint64_t* keys, uint64_t rows, const float* values,
                        int32_t values_on_device, void* stream, EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    Require(context != nullptr, "null optimizer context");
    Require(rows == 0 || values, "null gradient values");
    ApplyWithContext(s, *context, keys, rows, values, values_on_device != 0, nullptr, stream);
  });
}

int eps_b200_apply_compact(EpsB200Store* store, const EpsB200UpdateContext* context,
                           const EpsB200CompactGradients* gradients, void* stream,
                           EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    Require(context && gradients, "null compact gradient arguments");
    ApplyWithContext(s, *context, gradients->keys, gradients->rows, nullptr, false, gradients,
                     stream);
  });
}

int eps_b200_sync_reduce(EpsB200Store* store, uint32_t table, const EpsB200WorkerGradients* workers,
                         uint32_t worker_count, int32_t reduction, uint64_t* keys_out,
                         float* values_out, uint64_t capacity, uint64_t* rows_out, void* stream_arg,
                         EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    Require(workers && rows_out && worker_count >= 1 && worker_count <= 1023,
            "invalid synchronous gradient workers");
    Require(reduction >= EPS_B200_REDUCE_SUM && reduction <= EPS_B200_REDUCE_SAMPLE_MEAN,
            "invalid gradient reduction");
    std::lock_guard lock(s.mutex);
    s.Activate();
    const Table& t = s.Get(table);
    const unsigned D = t.def.dimension;
    // synchronous_gradients.cpp:92-97,104: the denominator and per-worker scale
    double denominator = 1;
    if (reduction == EPS_B200_REDUCE_WORKER_MEAN) denominator = worker_count;
    else if (reduction == EPS_B200_REDUCE_SAMPLE_MEAN) {
      denominator = 0;
      for (uint32_t w = 0; w < worker_count; ++w) denominator += double(workers[w].sample_count);
    }
    std::vector<double> scale(worker_count);
    std::vector<unsigned long long> row_base(worker_count + 1, 0);
    for (uint32_t w = 0; w < worker_count; ++w) {
      const auto& W = workers[w];
      Require(W.sample_count && W.sample_count <= (1ull << 40), "invalid sample count");
      Require(!W.rows || (W.keys && W.values), "null worker gradient buffer");
      scale[w] = (reduction == EPS_B200_REDUCE_SAMPLE_MEAN ? double(W.sample_count) : 1.) / denominator;
      row_base[w + 1] = row_base[w] + W.rows;
    }
    const unsigned long long n = row_base[worker_count];
    Require(n < (1ull << 31), "gradient rows exceed budget", EPS_B200_CAPACITY_EXCEEDED);
    Require(capacity >= n && (!n || (keys_out && values_out)), "reduce output capacity too small");
    cudaStream_t stream = s.Use(stream_arg);
    if (n == 0) { *rows_out = 0; return; }
    const unsigned bits = t.hashed ? 64u : std::max(1u, bits_for(t.def.key_space - 1));
    Carver c;
    const size_t at_w = c.take<SyncWorker>(worker_count);
    const size_t at_base = c.take<unsigned long long>(worker_count + 1);
    const size_t at_scale = c.take<double>(worker_count);
    const size_t at_k0 = c.take<unsigned long long>(n), at_k1 = c.take<unsigned long long>(n);
    const size_t at_r0 = c.take<unsigned>(n), at_r1 = c.take<unsigned>(n);
    const size_t at_seg = c.take<unsigned>(n + 1);
    const size_t at_zero = c.take<char>(sort_scratch_bytes(n, bits));
    const size_t at_segscr = c.take<char>(segment_scratch_bytes(n));
    const size_t at_tot = c.take<unsigned>(2);       // seg_total, error
    const size_t zero_bytes = c.offset - at_zero;
    char* slab = nullptr;
    Cuda(cudaMallocAsync(reinterpret_cast<void**>(&slab), c.offset, stream));
    try {
      auto P = [&](size_t at) { return slab + at; };
      Cuda(cudaMemsetAsync(P(at_zero), 0, zero_bytes, stream));
      s.Stage(P(at_w), workers, worker_count * sizeof(SyncWorker), stream);
      s.Stage(P(at_base), row_base.data(), row_base.size() * 8, stream);
      s.Stage(P(at_scale), scale.data(), scale.size() * 8, stream);
      unsigned* tot = reinterpret_cast<unsigned*>(P(at_tot));
      SyncLaunch lp{};
      lp.workers = reinterpret_cast<const SyncWorker*>(P(at_w));
      lp.worker_count = worker_count;
      lp.row_base = reinterpret_cast<const unsigned long long*>(P(at_base));
      lp.scale = reinterpret_cast<const double*>(P(at_scale));
      lp.total_rows = n;
      lp.dim = D;
      lp.key_space = t.hashed ? ~0ull : t.def.key_space;
      lp.shard_count = s.opt.shard_count;
      lp.shard_id = s.opt.shard_id;
      lp.keys = reinterpret_cast<unsigned long long*>(P(at_k0));
      lp.rows = reinterpret_cast<unsigned*>(P(at_r0));
      lp.error = tot + 1;
      Cuda(launch_sync_pack(lp, stream));
      SortLaunch sp{P(at_k0), P(at_k1), reinterpret_cast<unsigned*>(P(at_r0)),
                    reinterpret_cast<unsigned*>(P(at_r1)), n, bits, 1,
                    reinterpret_cast<unsigned*>(P(at_zero)), sort_tiles(n), tot + 1};
      int swapped = 0;
      Cuda(launch_sort(sp, stream, &swapped));
      SegmentLaunch gl{swapped ? P(at_k1) : P(at_k0), n, 1, reinterpret_cast<unsigned*>(P(at_seg)),
                       tot, reinterpret_cast<unsigned*>(P(at_segscr)), tot + 1};
      Cuda(launch_segments(gl, stream));
      lp.sorted_keys = reinterpret_cast<const unsigned long long*>(swapped ? P(at_k1) : P(at_k0));
      lp.sorted_rows = reinterpret_cast<const unsigned*>(swapped ? P(at_r1) : P(at_r0));
      lp.seg_start = reinterpret_cast<const unsigned*>(P(at_seg));
      lp.seg_total = tot;
      lp.keys_out = reinterpret_cast<unsigned long long*>(keys_out);
      lp.values_out = values_out;
      Cuda(launch_sync_accumulate(lp, stream));
      s.stats.kernel_launches += 2 + segment_launch_count(n) + sort_launch_count(sp);
      unsigned host[2];
      Cuda(cudaMemcpyAsync(host, tot, sizeof(host), cudaMemcpyDeviceToHost, stream));
      s.Sync(stream);
      char* owned = slab;
      slab = nullptr;
      Cuda(cudaFreeAsync(owned, stream));
      s.Done(stream);
      const unsigned err = host[1];
      // synchronous_gradients.cpp:75-77 (validation) and :120 (overflow)
      Require(!(err & 3u), "gradient keys must be unique, sorted and owned by this shard");
      Require(!(err & 4u), "non-finite gradient");
      Require(!(err & 16u), "gradient reduction overflow", EPS_B200_RUN_FAILED);
      Require(!(err & kLookupSortFailed), "coalescing sort wait ran out", EPS_B200_RUN_FAILED);
      *rows_out = host[0];
    } catch (...) {
      if (slab) cudaFreeAsync(slab, stream);
      throw;
    }
  });
}

}  // extern "C"

// ------------------------------------------------------------------ snapshots
// The reference's checksummed shard snapshot (src/store/snapshot.cpp): little-
// endian u64 / f32 fields, FNV-1a 64 over every byte before the trailing
// checksum.  Layout (format 2; format 1 lacks the weight-bounds field):
//   magic | run (u64 length + bytes) | shard | shard count | partition epoch |
//   tables | per table (ascending id): id, dim, shard count, epoch, lr, b1, b2,
//   eps, initial powers, bounds flag [+ min, max], init min/max, seed,
//   optimizer sequence, beta1/beta2 powers, rows, per row: key, row_updates,
//   w[D] m[D] v[D] | checksum.
namespace {
constexpr uint64_t kSnapMagicV1 = 0x3153504541524853ULL;
constexpr uint64_t kSnapMagicV2 = 0x3253504541524853ULL;
constexpr uint64_t kFnvOffset = 14695981039346656037ULL;
constexpr uint64_t kFnvPrime = 1099511628211ULL;

struct SnapWriter {
  FILE* f;
  uint64_t hash = kFnvOffset;
  std::vector<unsigned char> buf;
  void Bytes(const void* p, size_t n, bool hashed = true) {
    const auto* c = static_cast<const unsigned char*>(p);
    if (hashed) for (size_t i = 0; i < n; ++i) hash = (hash ^ c[i]) * kFnvPrime;
    buf.insert(buf.end(), c, c + n);
    if (buf.size() >= (1u << 20)) Flush();
  }
  void U64(uint64_t v, bool hashed = true) {
    unsigned char b[8];
    for (int i = 0; i < 8; ++i) b[i] = (v >> (8 * i)) & 255;
    Bytes(b, 8, hashed);
  }
  void F32(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    unsigned char b[4];
    for (int i = 0; i < 4; ++i) b[i] = (u >> (8 * i)) & 255;
    Bytes(b, 4);
  }
  void Flush() {
    if (!buf.empty())
      Require(std::fwrite(buf.data(), 1, buf.size(), f) == buf.size(), "snapshot write failed",
              EPS_B200_UNAVAILABLE);
    buf.clear();
  }
};

struct SnapReader {
  const std::vector<unsigned char>& d;
  size_t pos = 0;
  uint64_t hash = kFnvOffset;
  void Bytes(void* p, size_t n, bool hashed = true) {
    Require(pos + n <= d.size(), "snapshot truncated", EPS_B200_UNAVAILABLE);
    std::memcpy(p, d.data() + pos, n);
    if (hashed) for (size_t i = 0; i < n; ++i) hash = (hash ^ d[pos + i]) * kFnvPrime;
    pos += n;
  }
  uint64_t U64(bool hashed = true) {
    unsigned char b[8];
    Bytes(b, 8, hashed);
    uint64_t v = 0;
    for (int i = 0; i < 8; ++i) v |= uint64_t(b[i]) << (8 * i);
    return v;
  }
  float F32() {
    unsigned char b[4];
    Bytes(b, 4);
    uint32_t u = 0;
    for (int i = 0; i < 4; ++i) u |= uint32_t(b[i]) << (8 * i);
    float x;
    std::memcpy(&x, &u, 4);
    Require(std::isfinite(x), "snapshot contains non-finite state");
    return x;
  }
};

struct SnapTable {
  EpsB200Table def{};
  uint64_t sequence = 0;
  float beta1_power = 0, beta2_power = 0;
  std::vector<uint64_t> keys, updates;
  std::vector<float> state;                 // [rows][3D] (w | m | v)
};

std::vector<SnapTable> ParseSnapshot(const std::vector<unsigned char>& bytes, std::string* run,
                                     uint64_t* shard, uint64_t* count, uint64_t* epoch) {
  SnapReader r{bytes};
  const uint64_t magic = r.U64();
  Require(magic == kSnapMagicV1 || magic == kSnapMagicV2, "unsupported snapshot format");
  const uint64_t n = r.U64();
  Require(n <= 1024, "snapshot string too long");
  run->resize(n);
  r.Bytes(run->data(), n);
  *shard = r.U64();
  *count = r.U64();
  *epoch = r.U64();
  const uint64_t tables = r.U64();
  Require(tables <= 1024, "snapshot table count exceeds limit");
  std::vector<SnapTable> out(tables);
  for (auto& t : out) {
    auto& d = t.def;
    const uint64_t id = r.U64(), dim = r.U64(), sc = r.U64();
    Require(id <= UINT32_MAX && dim && dim <= 65536 && sc <= UINT32_MAX,
            "invalid snapshot table definition");
    d.id = (uint32_t)id;
    d.dimension = (uint32_t)dim;
    d.shard_count = (uint32_t)sc;
    d.partition_epoch = r.U64();
    d.learning_rate = r.F32(); d.beta1 = r.F32(); d.beta2 = r.F32(); d.epsilon = r.F32();
    d.initial_beta1_power = r.F32(); d.initial_beta2_power = r.F32();
    if (magic == kSnapMagicV2) {
      const uint64_t enabled = r.U64();
      Require(enabled <= 1, "invalid snapshot weight-bounds flag");
      d.has_weight_bounds = (int32_t)enabled;
      if (enabled) { d.weight_min = r.F32(); d.weight_max = r.F32(); }
    }
    d.initialization_min = r.F32();
    d.initialization_max = r.F32();
    d.initialization_seed = r.U64();
    t.sequence = r.U64();
    t.beta1_power = r.F32();
    t.beta2_power = r.F32();
    Require(t.beta1_power >= 0 && t.beta1_power < 1 && t.beta2_power >= 0 && t.beta2_power < 1,
            "invalid snapshot optimizer state");
    const uint64_t rows = r.U64();
    const uint64_t row_bytes = 16 + 12 * dim;
    Require(rows <= (bytes.size() - r.pos) / row_bytes, "snapshot truncated", EPS_B200_UNAVAILABLE);
    t.keys.resize(rows);
    t.updates.resize(rows);
    t.state.resize(rows * 3 * dim);
    for (uint64_t j = 0; j < rows; ++j) {
      t.keys[j] = r.U64();
      t.updates[j] = r.U64();
      float* row = t.state.data() + j * 3 * dim;
      for (uint64_t i = 0; i < 3 * dim; ++i) row[i] = r.F32();
      for (uint64_t i = 2 * dim; i < 3 * dim; ++i)
        Require(row[i] >= 0, "negative second moment in snapshot");
    }
  }
  const uint64_t actual = r.hash;
  const uint64_t expected = r.U64(false);
  Require(actual == expected, "snapshot checksum mismatch");
  Require(r.pos == bytes.size(), "snapshot contains trailing data");
  return out;
}

bool SameOptimizer(const EpsB200Table& a, const EpsB200Table& b) {
  return a.dimension == b.dimension && a.learning_rate == b.learning_rate && a.beta1 == b.beta1 &&
         a.beta2 == b.beta2 && a.epsilon == b.epsilon &&
         a.initial_beta1_power == b.initial_beta1_power &&
         a.initial_beta2_power == b.initial_beta2_power &&
         a.has_weight_bounds == b.has_weight_bounds &&
         (!a.has_weight_bounds || (a.weight_min == b.weight_min && a.weight_max == b.weight_max)) &&
         a.initialization_min == b.initialization_min &&
         a.initialization_max == b.initialization_max &&
         a.initialization_seed == b.initialization_seed;
}
}  // namespace

extern "C" {

namespace {
std::vector<unsigned char> ReadFile(const char* path) {
  std::vector<unsigned char> bytes;
  FILE* f = std::fopen(path, "rb");
  Require(f != nullptr, "cannot open snapshot", EPS_B200_UNAVAILABLE);
  unsigned char chunk[1 << 16];
  size_t n;
  while ((n = std::fread(chunk, 1, sizeof(chunk), f)) > 0) bytes.insert(bytes.end(), chunk, chunk + n);
  std::fclose(f);
  return bytes;
}
}  // namespace

int eps_b200_snapshot_inspect(const char* path, EpsB200SnapshotInfo* info,
                              EpsB200SnapshotTable* tables, uint64_t capacity,
                              EpsB200Status* status) {
  return Boundary(status, [&] {
    Require(path && info, "invalid snapshot arguments");
    auto bytes = ReadFile(path);
    std::string run;
    uint64_t shard = 0, count = 0, epoch = 0;
    auto parsed = ParseSnapshot(bytes, &run, &shard, &count, &epoch);
    std::memset(info, 0, sizeof(*info));
    uint64_t magic = 0;
    for (int i = 0; i < 8; ++i) magic |= uint64_t(bytes[i]) << (8 * i);
    info->format = magic == kSnapMagicV2 ? 2 : 1;
    std::strncpy(info->run, run.c_str(), sizeof(info->run) - 1);
    info->shard = shard;
    info->shard_count = count;
    info->partition_epoch = epoch;
    for (int i = 0; i < 8; ++i) info->checksum |= uint64_t(bytes[bytes.size() - 8 + i]) << (8 * i);
    info->tables = parsed.size();
    for (uint64_t i = 0; i < parsed.size() && tables && i < capacity; ++i) {
      auto& t = parsed[i];
      tables[i] = EpsB200SnapshotTable{t.def, t.sequence, t.beta1_power, t.beta2_power, t.keys.size()};
    }
  });
}

int eps_b200_snapshot_rows(const char* path, uint64_t table_index, uint64_t* keys,
                           uint64_t* row_updates, float* state, uint64_t capacity,
                           EpsB200Status* status) {
  return Boundary(status, [&] {
    Require(path != nullptr, "invalid snapshot arguments");
    auto bytes = ReadFile(path);
    std::string run;
    uint64_t shard = 0, count = 0, epoch = 0;
    auto parsed = ParseSnapshot(bytes, &run, &shard, &count, &epoch);
    Require(table_index < parsed.size(), "snapshot table index out of range");
    auto& t = parsed[table_index];
    Require(capacity >= t.keys.size(), "snapshot row capacity too small");
    if (keys) std::memcpy(keys, t.keys.data(), t.keys.size() * 8);
    if (row_updates) std::memcpy(row_updates, t.updates.data(), t.updates.size() * 8);
    if (state) std::memcpy(state, t.state.data(), t.state.size() * 4);
  });
}

int eps_b200_snapshot_write(EpsB200Store* store, const char* path, const char* run,
                            int32_t all_rows, EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    Require(path && run && std::strlen(run) > 0 && std::strlen(run) <= 1024, "invalid snapshot arguments");
    std::lock_guard lock(s.mutex);
    s.Activate();
    Require(s.tickets.empty(), "snapshot needs a drained store (live lookup tickets)",
            EPS_B200_UNAVAILABLE);
    cudaStream_t stream = s.Use(nullptr);
    s.Sync(stream);
    const std::string pending = std::string(path) + ".pending";
    FILE* f = std::fopen(pending.c_str(), "wbx");
    Require(f != nullptr, "cannot create snapshot staging file", EPS_B200_UNAVAILABLE);
    try {
      SnapWriter w{f};
      w.U64(kSnapMagicV2);
      const uint64_t n = std::strlen(run);
      w.U64(n);
      w.Bytes(run, n);
      w.U64(s.opt.shard_id);
      w.U64(s.opt.shard_count);
      w.U64(s.opt.partition_epoch);
      w.U64(s.tables.size());
      for (auto& [id, t] : s.tables) {             // ascending id, as the reference's map
        const auto& d = t.def;
        const unsigned D = d.dimension;
        w.U64(d.id); w.U64(D); w.U64(s.opt.shard_count); w.U64(d.partition_epoch);
        w.F32(d.learning_rate); w.F32(d.beta1); w.F32(d.beta2); w.F32(d.epsilon);
        w.F32(d.initial_beta1_power); w.F32(d.initial_beta2_power);
        w.U64(d.has_weight_bounds ? 1 : 0);
        if (d.has_weight_bounds) { w.F32(d.weight_min); w.F32(d.weight_max); }
        w.F32(d.initialization_min); w.F32(d.initialization_max); w.U64(d.initialization_seed);
        DeviceTable dt{};
        Cuda(cudaMemcpy(&dt, t.dtable, sizeof(dt), cudaMemcpyDeviceToHost));
        w.U64(dt.optimizer_sequence); w.F32(dt.beta1_power); w.F32(dt.beta2_power);
        // rows: every updated row (rows never updated hold their initial value,
        // which a restore reproduces), or every row with all_rows
        // a hashed table's rows are its slots in use, with their keys
        uint64_t nslots = t.rows;
        std::vector<unsigned long long> skeys;
        if (t.hashed) {
          unsigned long long used = 0;
          Cuda(cudaMemcpy(&used, t.index.used, 8, cudaMemcpyDeviceToHost));
          nslots = std::min<uint64_t>(used, t.rows);
          skeys.resize(nslots);
          if (nslots)
            Cuda(cudaMemcpy(skeys.data(), t.index.slot_keys, nslots * 8, cudaMemcpyDeviceToHost));
        }
        std::vector<unsigned long long> upd(nslots);
        if (nslots) Cuda(cudaMemcpy(upd.data(), t.updates, nslots * 8, cudaMemcpyDeviceToHost));
        uint64_t rows = 0;
        for (auto u : upd) rows += (all_rows || u) ? 1 : 0;
        w.U64(rows);
        const uint64_t chunk = std::max<uint64_t>(1, (64ull << 20) / (12ull * D));
        std::vector<float> st;
        for (uint64_t b = 0; b < nslots; b += chunk) {
          const uint64_t e = std::min<uint64_t>(nslots, b + chunk);
          bool any = all_rows != 0;
          for (uint64_t i = b; i < e && !any; ++i) any = upd[i] != 0;
          if (!any) continue;
          st.resize((e - b) * 3ull * D);
          Cuda(cudaMemcpy(st.data(), t.state + b * 3ull * D, st.size() * 4, cudaMemcpyDeviceToHost));
          for (uint64_t i = b; i < e; ++i) {
            if (!all_rows && !upd[i]) continue;
            w.U64(t.hashed ? skeys[i] : i * s.opt.shard_count + s.opt.shard_id);   // slot i's key
            w.U64(upd[i]);
            const float* row = st.data() + (i - b) * 3ull * D;
            for (unsigned k = 0; k < 3 * D; ++k) w.F32(row[k]);
          }
        }
      }
      w.U64(w.hash, false);
      w.Flush();
      Require(std::fflush(f) == 0 && ::fsync(fileno(f)) == 0, "snapshot fsync failed",
              EPS_B200_UNAVAILABLE);
      std::fclose(f);
      f = nullptr;
      // link: an atomic publication that never overwrites an existing snapshot
      Require(::link(pending.c_str(), path) == 0, "snapshot already exists or cannot be published",
              EPS_B200_UNAVAILABLE);
      ::unlink(pending.c_str());
    } catch (...) {
      if (f) std::fclose(f);
      ::unlink(pending.c_str());
      throw;
    }
    s.Done(stream);
  });
}

int eps_b200_snapshot_read(EpsB200Store* store, const char* path, const char* new_run,
                           EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    Require(path && new_run, "invalid snapshot arguments");
    std::vector<unsigned char> bytes;
    {
      FILE* f = std::fopen(path, "rb");
      Require(f != nullptr, "cannot open snapshot", EPS_B200_UNAVAILABLE);
      unsigned char chunk[1 << 16];
      size_t n;
      while ((n = std::fread(chunk, 1, sizeof(chunk), f)) > 0) bytes.insert(bytes.end(), chunk, chunk + n);
      std::fclose(f);
    }
    std::string old_run;
    uint64_t shard = 0, count = 0, epoch = 0;
    auto tables = ParseSnapshot(bytes, &old_run, &shard, &count, &epoch);
    // src/store/snapshot.cpp:226-231: a restore starts a new run on the same partition
    Require(old_run != new_run, "restore requires a new run ID");
    std::lock_guard lock(s.mutex);
    s.Activate();
    Require(shard == s.opt.shard_id && count == s.opt.shard_count && epoch == s.opt.partition_epoch,
            "snapshot partition does not match server");
    Require(s.tickets.empty(), "restore needs a drained store (live lookup tickets)",
            EPS_B200_UNAVAILABLE);
    Require(tables.size() == s.tables.size(), "snapshot table set does not match the store");
    for (auto& t : tables) {
      auto it = s.tables.find(t.def.id);
      Require(it != s.tables.end(), "snapshot table is not defined in the store");
      Require(SameOptimizer(t.def, it->second.def) && t.def.shard_count == count &&
              t.def.partition_epoch == epoch, "snapshot table definition differs from the store's");
      const Table& tab = it->second;
      for (auto k : t.keys)
        Require(k % count == shard && (tab.hashed || k < tab.def.key_space),
                "snapshot row outside this shard's key space");
      Require(!tab.hashed || t.keys.size() <= tab.rows, "snapshot rows exceed the table's capacity",
              EPS_B200_CAPACITY_EXCEEDED);
    }
    // every check passed: re-initialise, then write the snapshot's rows and powers
    cudaStream_t stream = s.Use(nullptr);
    for (auto& t : tables) {
      Table& tab = s.tables.at(t.def.id);
      const unsigned D = tab.def.dimension;
      const auto& d = tab.def;
      if (tab.hashed) {
        tab.ClearIndex(stream);              // rows are created again as their keys return
      } else {
        InitLaunch ip{tab.state, tab.updates, tab.rows, D, s.opt.shard_count, s.opt.shard_id,
                      d.id, d.initialization_seed, d.initialization_min, d.initialization_max,
                      d.has_weight_bounds, d.weight_min, d.weight_max};
        Cuda(launch_init(ip, stream));
      }
      DeviceTable dt{};
      dt.beta1_power = t.beta1_power;
      dt.beta2_power = t.beta2_power;
      dt.optimizer_sequence = t.sequence;
      float bound = std::max(std::fabs(d.initialization_min), std::fabs(d.initialization_max));
      if (d.has_weight_bounds)
        bound = std::max(bound, std::max(std::fabs(d.weight_min), std::fabs(d.weight_max)));
      std::memcpy(&dt.state_absmax_bits, &bound, 4);
      Cuda(cudaMemcpyAsync(tab.dtable, &dt, sizeof(dt), cudaMemcpyHostToDevice, stream));
      s.Sync(stream);
      const uint64_t rows = t.keys.size();
      if (!rows) continue;
      std::vector<unsigned long long> slots(rows);
      for (uint64_t j = 0; j < rows; ++j) slots[j] = t.keys[j];
      char* buf = nullptr;
      const size_t kb = align256(rows * 8), pb = align256(rows * 12ull * D), ub = align256(rows * 8);
      const size_t hb = tab.hashed ? align256(rows * 4) : 0;
      Cuda(cudaMallocAsync(reinterpret_cast<void**>(&buf), kb + pb + ub + 2 * hb + 256, stream));
      try {
        Cuda(cudaMemcpyAsync(buf, slots.data(), rows * 8, cudaMemcpyHostToDevice, stream));
        Cuda(cudaMemcpyAsync(buf + kb, t.state.data(), rows * 12ull * D, cudaMemcpyHostToDevice, stream));
        Cuda(cudaMemcpyAsync(buf + kb + pb, t.updates.data(), rows * 8, cudaMemcpyHostToDevice, stream));
        const auto* dkeys = reinterpret_cast<unsigned long long*>(buf);
        if (tab.hashed) {
          auto* rslots = reinterpret_cast<unsigned*>(buf + kb + pb + ub + hb);
          auto* err = reinterpret_cast<unsigned*>(buf + kb + pb + ub + 2 * hb);
          Cuda(cudaMemsetAsync(err, 0, 4, stream));
          ResolveKeys(tab, dkeys, rows, reinterpret_cast<unsigned*>(buf + kb + pb + ub), rslots, err,
                      stream);
          Cuda(launch_write_slots(tab.state, tab.updates, D, rslots, rows,
                                  reinterpret_cast<float*>(buf + kb),
                                  reinterpret_cast<unsigned long long*>(buf + kb + pb), tab.dtable,
                                  stream));
        } else {
          Cuda(launch_write_rows(tab.state, tab.updates, D, tab.rows, s.opt.shard_count, dkeys, rows,
                                 reinterpret_cast<float*>(buf + kb),
                                 reinterpret_cast<unsigned long long*>(buf + kb + pb), tab.dtable,
                                 stream));
        }
        char* owned = buf;
        buf = nullptr;
        Cuda(cudaFreeAsync(owned, stream));
        s.Sync(stream);
      } catch (...) {
        cudaStreamSynchronize(stream);
        if (buf) cudaFreeAsync(buf, stream);
        throw;
      }
    }
    s.Done(stream);
  });
}

}  // extern "C"

namespace eps_b200 {
// Internal queries for the sharded client (client.cu).
bool store_table_dimension(EpsB200Store* s, unsigned table, unsigned* dim) {
  if (!s) return false;
  std::lock_guard lock(s->mutex);
  auto it = s->tables.find(table);
  if (it == s->tables.end()) return false;
  *dim = it->second.def.dimension;
  return true;
}
int store_device(EpsB200Store* s) { return s ? s->opt.device : -1; }
unsigned store_shard(EpsB200Store* s, unsigned* count) {
  *count = s->opt.shard_count;
  return s->opt.shard_id;
}
}  // namespace eps_b200

extern "C" {

int eps_b200_stats(EpsB200Store* store, EpsB200Stats* out, EpsB200Status* status) {
  return Boundary(status, [&] {
    auto& s = *Checked(store);
    Require(out != nullptr, "null stats output");
    std::lock_guard lock(s.mutex);
    s.stats.live_tickets = s.tickets.size();
    s.stats.tables = s.tables.size();
    *out = s.stats;
  });
}

}  // extern "C"
