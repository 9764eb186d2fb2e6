// ref_harness.cpp -- drives the UNMODIFIED reference CPU parameter server
// (eps_core compiled from the reference sources by oracle/Makefile) through its
// own public API: n in-process CpuParameterService shards behind a
// DistributedClient (include/eps/distributed_client.hpp:32-70), exactly as the
// reference's tests/weight_bounds_tests.cpp:23-33 does.
//
// TEST INFRASTRUCTURE ONLY: used by tests/golden/make_golden.py, the parity
// tests and bench.py's CPU-baseline / --impl reference legs.  Never linked by
// the product.
//
// Exposes a small C interface so Python (ctypes) can call it.
#include <algorithm>
#include <chrono>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "eps/distributed_client.hpp"
#include "eps/prepared_lookup.hpp"
#include "eps/runtime.hpp"
#ifdef EPS_REF_CUDA
#include "eps/cache_resolver.hpp"
#include "eps/cuda_cache_backend.hpp"
#endif

using namespace eps;

namespace {
struct Harness {
  std::vector<std::shared_ptr<CpuParameterService>> shards;
  std::unique_ptr<DistributedClient> client;
  std::map<std::uint64_t, DistributedBatch> batches;
  std::uint64_t sequence = 0;
  std::string run = "oracle";
  std::uint32_t learner = 0;
  std::shared_ptr<CacheBackend> agent;   // the reference's CUDA backend, when attached
};

void Message(char* err, const std::string& text) {
  if (err) { std::strncpy(err, text.c_str(), 1023); err[1023] = 0; }
}
template <typename T> int Take(Result<T>&& r, T* out, char* err) {
  if (auto e = std::get_if<Error>(&r)) { Message(err, e->message); return int(e->code) + 1; }
  if (out) *out = std::get<T>(std::move(r));
  return 0;
}
}  // namespace

extern "C" {

struct RhTable {
  std::uint32_t id, dimension;
  float learning_rate, beta1, beta2, epsilon, initial_beta1_power, initial_beta2_power;
  std::int32_t has_bounds; float bound_min, bound_max;
  float init_min, init_max; std::uint64_t init_seed;
};

struct RhFeature {
  std::uint32_t table, feature, pooling;
  const std::uint64_t* keys; std::uint64_t key_count;
  const std::uint64_t* offsets; std::uint64_t offset_count;
};

void* rh_create_run(std::uint32_t shard_count, std::uint64_t state_bytes, const char* run,
                    const char* snapshot_dir, char* err) {
  try {
    auto h = std::make_unique<Harness>();
    if (run) h->run = run;
    for (std::uint32_t s = 0; s < shard_count; ++s) {
      RuntimeOptions o;
      o.run_id = h->run; o.shard_id = s; o.shard_count = shard_count;
      if (snapshot_dir) o.snapshot_directory = snapshot_dir;
      // Raise the default request/ticket budgets (include/eps/runtime.hpp:20-23)
      // so the benchmark batch sizes are admitted.
      o.state_bytes = state_bytes;
      o.max_request_bytes = 1ULL << 40;
      o.ticket_payload_bytes = 1ULL << 40;
      o.queue_payload_bytes = 1ULL << 40;
      o.dependency_payload_bytes = 1ULL << 40;
      h->shards.push_back(std::make_shared<CpuParameterService>(o));
    }
    std::vector<std::shared_ptr<ParameterService>> services(h->shards.begin(), h->shards.end());
    h->client = std::make_unique<DistributedClient>(services);
    return h.release();
  } catch (const std::exception& e) { Message(err, e.what()); return nullptr; }
}

void* rh_create(std::uint32_t shard_count, std::uint64_t state_bytes, char* err) {
  return rh_create_run(shard_count, state_bytes, nullptr, nullptr, err);
}

void rh_destroy(void* p) { delete static_cast<Harness*>(p); }

// CpuParameterService::DrainAndFlush (include/eps/runtime.hpp:116-117) on one
// shard: writes its snapshot state file; the path goes to path_out.
int rh_snapshot(void* p, std::uint32_t shard, const char* id, char* path_out, char* err) {
  auto& h = *static_cast<Harness*>(p);
  try {
    SnapshotMetadata meta;
    const int rc = Take(h.shards.at(shard)->DrainAndFlush(id).get(), &meta, err);
    if (rc) return rc;
    Message(path_out, meta.state_files.at(0));
    return 0;
  } catch (const std::exception& e) { Message(err, e.what()); return 6; }
}

// CpuParameterService::Restore (include/eps/runtime.hpp:121) of one shard.
int rh_restore(void* p, std::uint32_t shard, const char* path, char* err) {
  auto& h = *static_cast<Harness*>(p);
  try {
    Ack ack;
    return Take(h.shards.at(shard)->Restore(path).get(), &ack, err);
  } catch (const std::exception& e) { Message(err, e.what()); return 6; }
}

int rh_create_table(void* p, const RhTable* t, char* err) {
  auto& h = *static_cast<Harness*>(p);
  TableDefinition d{t->id, t->dimension, std::uint32_t(h.shards.size()), 1,
      {t->learning_rate, t->beta1, t->beta2, t->epsilon, t->initial_beta1_power,
       t->initial_beta2_power}, t->init_min, t->init_max, t->init_seed};
  if (t->has_bounds) d.optimizer.weight_bounds = WeightBounds{t->bound_min, t->bound_max};
  Ack ack;
  return Take(h.client->CreateTable(d), &ack, err);
}

// Lookup through PrepareLookupInputs with raised limits + LookupPrepared
// (the default-limit Lookup would reject benchmark-sized batches,
// src/client/distributed_client.cpp:39).  outputs[f] receive the merged,
// mean-normalised feature tensors.
int rh_lookup(void* p, std::uint32_t count, const RhFeature* features, std::int32_t read_only,
              float** outputs, std::uint64_t* batch_out, char* err) {
  auto& h = *static_cast<Harness*>(p);
  std::vector<FeatureInput> input;
  for (std::uint32_t i = 0; i < count; ++i) {
    const auto& f = features[i];
    FeatureInput x{f.table, f.feature, static_cast<Pooling>(f.pooling),
                   std::vector<Key>(f.keys, f.keys + f.key_count),
                   std::vector<std::uint64_t>(f.offsets, f.offsets + f.offset_count), {}};
    for (std::uint64_t b = 0; b + 1 < f.offset_count; ++b)
      x.valid_lengths.push_back(f.offsets[b + 1] - f.offsets[b]);
    input.push_back(std::move(x));
  }
  PreparationLimits limits{1ULL << 40, 1ULL << 40, 1024};
  auto prepared = PrepareLookupInputs(std::move(input), h.shards.size(), limits);
  PreparedLookup lookup;
  if (int rc = Take(std::move(prepared), &lookup, err)) return rc;
  const auto seq = h.sequence++;
  auto result = h.client->LookupPrepared({h.run, h.learner, seq, Phase::lookup}, 1,
                                         read_only != 0, std::move(lookup));
  DistributedBatch batch;
  if (int rc = Take(std::move(result), &batch, err)) return rc;
  for (std::uint32_t i = 0; i < count; ++i) {
    const auto& values = batch.features()[i].values;
    if (outputs && outputs[i]) std::memcpy(outputs[i], values.data(), values.size() * 4);
  }
  h.batches.emplace(seq, std::move(batch));
  if (batch_out) *batch_out = seq;
  return 0;
}

int rh_push(void* p, std::uint64_t batch, std::uint32_t count, const std::uint32_t* feature_ids,
            const float* const* grads, const std::uint64_t* rows, const std::uint32_t* dims,
            char* err) {
  auto& h = *static_cast<Harness*>(p);
  auto it = h.batches.find(batch);
  if (it == h.batches.end()) { Message(err, "unknown batch"); return 1; }
  std::vector<TensorBlock> gradients;
  for (std::uint32_t i = 0; i < count; ++i)
    gradients.push_back({feature_ids[i], {rows[i], dims[i]},
                         std::vector<float>(grads[i], grads[i] + rows[i] * dims[i])});
  Ack ack;
  int rc = Take(h.client->Push(it->second, std::move(gradients)), &ack, err);
  if (rc == 0) h.batches.erase(it);
  return rc;
}

int rh_release(void* p, std::uint64_t batch, char* err) {
  auto& h = *static_cast<Harness*>(p);
  auto it = h.batches.find(batch);
  if (it == h.batches.end()) { Message(err, "unknown batch"); return 1; }
  Ack ack;
  int rc = Take(h.client->Release(it->second), &ack, err);
  h.batches.erase(it);
  return rc;
}

// ParameterService::ReadState for one row on its home shard key % n.
int rh_read(void* p, std::uint32_t table, std::uint64_t key, float* w, float* m, float* v,
            std::uint64_t* updates, char* err) {
  auto& h = *static_cast<Harness*>(p);
  const auto home = ShardId(key % h.shards.size());
  std::vector<RowState> rows;
  int rc = Take(h.shards[home]->ReadState({{{table, key}, home, Placement::cpu, 0, 0, 0}}).get(),
                &rows, err);
  if (rc) return rc;
  const auto& r = rows.at(0);
  std::memcpy(w, r.weights.data(), r.weights.size() * 4);
  std::memcpy(m, r.first_moment.data(), r.first_moment.size() * 4);
  std::memcpy(v, r.second_moment.data(), r.second_moment.size() * 4);
  *updates = r.row_updates;
  return 0;
}

// ParameterService::ReadState of many rows of one table: the keys are grouped by
// home shard (key % n) and read in chunks of 4096 rows per call, within the
// service's request byte budget.  w / m / v are [count][dimension].
int rh_read_many(void* p, std::uint32_t table, const std::uint64_t* keys, std::uint64_t count,
                 std::uint32_t dimension, float* w, float* m, float* v, std::uint64_t* updates,
                 char* err) {
  auto& h = *static_cast<Harness*>(p);
  const std::size_t n = h.shards.size();
  std::vector<std::vector<std::uint64_t>> by_shard(n);
  for (std::uint64_t i = 0; i < count; ++i) by_shard[keys[i] % n].push_back(i);
  for (std::size_t s = 0; s < n; ++s) {
    const auto& idx = by_shard[s];
    for (std::size_t at = 0; at < idx.size(); at += 4096) {
      const std::size_t end = std::min(idx.size(), at + 4096);
      std::vector<LocatedRow> req;
      req.reserve(end - at);
      for (std::size_t j = at; j < end; ++j)
        req.push_back({{table, keys[idx[j]]}, ShardId(s), Placement::cpu, 0, 0, 0});
      std::vector<RowState> rows;
      if (int rc = Take(h.shards[s]->ReadState(std::move(req)).get(), &rows, err)) return rc;
      if (rows.size() != end - at) { Message(err, "short ReadState reply"); return 6; }
      for (std::size_t j = at; j < end; ++j) {
        const auto& r = rows[j - at];
        const std::uint64_t i = idx[j];
        if (r.weights.size() != dimension) { Message(err, "dimension mismatch"); return 1; }
        std::memcpy(w + i * dimension, r.weights.data(), dimension * 4);
        std::memcpy(m + i * dimension, r.first_moment.data(), dimension * 4);
        std::memcpy(v + i * dimension, r.second_moment.data(), dimension * 4);
        updates[i] = r.row_updates;
      }
    }
  }
  return 0;
}

// Shard-level phase counters (include/eps/runtime.hpp:76-80) summed over shards.
int rh_stats(void* p, std::uint64_t* out4, char* err) {
  auto& h = *static_cast<Harness*>(p);
  out4[0] = out4[1] = out4[2] = out4[3] = 0;
  for (auto& s : h.shards) {
    RuntimeStats st;
    if (int rc = Take(s->Stats().get(), &st, err)) return rc;
    out4[0] += st.lookup_prepare_nanoseconds;
    out4[1] += st.gradient_prepare_nanoseconds;
    out4[2] += st.cpu_optimizer_nanoseconds;
    out4[3] += st.rows;
  }
  return 0;
}


#ifdef EPS_REF_CUDA
// The reference's own GPU path on one GPU (libeps_ref_cuda.so only): its
// CudaCacheBackend (src/cuda/cache_backend.cu, compiled from the reference
// sources for sm_100a) attached to the single shard as agent 0, the given rows
// of `table` migrated to it with MoveRows, and the client's gathers resolved
// through the reference's MakeCacheResolver -- the wiring of the reference's
// tests/cache_tests.cpp:45-49 with the CUDA backend in place of the host one.
// Lookups and pushes of those rows then run the reference's CUDA kernels.  The
// backend is attached by the first call; later calls migrate more rows (of any
// table) to it.
int rh_attach_cuda(void* p, std::int32_t device, std::uint64_t rows_per_table,
                   std::uint64_t state_bytes, std::uint32_t table, std::uint32_t dimension,
                   const std::uint64_t* keys, std::uint64_t key_count, char* err) {
  auto& h = *static_cast<Harness*>(p);
  if (h.shards.size() != 1) { Message(err, "the CUDA agent path runs one shard"); return 1; }
  try {
    if (!h.agent) {                               // attached once; later calls only migrate
      CudaCacheOptions o;
      o.agent = 0;
      o.device = device;
      o.state_bytes = state_bytes;
      o.rows_per_table = rows_per_table;
      o.transfer_bytes = 64ULL << 20;             // the backend's maximum staging
      o.outstanding_output_bytes = 1ULL << 30;
      auto backend = std::make_shared<CudaCacheBackend>(o);
      Ack ack;
      if (int rc = Take(h.shards[0]->AttachAgent(0, backend).get(), &ack, err)) return rc;
      if (int rc = Take(h.shards[0]->ConfigureAccess(0, AccessRoute::transfer_unique).get(), &ack, err))
        return rc;
      h.agent = backend;
      h.client->SetCacheResolver(MakeCacheResolver({{0, backend}}));
    }
    // migrate in chunks within the service's 4096 rows per MoveRows
    // (src/server/service.cpp:394) and the backend's staging buffer
    const std::uint64_t chunk = std::min<std::uint64_t>(
        4096, std::max<std::uint64_t>(1, (16ULL << 20) / (12ULL * dimension + 8)));
    for (std::uint64_t i = 0; i < key_count; i += chunk) {
      std::vector<RowKey> rows;
      for (std::uint64_t k = i; k < std::min(key_count, i + chunk); ++k) rows.push_back({table, keys[k]});
      MoveRowsRequest move{h.run, std::move(rows), 0, Placement::gpu, {1ULL << 40, 64ULL << 20, 8, 0}};
      std::vector<LocatedRow> moved;
      if (int rc = Take(h.shards[0]->MoveRows(std::move(move)).get(), &moved, err)) return rc;
    }
    return 0;
  } catch (const std::exception& e) { Message(err, e.what()); return int(Error::Code::run_failed) + 1; }
}
#endif

}  // extern "C"
