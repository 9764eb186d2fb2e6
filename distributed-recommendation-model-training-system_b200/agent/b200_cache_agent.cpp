// B200CacheAgent over libeps_b200.so (the interface is described in
// b200_cache_agent.hpp).  Validation and error messages follow the reference's
// CUDA backend (src/cuda/cache_backend.cu) method by method; the device work is
// the B200 store's.
#include "b200_cache_agent.hpp"

#include <algorithm>
#include <cmath>
#include <condition_variable>
#include <deque>
#include <functional>
#include <map>
#include <mutex>
#include <set>
#include <stdexcept>
#include <string>
#include <thread>
#include <unordered_map>
#include <utility>

#include <cuda_runtime_api.h>

#include "eps_b200.h"

namespace eps {
namespace {

constexpr std::uint64_t kSkipped = UINT64_MAX;   // occurrence not served by this agent
constexpr std::uint64_t kMaxLookupFeatures = 1024;

struct AgentFailure {
  Error error;
};

void Require(bool ok, const char* message, Error::Code code = Error::Code::invalid_argument) {
  if (!ok) throw AgentFailure{Error{code, message}};
}

// C ABI status -> eps::Error (the ABI's codes are Error::Code + 1).
void Check(int rc, const EpsB200Status& status) {
  if (rc == EPS_B200_OK) return;
  const int code = rc >= EPS_B200_INVALID_ARGUMENT && rc <= EPS_B200_RUN_FAILED
                       ? rc - 1 : static_cast<int>(Error::Code::run_failed);
  throw AgentFailure{Error{static_cast<Error::Code>(code), status.message}};
}

void CheckCuda(cudaError_t e) {
  if (e == cudaSuccess) return;
  throw AgentFailure{Error{e == cudaErrorMemoryAllocation ? Error::Code::capacity_exceeded
                                                          : Error::Code::run_failed,
                           cudaGetErrorString(e)}};
}

// One worker thread running submitted calls in order (the reference's
// OrderedExecutor contract, src/common/executor.hpp:11-50: a bounded queue whose
// overflow is capacity_exceeded; failures become the future's Error).
class OrderedWorker {
 public:
  explicit OrderedWorker(std::size_t limit) : limit_(limit) {
    thread_ = std::thread([this] {
      for (;;) {
        std::function<void()> job;
        {
          std::unique_lock lock(mutex_);
          changed_.wait(lock, [&] { return stop_ || !jobs_.empty(); });
          if (stop_ && jobs_.empty()) return;
          job = std::move(jobs_.front());
          jobs_.pop_front();
        }
        job();
      }
    });
  }
  ~OrderedWorker() { Stop(); }
  void Stop() {
    std::call_once(stopped_, [this] {
      {
        std::lock_guard lock(mutex_);
        stop_ = true;
      }
      changed_.notify_all();
      thread_.join();
    });
  }
  template <typename T, typename F>
  std::future<Result<T>> Submit(F fn) {
    auto promise = std::make_shared<std::promise<Result<T>>>();
    auto future = promise->get_future();
    {
      std::lock_guard lock(mutex_);
      if (stop_ || jobs_.size() >= limit_) {
        promise->set_value(Error{Error::Code::capacity_exceeded, "agent queue is full"});
        return future;
      }
      jobs_.emplace_back([promise, fn = std::move(fn)]() mutable {
        try {
          promise->set_value(fn());
        } catch (const AgentFailure& f) {
          promise->set_value(f.error);
        } catch (const std::bad_alloc&) {
          promise->set_value(Error{Error::Code::capacity_exceeded, "agent allocation failed"});
        } catch (const std::exception& e) {
          promise->set_value(Error{Error::Code::run_failed, e.what()});
        }
      });
    }
    changed_.notify_one();
    return future;
  }

 private:
  std::size_t limit_;
  std::mutex mutex_;
  std::condition_variable changed_;
  std::deque<std::function<void()>> jobs_;
  bool stop_ = false;
  std::thread thread_;
  std::once_flag stopped_;
};

// Outstanding GatherDevice output bytes (CudaCacheOptions::outstanding_output_bytes).
struct OutputBudget {
  std::mutex mutex;
  std::uint64_t used = 0, limit = 0;
};

// One GatherDevice result: a device allocation shared by its feature views,
// freed when the last view goes (it may outlive the agent).
struct DeviceOutput {
  int device = 0;
  float* data = nullptr;
  std::uint64_t bytes = 0;
  cudaEvent_t ready = nullptr;
  std::shared_ptr<OutputBudget> budget;
  DeviceOutput(int d, std::uint64_t n, std::shared_ptr<OutputBudget> b)
      : device(d), bytes(n), budget(std::move(b)) {
    {
      std::lock_guard lock(budget->mutex);
      Require(n <= budget->limit - budget->used, "outstanding device output budget exhausted",
              Error::Code::capacity_exceeded);
      budget->used += n;
    }
    try {
      CheckCuda(cudaSetDevice(device));
      if (n) CheckCuda(cudaMalloc(reinterpret_cast<void**>(&data), n));
      CheckCuda(cudaEventCreateWithFlags(&ready, cudaEventDisableTiming));
    } catch (...) {
      Release();
      throw;
    }
  }
  ~DeviceOutput() { Release(); }
  void Release() {
    if (data || ready) cudaSetDevice(device);
    if (ready) cudaEventDestroy(ready);
    if (data) cudaFree(data);
    ready = nullptr;
    data = nullptr;
    if (budget) {
      std::lock_guard lock(budget->mutex);
      budget->used -= bytes;
      budget.reset();
    }
  }
};

class DeviceView final : public DeviceTensor {
 public:
  DeviceView(std::shared_ptr<DeviceOutput> owner, std::uint64_t offset, std::uint64_t count)
      : owner_(std::move(owner)), offset_(offset), count_(count) {}
  void* data() const override { return owner_->data ? owner_->data + offset_ : nullptr; }
  std::uint64_t elements() const override { return count_; }
  int device() const override { return owner_->device; }
  void WaitOnStream(void* stream) const override {
    Throw(cudaSetDevice(owner_->device));
    Throw(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), owner_->ready, 0));
  }
  std::vector<float> CopyToHost() const override {
    Throw(cudaSetDevice(owner_->device));
    Throw(cudaEventSynchronize(owner_->ready));
    std::vector<float> values(count_);
    if (count_)
      Throw(cudaMemcpy(values.data(), data(), count_ * sizeof(float), cudaMemcpyDeviceToHost));
    return values;
  }

 private:
  static void Throw(cudaError_t e) {
    if (e != cudaSuccess) throw std::runtime_error(cudaGetErrorString(e));
  }
  std::shared_ptr<DeviceOutput> owner_;
  std::uint64_t offset_, count_;
};

}  // namespace

struct B200CacheAgent::Impl {
  struct Entry {
    LocatedRow location;
    std::uint64_t updates;
  };
  struct Table {
    TableDefinition definition;
    std::vector<std::uint64_t> free;            // free slots, next one at the back
    std::unordered_map<Key, Entry> rows;        // resident rows
  };
  // One feature of a gather: resident rows go to the device lookup, rows
  // transferred from the service's CPU pool are summed here.
  struct Part {
    std::uint32_t feature;
    const Table* table;
    const FeatureInput* input;
    const AgentWork* task;
    bool transfer;
    std::uint64_t rows;                          // output rows
    std::uint64_t output_offset;                 // floats into the gather's output
    std::vector<std::uint64_t> slots;            // per occurrence; kSkipped when not served
  };

  explicit Impl(B200CacheOptions o) : options(o), budget(std::make_shared<OutputBudget>()) {
    if (!(o.rows_per_table > 0 && o.rows_per_table <= (1ULL << 31) && o.queue_limit > 0))
      throw std::invalid_argument("B200 cache agent: invalid cache limits");
    budget->limit = o.outstanding_output_bytes;
    EpsB200Options so{};
    so.device = o.device;
    so.shard_id = 0;
    so.shard_count = 1;                          // slots, not keys: every slot is this store's
    so.max_live_tickets = 1;                     // the agent only reads (read_only lookups)
    so.partition_epoch = 0;
    so.state_bytes = o.state_bytes;
    EpsB200Status st{};
    if (eps_b200_create(&so, &store, &st) != EPS_B200_OK)
      throw std::runtime_error(std::string("B200 cache agent: ") + st.message);
    worker = std::make_unique<OrderedWorker>(o.queue_limit);
  }
  ~Impl() {
    if (worker) worker->Stop();
    // the store synchronizes the last stream it ran on when it is destroyed, so
    // that stream (GatherDevice's) must outlive the store
    eps_b200_destroy(store);
    if (stream) {
      cudaSetDevice(options.device);
      cudaStreamSynchronize(stream);
      cudaStreamDestroy(stream);
    }
  }

  Table& Get(TableId id) {
    auto it = tables.find(id);
    Require(it != tables.end(), "unknown B200 cache table");
    return it->second;
  }
  // The reference's residency check (src/cuda/cache_backend.cu:238-245).
  Entry& Find(const LocatedRow& loc) {
    auto& t = Get(loc.row.table);
    auto it = t.rows.find(loc.row.key);
    Require(it != t.rows.end() && loc.agent == options.agent &&
                it->second.location.generation == loc.generation &&
                it->second.location.slot == loc.slot && it->second.location.home == loc.home,
            "B200 cache generation mismatch", Error::Code::stale_generation);
    return it->second;
  }

  // Validation of a gather (src/cuda/cache_backend.cu:251-308) and the slot of
  // every served occurrence.
  std::vector<Part> Prepare(const std::vector<AgentWork>& work,
                            const std::vector<FeatureInput>& layouts, std::uint64_t* values) {
    std::vector<Part> parts;
    parts.reserve(work.size());
    *values = 0;
    for (const auto& task : work) {
      auto it = std::find_if(layouts.begin(), layouts.end(),
                             [&](const auto& f) { return f.feature == task.feature; });
      Require(it != layouts.end() && task.agent == options.agent &&
                  (task.route == AccessRoute::resident_gpu ||
                   task.route == AccessRoute::transfer_unique),
              "invalid B200 gather work");
      const auto& f = *it;
      const auto& t = Get(f.table);
      const auto dim = t.definition.dimension;
      const bool transfer = task.route == AccessRoute::transfer_unique;
      Require(transfer ? task.transferred_weights.size() == task.rows.size() * dim
                       : task.transferred_weights.empty(),
              "invalid B200 transferred weights");
      if (transfer)
        for (float w : task.transferred_weights)
          Require(std::isfinite(w), "non-finite transferred weight");
      Require(task.occurrence_to_unique.size() == f.keys.size() && !f.offsets.empty() &&
                  f.offsets.front() == 0 && f.offsets.back() == f.keys.size() &&
                  std::is_sorted(f.offsets.begin(), f.offsets.end()),
              "invalid B200 gather layout");
      Part p{f.feature, &t, &f, &task, transfer,
             f.pooling == Pooling::sequence ? f.keys.size() : f.offsets.size() - 1, *values, {}};
      p.slots.resize(f.keys.size());
      for (std::size_t i = 0; i < f.keys.size(); ++i) {
        const auto unique = task.occurrence_to_unique[i];
        if (unique == kSkipped) {
          p.slots[i] = kSkipped;
          continue;
        }
        Require(unique < task.rows.size() && task.rows[unique].row == RowKey{f.table, f.keys[i]},
                "invalid B200 occurrence map");
        if (transfer) {
          Require(task.rows[unique].placement == Placement::cpu,
                  "transferred row is not CPU-owned");
          p.slots[i] = unique;
        } else {
          p.slots[i] = Find(task.rows[unique]).location.slot;
        }
      }
      // keep every feature's output 16-byte aligned in a shared device buffer
      *values += (p.rows * dim + 3) / 4 * 4;
      parts.push_back(std::move(p));
    }
    return parts;
  }

  // Position-order sum of transferred CPU-pool weights (the reference sums them
  // in the same gather, src/cuda/cache_backend.cu:81-94): out starts at 0.
  static void SumTransferred(const Part& p, float* out) {
    const auto dim = p.table->definition.dimension;
    const auto& f = *p.input;
    const float* weights = p.task->transferred_weights.data();
    std::fill(out, out + p.rows * dim, 0.0f);
    for (std::size_t b = 0; b + 1 < f.offsets.size(); ++b)
      for (auto i = f.offsets[b]; i < f.offsets[b + 1]; ++i) {
        if (p.slots[i] == kSkipped) continue;
        float* row = out + (f.pooling == Pooling::sequence ? i : b) * dim;
        const float* w = weights + p.slots[i] * dim;
        for (std::uint32_t d = 0; d < dim; ++d) row[d] += w[d];
      }
  }

  // One eps_b200_lookup per <= 1024 resident features: shard partial (no mean
  // division), read only, padding = the skipped occurrences.  Host inputs make
  // the call synchronous, so errors are reported here.
  void GatherResident(const std::vector<Part>& parts, const std::vector<float*>& outputs,
                      int output_device, cudaStream_t s) {
    std::vector<EpsB200Feature> features;
    std::vector<EpsB200Buffer> buffers;
    auto flush = [&] {
      if (features.empty()) return;
      EpsB200Status st{};
      Check(eps_b200_lookup(store, features.data(), features.size(), 0, 1, 1, buffers.data(),
                            s, nullptr, &st), st);
      features.clear();
      buffers.clear();
    };
    for (std::size_t i = 0; i < parts.size(); ++i) {
      const auto& p = parts[i];
      if (p.transfer) continue;
      const auto& f = *p.input;
      EpsB200Feature x{};
      x.table = f.table;
      x.feature = static_cast<std::uint32_t>(i);   // unique within the call
      x.pooling = f.pooling == Pooling::sequence ? EPS_B200_SEQUENCE : EPS_B200_SUM;
      x.has_padding = 1;
      x.keys = p.slots.data();
      x.key_count = p.slots.size();
      x.offsets = f.offsets.data();
      x.offset_count = f.offsets.size();
      x.valid_lengths = nullptr;
      x.padding_key = kSkipped;
      EpsB200Buffer o{};
      o.feature = x.feature;
      o.rows = p.rows;
      o.columns = p.table->definition.dimension;
      o.data = outputs[i];
      o.device = output_device;
      features.push_back(x);
      buffers.push_back(o);
      if (features.size() == kMaxLookupFeatures) flush();
    }
    flush();
  }

  // Owner and context checks of an update (src/cuda/cache_backend.cu:309-320).
  Table& ValidateUpdate(const UpdateContext& c, const std::vector<RowKey>& rows) {
    auto& t = Get(c.table);
    Require(std::isfinite(c.learning_rate) && c.learning_rate > 0 && c.beta1_power >= 0 &&
                c.beta1_power < 1 && c.beta2_power >= 0 && c.beta2_power < 1,
            "invalid B200 update context");
    std::set<Key> unique;
    for (const auto& row : rows) {
      auto it = t.rows.find(row.key);
      Require(row.table == c.table && unique.insert(row.key).second && it != t.rows.end() &&
                  it->second.location.home == c.shard && it->second.updates != UINT64_MAX,
              "invalid B200 gradient owner/counter");
    }
    return t;
  }
  std::vector<std::uint64_t> Slots(Table& t, const std::vector<RowKey>& rows) {
    std::vector<std::uint64_t> slots(rows.size());
    for (std::size_t i = 0; i < rows.size(); ++i) slots[i] = t.rows.at(rows[i].key).location.slot;
    return slots;
  }
  static EpsB200UpdateContext Context(const UpdateContext& c) {
    EpsB200UpdateContext x{};
    x.table = c.table;
    x.learning_rate = c.learning_rate;
    x.beta1_power = c.beta1_power;
    x.beta2_power = c.beta2_power;
    x.optimizer_sequence = c.optimizer_sequence;
    return x;
  }

  cudaStream_t Stream() {
    if (!stream) {
      CheckCuda(cudaSetDevice(options.device));
      CheckCuda(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    }
    return stream;
  }

  B200CacheOptions options;
  EpsB200Store* store = nullptr;
  std::map<TableId, Table> tables;
  std::uint64_t allocated_state = 0;
  std::shared_ptr<OutputBudget> budget;
  cudaStream_t stream = nullptr;                // GatherDevice's stream, created on first use
  // Last member: the worker stops before the state its jobs reference goes.
  std::unique_ptr<OrderedWorker> worker;
};

B200CacheAgent::B200CacheAgent(B200CacheOptions options)
    : impl_(std::make_unique<Impl>(options)) {}

B200CacheAgent::~B200CacheAgent() { impl_->worker->Stop(); }

// CacheBackend::Define (src/cuda/cache_backend.cu:353-371): a table of
// rows_per_table slots, idempotent for an identical definition.
std::future<Result<Ack>> B200CacheAgent::Define(TableDefinition d) {
  return impl_->worker->Submit<Ack>([this, d] {
    const auto& o = d.optimizer;
    if (o.weight_bounds)
      Require(std::isfinite(o.weight_bounds->minimum) && std::isfinite(o.weight_bounds->maximum) &&
                  o.weight_bounds->minimum <= o.weight_bounds->maximum,
              "invalid optimizer weight bounds");
    Require(d.dimension > 0 && d.dimension <= 65536, "invalid B200 cache dimension");
    if (auto it = impl_->tables.find(d.id); it != impl_->tables.end()) {
      Require(it->second.definition == d, "B200 cache table configuration mismatch");
      return Ack{};
    }
    const auto slots = impl_->options.rows_per_table;
    const auto bytes = slots * (std::uint64_t(d.dimension) * 12 + 8);
    Require(impl_->allocated_state <= impl_->options.state_bytes &&
                bytes <= impl_->options.state_bytes - impl_->allocated_state,
            "B200 cache table state budget exhausted", Error::Code::capacity_exceeded);
    EpsB200Table t{};
    t.id = d.id;
    t.dimension = d.dimension;
    t.shard_count = 1;
    t.has_weight_bounds = o.weight_bounds.has_value() ? 1 : 0;
    t.partition_epoch = 0;
    t.learning_rate = o.learning_rate;
    t.beta1 = o.beta1;
    t.beta2 = o.beta2;
    t.epsilon = o.epsilon;
    t.initial_beta1_power = o.initial_beta1_power;
    t.initial_beta2_power = o.initial_beta2_power;
    t.weight_min = o.weight_bounds ? o.weight_bounds->minimum : 0.0f;
    t.weight_max = o.weight_bounds ? o.weight_bounds->maximum : 0.0f;
    t.initialization_min = d.initialization_min;
    t.initialization_max = d.initialization_max;
    t.initialization_seed = d.initialization_seed;
    t.key_space = slots;
    EpsB200Status st{};
    Check(eps_b200_create_table(impl_->store, &t, &st), st);
    Impl::Table table;
    table.definition = d;
    table.free.resize(slots);
    for (std::uint64_t i = 0; i < slots; ++i) table.free[i] = slots - 1 - i;
    impl_->tables.emplace(d.id, std::move(table));
    impl_->allocated_state += bytes;
    return Ack{};
  });
}

std::future<Result<std::uint64_t>> B200CacheAgent::FreeSlots(TableId id) {
  return impl_->worker->Submit<std::uint64_t>(
      [this, id] { return std::uint64_t(impl_->Get(id).free.size()); });
}

// CacheBackend::Load (src/cuda/cache_backend.cu:378-460): validate every row,
// take slots (rolled back on failure), write the states with one
// eps_b200_load_state per table.
std::future<Result<std::vector<LocatedRow>>> B200CacheAgent::Load(MigrationPlan plan,
                                                                 std::vector<RowState> states) {
  return impl_->worker->Submit<std::vector<LocatedRow>>(
      [this, plan = std::move(plan), states = std::move(states)] {
        Require(plan.agent == impl_->options.agent && plan.rows.size() == states.size() &&
                    plan.destination == Placement::gpu,
                "invalid B200 load plan");
        std::map<TableId, std::vector<std::size_t>> groups;
        std::set<std::pair<TableId, Key>> unique;
        for (std::size_t i = 0; i < states.size(); ++i) {
          const auto& row = states[i];
          auto& t = impl_->Get(row.row.table);
          const auto dim = t.definition.dimension;
          Require(row.row == plan.rows[i].row && !t.rows.contains(row.row.key) &&
                      unique.emplace(row.row.table, row.row.key).second,
                  "duplicate/existing B200 load row");
          Require(row.weights.size() == dim && row.first_moment.size() == dim &&
                      row.second_moment.size() == dim,
                  "B200 load shape mismatch");
          for (auto* v : {&row.weights, &row.first_moment, &row.second_moment})
            for (auto x : *v) Require(std::isfinite(x), "non-finite B200 load state");
          for (auto x : row.second_moment) Require(x >= 0, "negative B200 second moment");
          groups[row.row.table].push_back(i);
        }
        for (const auto& [id, rows] : groups) {
          auto& t = impl_->Get(id);
          Require(plan.reserve_slots <= t.free.size() &&
                      rows.size() <= t.free.size() - plan.reserve_slots,
                  "B200 cache slots or reserve exhausted", Error::Code::capacity_exceeded);
        }
        std::vector<LocatedRow> result(states.size());
        std::vector<std::pair<TableId, Key>> inserted;
        inserted.reserve(states.size());
        try {
          for (const auto& [id, rows] : groups) {
            auto& t = impl_->Get(id);
            const auto dim = t.definition.dimension;
            std::vector<std::uint64_t> slots, updates;
            std::vector<float> w, m, v;
            slots.reserve(rows.size());
            updates.reserve(rows.size());
            w.reserve(rows.size() * dim);
            m.reserve(rows.size() * dim);
            v.reserve(rows.size() * dim);
            for (auto i : rows) {
              const auto slot = t.free.back();
              auto loc = plan.rows[i];
              loc.slot = slot;
              loc.agent = impl_->options.agent;
              loc.placement = Placement::gpu;
              t.rows.emplace(loc.row.key, Impl::Entry{loc, states[i].row_updates});
              t.free.pop_back();
              inserted.emplace_back(id, loc.row.key);
              result[i] = loc;
              slots.push_back(slot);
              updates.push_back(states[i].row_updates);
              w.insert(w.end(), states[i].weights.begin(), states[i].weights.end());
              m.insert(m.end(), states[i].first_moment.begin(), states[i].first_moment.end());
              v.insert(v.end(), states[i].second_moment.begin(), states[i].second_moment.end());
            }
            EpsB200Status st{};
            Check(eps_b200_load_state(impl_->store, id, slots.data(), slots.size(), w.data(),
                                      m.data(), v.data(), updates.data(), &st),
                  st);
          }
          return result;
        } catch (...) {
          for (auto [id, key] : inserted) {
            auto& t = impl_->Get(id);
            t.free.push_back(t.rows.at(key).location.slot);
            t.rows.erase(key);
          }
          throw;
        }
      });
}

// CacheBackend::GatherHost (src/cuda/cache_backend.cu:462-479).
std::future<Result<std::vector<TensorBlock>>> B200CacheAgent::GatherHost(
    std::vector<AgentWork> work, std::vector<FeatureInput> layouts) {
  return impl_->worker->Submit<std::vector<TensorBlock>>(
      [this, work = std::move(work), layouts = std::move(layouts)] {
        std::uint64_t values = 0;
        auto parts = impl_->Prepare(work, layouts, &values);
        std::vector<TensorBlock> out;
        out.reserve(parts.size());
        std::vector<float*> outputs;
        outputs.reserve(parts.size());
        for (const auto& p : parts) {
          const auto dim = p.table->definition.dimension;
          out.push_back({p.feature, {p.rows, dim}, std::vector<float>(p.rows * dim)});
          outputs.push_back(out.back().values.data());
        }
        impl_->GatherResident(parts, outputs, -1, nullptr);
        for (std::size_t i = 0; i < parts.size(); ++i)
          if (parts[i].transfer) Impl::SumTransferred(parts[i], outputs[i]);
        return out;
      });
}

// GpuCacheAgent::GatherDevice (src/cuda/cache_backend.cu:480-498): one device
// allocation per call holds every feature; the views keep it alive.
std::future<Result<std::vector<DeviceTensorBlock>>> B200CacheAgent::GatherDevice(
    std::vector<AgentWork> work, std::vector<FeatureInput> layouts) {
  return impl_->worker->Submit<std::vector<DeviceTensorBlock>>(
      [this, work = std::move(work), layouts = std::move(layouts)] {
        std::uint64_t values = 0;
        auto parts = impl_->Prepare(work, layouts, &values);
        const cudaStream_t s = impl_->Stream();
        auto output = std::make_shared<DeviceOutput>(impl_->options.device, values * 4,
                                                     impl_->budget);
        std::vector<float*> outputs;
        outputs.reserve(parts.size());
        for (const auto& p : parts) outputs.push_back(output->data + p.output_offset);
        impl_->GatherResident(parts, outputs, impl_->options.device, s);
        std::vector<std::vector<float>> staged;
        for (std::size_t i = 0; i < parts.size(); ++i) {
          if (!parts[i].transfer || !parts[i].rows) continue;
          staged.emplace_back(parts[i].rows * parts[i].table->definition.dimension);
          Impl::SumTransferred(parts[i], staged.back().data());
          CheckCuda(cudaMemcpyAsync(outputs[i], staged.back().data(),
                                    staged.back().size() * sizeof(float),
                                    cudaMemcpyHostToDevice, s));
        }
        CheckCuda(cudaEventRecord(output->ready, s));
        // the staged host sums must outlive their copies
        if (!staged.empty()) CheckCuda(cudaEventSynchronize(output->ready));
        std::vector<DeviceTensorBlock> out;
        out.reserve(parts.size());
        for (const auto& p : parts) {
          const auto dim = p.table->definition.dimension;
          out.push_back({p.feature, {p.rows, dim},
                         std::make_shared<DeviceView>(output, p.output_offset, p.rows * dim)});
        }
        return out;
      });
}

// CacheBackend::ApplyHost (src/cuda/cache_backend.cu:499-513; LazyAdam of
// src/cache/host_backend.cpp:119-146 with the context's powers).
std::future<Result<Ack>> B200CacheAgent::ApplyHost(UpdateContext c, RowGradients g) {
  return impl_->worker->Submit<Ack>([this, c, g = std::move(g)] {
    auto& t = impl_->ValidateUpdate(c, g.rows);
    const auto dim = t.definition.dimension;
    Require(g.values.size() == g.rows.size() * dim, "invalid B200 gradient shape");
    if (g.rows.empty()) return Ack{};
    const auto slots = impl_->Slots(t, g.rows);
    const auto x = Impl::Context(c);
    EpsB200Status st{};
    Check(eps_b200_apply_rows(impl_->store, &x, slots.data(), slots.size(), g.values.data(), 0,
                              nullptr, &st),
          st);
    for (const auto& row : g.rows) ++t.rows.at(row.key).updates;
    return Ack{};
  });
}

// CacheBackend::ApplyCompact (src/cuda/cache_backend.cu:514-539): the CSR
// packet's own validation (src/access/compact_gradients.cpp:43-72) and the
// in-order expansion run in eps_b200_apply_compact.
std::future<Result<Ack>> B200CacheAgent::ApplyCompact(UpdateContext c, CompactGradients p) {
  return impl_->worker->Submit<Ack>([this, c, p = std::move(p)] {
    auto& t = impl_->ValidateUpdate(c, p.rows);
    const auto dim = t.definition.dimension;
    Require(p.dimension == dim, "compact B200 table dimension mismatch");
    Require(p.source_values.size() % dim == 0, "invalid compact gradient values");
    if (p.rows.empty()) return Ack{};
    Require(p.row_offsets.size() == p.rows.size() + 1 && p.source_rows.size() == p.scales.size(),
            "invalid compact gradient offsets");
    const auto slots = impl_->Slots(t, p.rows);
    EpsB200CompactGradients cg{};
    cg.keys = slots.data();
    cg.rows = slots.size();
    cg.dimension = p.dimension;
    cg.source_values = p.source_values.data();
    cg.sources = p.source_values.size() / dim;
    cg.row_offsets = p.row_offsets.data();
    cg.source_rows = p.source_rows.data();
    cg.scales = p.scales.data();
    cg.refs = p.scales.size();
    const auto x = Impl::Context(c);
    EpsB200Status st{};
    Check(eps_b200_apply_compact(impl_->store, &x, &cg, nullptr, &st), st);
    for (const auto& row : p.rows) ++t.rows.at(row.key).updates;
    return Ack{};
  });
}

// CacheBackend::ReadBack (src/cuda/cache_backend.cu:540-580): rows stay resident.
std::future<Result<std::vector<RowState>>> B200CacheAgent::ReadBack(MigrationPlan plan) {
  return impl_->worker->Submit<std::vector<RowState>>([this, plan = std::move(plan)] {
    std::map<TableId, std::vector<std::size_t>> groups;
    for (std::size_t i = 0; i < plan.rows.size(); ++i) {
      impl_->Find(plan.rows[i]);
      groups[plan.rows[i].row.table].push_back(i);
    }
    std::vector<RowState> out(plan.rows.size());
    for (const auto& [id, rows] : groups) {
      const auto dim = impl_->Get(id).definition.dimension;
      std::vector<std::uint64_t> slots, updates(rows.size());
      for (auto i : rows) slots.push_back(plan.rows[i].slot);
      std::vector<float> w(rows.size() * dim), m(rows.size() * dim), v(rows.size() * dim);
      EpsB200Status st{};
      Check(eps_b200_read_state(impl_->store, id, slots.data(), slots.size(), w.data(), m.data(),
                                v.data(), updates.data(), &st),
            st);
      for (std::size_t k = 0; k < rows.size(); ++k) {
        auto& r = out[rows[k]];
        r.row = plan.rows[rows[k]].row;
        r.weights.assign(w.begin() + k * dim, w.begin() + (k + 1) * dim);
        r.first_moment.assign(m.begin() + k * dim, m.begin() + (k + 1) * dim);
        r.second_moment.assign(v.begin() + k * dim, v.begin() + (k + 1) * dim);
        r.row_updates = updates[k];
      }
    }
    return out;
  });
}

// CacheBackend::CommitEviction (src/cuda/cache_backend.cu:581-594).
std::future<Result<Ack>> B200CacheAgent::CommitEviction(MigrationPlan plan) {
  return impl_->worker->Submit<Ack>([this, plan = std::move(plan)] {
    std::set<std::pair<TableId, Key>> unique;
    for (const auto& loc : plan.rows) {
      impl_->Find(loc);
      Require(unique.emplace(loc.row.table, loc.row.key).second, "duplicate B200 eviction row");
    }
    for (const auto& loc : plan.rows) {
      auto& t = impl_->Get(loc.row.table);
      t.free.push_back(loc.slot);
      t.rows.erase(loc.row.key);
    }
    return Ack{};
  });
}

}  // namespace eps
