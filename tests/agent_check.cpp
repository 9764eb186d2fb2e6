// agent_check.cpp -- drives eps::B200CacheAgent (the GpuCacheAgent adapter
// over libeps_b200.so) and the reference's own eps::HostCacheBackend
// (src/cache/host_backend.cpp) through the same seeded calls and requires
// identical results, bit for bit, and identical error codes:
//   1. the backend contract directly: Define, Load, GatherHost (sum / mean /
//      sequence, skipped occurrences, ragged and empty bags, CPU-pool rows
//      transferred with the request), ApplyHost and ApplyCompact rounds with
//      weight bounds, ReadBack, CommitEviction and reload with a new
//      generation, plus rejected calls (stale generation, duplicate rows,
//      wrong owner, optimizer overflow with the state left unchanged);
//   2. as a drop-in behind the reference's shard service: a CpuParameterService
//      with the agent attached (AttachAgent, include/eps/runtime.hpp:133) and a
//      DistributedClient resolving cached rows through GatherHost, in the flow
//      of the reference's tests/cache_tests.cpp -- the same rounds against a
//      service with a HostCacheBackend attached;
//   3. under the reference's AgentRuntime (include/eps/agent_runtime.hpp), the
//      command layer its BRPC agent server dispatches to: retried commands
//      replay their first result without applying twice, older commands are
//      retired, and eviction reclaims the slots -- the same with either backend;
//   4. the adapter alone: slot, reserve and state-budget limits refused whole;
//      calls from four threads (each result equals the single-thread one); and,
//      on a machine with a GPU, GatherDevice results (equal to the host
//      backend's gather, ordered on a consumer stream, outliving the agent).
// Linked against the real library it checks the B200 path; linked against
// oracle/fake_b200_abi.cpp it checks the adapter's host logic without a GPU.
// Prints "agent_check: PASS ..." and exits 0, or names the first difference.
#include <execinfo.h>
#include <unistd.h>

#include <cmath>
#include <csignal>
#include <cstdint>
#include <cstring>
#include <future>
#include <iostream>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <type_traits>
#include <utility>
#include <variant>
#include <vector>

#include <cuda_runtime_api.h>

#include "b200_cache_agent.hpp"
#include "eps/agent_runtime.hpp"
#include "eps/cache_backend.hpp"
#include "eps/distributed_client.hpp"
#include "eps/runtime.hpp"
#include "eps/worker_cache_agent.hpp"

using namespace eps;

// The training process's owner of a cache agent (include/eps/worker_cache_agent.hpp,
// served over BRPC, which is not built here) takes the adapter unchanged.
static_assert(std::is_constructible_v<WorkerCacheAgent, WorkerCacheOptions,
                                      std::shared_ptr<B200CacheAgent>>);
static_assert(std::is_convertible_v<std::shared_ptr<B200CacheAgent>, std::shared_ptr<GpuCacheAgent>>);

namespace {

struct Rng {
  std::uint64_t s;
  std::uint64_t Next() {
    s = s * 6364136223846793005ULL + 1442695040888963407ULL;
    return s >> 11;
  }
  double Unit() { return double(Next() >> 11) * (1.0 / 9007199254740992.0); }
  float Uniform(float lo, float hi) { return float(lo + (hi - lo) * Unit()); }
  std::uint64_t Below(std::uint64_t n) { return Next() % n; }
};

void Check(bool ok, const std::string& what) {
  if (!ok) throw std::runtime_error(what);
}
template <typename T>
T Take(std::future<Result<T>> f, const std::string& what) {
  auto r = f.get();
  if (auto e = std::get_if<Error>(&r)) throw std::runtime_error(what + ": " + e->message);
  return std::get<T>(std::move(r));
}
template <typename T>
T Take(Result<T> r, const std::string& what) {
  if (auto e = std::get_if<Error>(&r)) throw std::runtime_error(what + ": " + e->message);
  return std::get<T>(std::move(r));
}
// Both calls must fail with the same code.
template <typename T>
void SameRejection(std::future<Result<T>> a, std::future<Result<T>> b, const std::string& what) {
  auto x = a.get();
  auto y = b.get();
  auto* ex = std::get_if<Error>(&x);
  auto* ey = std::get_if<Error>(&y);
  Check(ex && ey, what + ": expected both backends to reject (b200 " +
                      (ex ? "rejected" : "accepted") + ", host " + (ey ? "rejected" : "accepted") + ")");
  Check(ex->code == ey->code, what + ": error codes differ (b200 '" + ex->message + "', host '" +
                                  ey->message + "')");
}
bool SameBits(const std::vector<float>& a, const std::vector<float>& b) {
  return a.size() == b.size() && (a.empty() || !std::memcmp(a.data(), b.data(), a.size() * 4));
}

// The shapes of the reference's CUDA-backend test (tests/cuda_tests.cpp:73-151).
constexpr std::uint32_t kDim1 = 128, kDim2 = 64;

TableDefinition Table1() {
  return {1, kDim1, 2, 1, {0.01f, 0.9f, 0.999f, 1e-8f, 0.9f, 0.999f}, -0.05f, 0.05f, 7};
}
TableDefinition Table2() {
  OptimizerConfig o{0.05f, 0.8f, 0.99f, 1e-7f, 0.8f, 0.99f, WeightBounds{-0.03f, 0.03f}};
  return {2, kDim2, 2, 1, o, -0.05f, 0.05f, 11};
}

// Resident rows of one backend: its own LocatedRow per key (slots differ).
using Residency = std::map<std::pair<TableId, Key>, LocatedRow>;

RowState RandomState(Rng& r, RowKey row, std::uint32_t dim) {
  RowState s{row, {}, {}, {}, r.Below(6)};
  for (std::uint32_t d = 0; d < dim; ++d) {
    s.weights.push_back(r.Uniform(-0.1f, 0.1f));
    s.first_moment.push_back(r.Uniform(-0.01f, 0.01f));
    s.second_moment.push_back(r.Uniform(0.0f, 1e-4f));
  }
  return s;
}

struct Feature {
  FeatureInput input;
  AccessRoute route;
};

// Seeded features over table 1 keys [0, 40) and table 2 keys [100, 120):
// resident or not, ragged bags (empty ones included).
std::vector<Feature> MakeFeatures(Rng& r) {
  std::vector<Feature> out;
  auto feature = [&](std::uint32_t id, TableId table, Pooling pooling, Key base, Key span,
                     std::uint32_t bags) {
    FeatureInput f{table, id, pooling, {}, {0}, {}};
    for (std::uint32_t b = 0; b < bags; ++b) {
      const auto len = r.Below(6);               // 0 .. 5: empty bags too
      for (std::uint64_t k = 0; k < len; ++k) f.keys.push_back(base + r.Below(span));
      f.offsets.push_back(f.keys.size());
      f.valid_lengths.push_back(len);
    }
    return f;
  };
  out.push_back({feature(10, 1, Pooling::sum, 0, 40, 24), AccessRoute::resident_gpu});
  out.push_back({feature(11, 1, Pooling::mean, 0, 40, 17), AccessRoute::resident_gpu});
  out.push_back({feature(12, 2, Pooling::sequence, 100, 24, 9), AccessRoute::resident_gpu});
  out.push_back({feature(13, 1, Pooling::sum, 200, 12, 11), AccessRoute::transfer_unique});
  out.push_back({feature(14, 2, Pooling::sequence, 200, 6, 5), AccessRoute::transfer_unique});
  return out;
}

// The AgentWork the shard service would send: unique rows of the feature that
// this agent serves, and UINT64_MAX for every other occurrence.
std::vector<AgentWork> MakeWork(std::vector<Feature>& features, const Residency& resident,
                                Rng& r) {
  std::vector<AgentWork> work;
  for (auto& f : features) {
    AgentWork w{f.input.feature, f.route, 0, {}, {}, {}};
    std::map<Key, std::uint64_t> index;
    const bool transfer = f.route == AccessRoute::transfer_unique;
    const auto dim = f.input.table == 1 ? kDim1 : kDim2;
    for (auto key : f.input.keys) {
      auto it = resident.find({f.input.table, key});
      const bool served = transfer ? key % 5 != 0 : it != resident.end();
      if (!served) {
        w.occurrence_to_unique.push_back(UINT64_MAX);
        continue;
      }
      auto [slot, added] = index.try_emplace(key, w.rows.size());
      if (added) {
        if (transfer) {
          w.rows.push_back({{f.input.table, key}, 0, Placement::cpu, 0, 0, 0});
          for (std::uint32_t d = 0; d < dim; ++d) w.transferred_weights.push_back(r.Uniform(-0.2f, 0.2f));
        } else {
          w.rows.push_back(it->second);
        }
      }
      w.occurrence_to_unique.push_back(slot->second);
    }
    work.push_back(std::move(w));
  }
  return work;
}

std::vector<FeatureInput> Layouts(const std::vector<Feature>& features) {
  std::vector<FeatureInput> out;
  for (const auto& f : features) out.push_back(f.input);
  return out;
}

void CompareBlocks(const std::vector<TensorBlock>& a, const std::vector<TensorBlock>& b,
                   const std::string& what) {
  Check(a.size() == b.size(), what + ": block counts differ");
  for (std::size_t i = 0; i < a.size(); ++i) {
    Check(a[i].feature == b[i].feature && a[i].shape == b[i].shape,
          what + ": block layout differs for feature " + std::to_string(b[i].feature));
    Check(SameBits(a[i].values, b[i].values),
          what + ": values differ for feature " + std::to_string(b[i].feature));
  }
}

MigrationPlan Plan(const std::vector<LocatedRow>& rows, Placement destination) {
  return {"plan", 0, rows, destination, 0, 0};
}
std::vector<LocatedRow> Rows(const Residency& r) {
  std::vector<LocatedRow> out;
  for (const auto& [k, loc] : r) out.push_back(loc);
  return out;
}

void CompareStates(B200CacheAgent& a, HostCacheBackend& b, const Residency& ra,
                   const Residency& rb, const std::string& what) {
  auto sa = Take(a.ReadBack(Plan(Rows(ra), Placement::cpu)), what + " b200 readback");
  auto sb = Take(b.ReadBack(Plan(Rows(rb), Placement::cpu)), what + " host readback");
  Check(sa.size() == sb.size(), what + ": row counts differ");
  for (std::size_t i = 0; i < sa.size(); ++i) {
    Check(sa[i].row == sb[i].row && sa[i].row_updates == sb[i].row_updates,
          what + ": row or update count differs at key " + std::to_string(sb[i].row.key));
    Check(SameBits(sa[i].weights, sb[i].weights) && SameBits(sa[i].first_moment, sb[i].first_moment) &&
              SameBits(sa[i].second_moment, sb[i].second_moment),
          what + ": state differs at key " + std::to_string(sb[i].row.key));
  }
}

UpdateContext Context(TableId table, std::uint64_t step, float lr, float b1, float b2) {
  return {{"agent-check", 0, step, Phase::push}, 0, table, step, lr,
          float(std::pow(double(b1), double(step))), float(std::pow(double(b2), double(step)))};
}

RowGradients Gradients(Rng& r, const Residency& resident, TableId table, std::uint32_t dim,
                       float scale) {
  RowGradients g;
  for (const auto& [k, loc] : resident)
    if (k.first == table && r.Below(3) != 0) {
      g.rows.push_back(loc.row);
      for (std::uint32_t d = 0; d < dim; ++d) g.values.push_back(scale * r.Uniform(-1.0f, 1.0f));
    }
  return g;
}

CompactGradients Compact(Rng& r, const Residency& resident, TableId table, std::uint32_t dim) {
  CompactGradients p{{}, dim, {}, {0}, {}, {}};
  const std::uint64_t sources = 7;
  for (std::uint64_t i = 0; i < sources * dim; ++i) p.source_values.push_back(r.Uniform(-0.02f, 0.02f));
  for (const auto& [k, loc] : resident)
    if (k.first == table && r.Below(2)) {
      p.rows.push_back(loc.row);
      const auto refs = 1 + r.Below(4);
      for (std::uint64_t j = 0; j < refs; ++j) {
        p.source_rows.push_back(r.Below(sources));
        p.scales.push_back(r.Below(2) ? 1.0f : 1.0f / float(1 + r.Below(5)));
      }
      p.row_offsets.push_back(p.source_rows.size());
    }
  return p;
}

void BackendContract() {
  Rng r{12345};
  B200CacheOptions o;
  o.rows_per_table = 64;
  o.state_bytes = 1ULL << 28;
  B200CacheAgent a(o);
  HostCacheBackend b(0, 1 << 20);
  for (auto t : {Table1(), Table2()}) {
    Take(a.Define(t), "b200 define");
    Take(b.Define(t), "host define");
    Take(a.Define(t), "b200 define again");
  }
  {
    auto changed = Table1();
    changed.optimizer.learning_rate = 0.02f;
    SameRejection(a.Define(changed), b.Define(changed), "redefinition with another optimizer");
  }

  // ---- Load: table 1 keys [0, 30), table 2 keys [100, 118)
  std::vector<LocatedRow> plan_rows;
  std::vector<RowState> states;
  for (Key k = 0; k < 30; ++k) {
    plan_rows.push_back({{1, k}, 0, Placement::loading, 0, 1 + k % 3, 0});
    states.push_back(RandomState(r, {1, k}, kDim1));
  }
  for (Key k = 100; k < 118; ++k) {
    plan_rows.push_back({{2, k}, 0, Placement::loading, 0, 2, 0});
    states.push_back(RandomState(r, {2, k}, kDim2));
  }
  auto la = Take(a.Load(Plan(plan_rows, Placement::gpu), states), "b200 load");
  auto lb = Take(b.Load(Plan(plan_rows, Placement::gpu), states), "host load");
  Residency ra, rb;
  Check(la.size() == lb.size(), "load: result sizes differ");
  for (std::size_t i = 0; i < la.size(); ++i) {
    Check(la[i].row == lb[i].row && la[i].home == lb[i].home && la[i].placement == lb[i].placement &&
              la[i].agent == lb[i].agent && la[i].generation == lb[i].generation,
          "load: located row differs");
    ra[{la[i].row.table, la[i].row.key}] = la[i];
    rb[{lb[i].row.table, lb[i].row.key}] = lb[i];
  }
  Check(Take(a.FreeSlots(1), "free slots") == 64 - 30, "free slots after load");
  SameRejection(a.Load(Plan({plan_rows[0]}, Placement::gpu), {states[0]}),
                b.Load(Plan({plan_rows[0]}, Placement::gpu), {states[0]}), "load of a resident row");
  {
    auto bad = RandomState(r, {1, 35}, kDim1);
    bad.second_moment[3] = -1.0f;
    LocatedRow loc{{1, 35}, 0, Placement::loading, 0, 1, 0};
    SameRejection(a.Load(Plan({loc}, Placement::gpu), {bad}), b.Load(Plan({loc}, Placement::gpu), {bad}),
                  "load of a negative second moment");
  }
  CompareStates(a, b, ra, rb, "after load");

  // ---- gathers and 9 update steps per table: 7 ApplyHost, 2 ApplyCompact
  for (int round = 0; round < 9; ++round) {
    Rng fr{1000u + round};
    auto features = MakeFeatures(fr);
    Rng wa{77u + round}, wb{77u + round};
    auto work_a = MakeWork(features, ra, wa);
    auto work_b = MakeWork(features, rb, wb);
    CompareBlocks(Take(a.GatherHost(work_a, Layouts(features)), "b200 gather"),
                  Take(b.GatherHost(work_b, Layouts(features)), "host gather"),
                  "gather round " + std::to_string(round));
    for (TableId t : {1u, 2u}) {
      const auto dim = t == 1 ? kDim1 : kDim2;
      const auto def = t == 1 ? Table1() : Table2();
      auto c = Context(t, round + 1, def.optimizer.learning_rate, def.optimizer.beta1, def.optimizer.beta2);
      if (round == 2 || round == 6) {
        Rng ca{900u + round * 7 + t};
        auto p = Compact(ca, ra, t, dim);
        Take(a.ApplyCompact(c, p), "b200 compact apply");
        Take(b.ApplyCompact(c, p), "host compact apply");
      } else {
        Rng ga{500u + round * 7 + t};
        auto g = Gradients(ga, ra, t, dim, t == 1 ? 0.01f : 0.5f);
        Take(a.ApplyHost(c, g), "b200 apply");
        Take(b.ApplyHost(c, g), "host apply");
      }
    }
    CompareStates(a, b, ra, rb, "after update round " + std::to_string(round));
  }

  // ---- rejected calls: same code, state unchanged
  {
    auto c = Context(1, 9, 0.01f, 0.9f, 0.999f);
    Rng g1{31};
    auto g = Gradients(g1, ra, 1, kDim1, 0.01f);
    auto dup = g;
    dup.rows.push_back(g.rows.front());
    dup.values.insert(dup.values.end(), g.values.begin(), g.values.begin() + kDim1);
    SameRejection(a.ApplyHost(c, dup), b.ApplyHost(c, dup), "duplicate gradient row");
    auto overflow = g;
    overflow.values[5] = 1e30f;                 // (1 - beta2) g^2 overflows the second moment
    SameRejection(a.ApplyHost(c, overflow), b.ApplyHost(c, overflow), "optimizer overflow");
    auto nan = g;
    nan.values[0] = std::nanf("");
    SameRejection(a.ApplyHost(c, nan), b.ApplyHost(c, nan), "non-finite gradient");
    auto other = c;
    other.shard = 1;
    SameRejection(a.ApplyHost(other, g), b.ApplyHost(other, g), "gradient for another shard");
    RowGradients absent{{{1, 33}}, std::vector<float>(kDim1, 0.001f)};
    SameRejection(a.ApplyHost(c, absent), b.ApplyHost(c, absent), "gradient of a row not resident");
    auto bad_power = c;
    bad_power.beta1_power = 1.0f;
    SameRejection(a.ApplyHost(bad_power, g), b.ApplyHost(bad_power, g), "invalid update context");
    CompareStates(a, b, ra, rb, "after rejected updates");
    auto stale_a = ra.begin()->second, stale_b = rb.begin()->second;
    ++stale_a.generation;
    ++stale_b.generation;
    SameRejection(a.ReadBack(Plan({stale_a}, Placement::cpu)), b.ReadBack(Plan({stale_b}, Placement::cpu)),
                  "readback of a stale generation");
    Rng fr{4242};
    auto features = MakeFeatures(fr);
    Rng wa{5}, wb{5};
    auto work_a = MakeWork(features, ra, wa);
    auto work_b = MakeWork(features, rb, wb);
    for (auto* w : {&work_a, &work_b})
      for (auto& task : *w)
        if (task.route == AccessRoute::resident_gpu && !task.rows.empty()) ++task.rows[0].generation;
    SameRejection(a.GatherHost(work_a, Layouts(features)), b.GatherHost(work_b, Layouts(features)),
                  "gather of a stale generation");
    // malformed compact packets (src/access/compact_gradients.cpp:10-22)
    Rng pr{57};
    const auto good = Compact(pr, ra, 1, kDim1);
    Check(good.rows.size() >= 2 && good.source_rows.size() >= 2, "compact packet too small");
    auto bad = [&](const char* what, auto mutate) {
      auto p = good;
      mutate(p);
      SameRejection(a.ApplyCompact(c, p), b.ApplyCompact(c, p), std::string("compact: ") + what);
    };
    bad("offsets not from 0", [](CompactGradients& p) { p.row_offsets[0] = 1; });
    bad("decreasing offsets", [](CompactGradients& p) { std::swap(p.row_offsets[1], p.row_offsets[2]); });
    bad("offsets short", [](CompactGradients& p) { p.row_offsets.pop_back(); });
    bad("source out of range", [](CompactGradients& p) { p.source_rows[1] = 7; });
    bad("negative scale", [](CompactGradients& p) { p.scales[0] = -0.5f; });
    bad("non-finite scale", [](CompactGradients& p) { p.scales[1] = std::nanf(""); });
    bad("non-finite value", [](CompactGradients& p) { p.source_values[3] = INFINITY; });
    bad("dimension mismatch", [](CompactGradients& p) { p.dimension = kDim1 / 2; });
    bad("duplicate row", [](CompactGradients& p) {
      p.rows.push_back(p.rows.front());
      p.row_offsets.push_back(p.row_offsets.back());
    });
    CompareStates(a, b, ra, rb, "after rejected compact packets");
    SameRejection(a.CommitEviction(Plan({ra.begin()->second, ra.begin()->second}, Placement::cpu)),
                  b.CommitEviction(Plan({rb.begin()->second, rb.begin()->second}, Placement::cpu)),
                  "duplicate eviction row");
  }

  // ---- evict ten rows, reload them with a new generation, gather again
  {
    std::vector<LocatedRow> ea, eb;
    for (Key k = 5; k < 15; ++k) {
      ea.push_back(ra.at({1, k}));
      eb.push_back(rb.at({1, k}));
    }
    auto sa = Take(a.ReadBack(Plan(ea, Placement::cpu)), "b200 readback before eviction");
    Take(a.CommitEviction(Plan(ea, Placement::cpu)), "b200 eviction");
    Take(b.CommitEviction(Plan(eb, Placement::cpu)), "host eviction");
    Check(Take(a.FreeSlots(1), "free slots") == 64 - 20, "free slots after eviction");
    SameRejection(a.ReadBack(Plan({ea[0]}, Placement::cpu)), b.ReadBack(Plan({eb[0]}, Placement::cpu)),
                  "readback of an evicted row");
    std::vector<LocatedRow> again;
    for (auto loc : ea) {
      loc.generation += 1;
      loc.placement = Placement::loading;
      loc.slot = 0;
      again.push_back(loc);
    }
    auto la2 = Take(a.Load(Plan(again, Placement::gpu), sa), "b200 reload");
    auto lb2 = Take(b.Load(Plan(again, Placement::gpu), sa), "host reload");
    for (Key k = 5; k < 15; ++k) {
      ra.erase({1, k});
      rb.erase({1, k});
    }
    for (std::size_t i = 0; i < la2.size(); ++i) {
      ra[{la2[i].row.table, la2[i].row.key}] = la2[i];
      rb[{lb2[i].row.table, lb2[i].row.key}] = lb2[i];
    }
    CompareStates(a, b, ra, rb, "after reload");
    Rng fr{777};
    auto features = MakeFeatures(fr);
    Rng wa{9}, wb{9};
    auto work_a = MakeWork(features, ra, wa);
    auto work_b = MakeWork(features, rb, wb);
    CompareBlocks(Take(a.GatherHost(work_a, Layouts(features)), "b200 gather"),
                  Take(b.GatherHost(work_b, Layouts(features)), "host gather"), "gather after reload");
  }
  Check(Take(a.GatherHost({}, {}), "empty gather").empty(), "empty gather returns blocks");
}

// ---- the shard service with the agent attached (flow of tests/cache_tests.cpp)
RuntimeOptions ServiceOptions(const char* run) {
  RuntimeOptions o;
  o.run_id = run;
  return o;
}
LookupRequest Request(std::uint64_t seq, bool read_only) {
  return {{"agent-service", 0, seq, Phase::lookup}, 1, read_only,
          {{1, 0, Pooling::mean, {1, 1, 2, 3, 5, 8}, {0, 3, 4, 6}, {3, 1, 2}},
           {1, 1, Pooling::sequence, {3, 2, 1, 8, 13}, {0, 2, 3, 5}, {2, 1, 2}},
           {1, 2, Pooling::sum, {13, 21, 1, 2, 34}, {0, 1, 5}, {1, 4}}}};
}
MoveRowsRequest Move(std::vector<RowKey> rows, Placement destination) {
  return {"agent-service", std::move(rows), 0, destination, {1 << 20, 1 << 20, 8, 0}};
}
std::vector<RowState> ServiceState(CpuParameterService& s, const std::vector<Key>& keys) {
  std::vector<RowKey> rows;
  for (auto k : keys) rows.push_back({1, k});
  auto loc = Take(s.Locations(rows), "locations");
  return Take(s.ReadState(loc), "read state");
}

void ServiceDropIn() {
  const TableDefinition table{1, 4, 1, 1, {0.1f, 0.9f, 0.999f, 1e-8f, 0.9f, 0.999f}, -0.25f, 0.25f, 42};
  B200CacheOptions o;
  o.rows_per_table = 32;
  o.state_bytes = 1ULL << 26;
  auto agent = std::make_shared<B200CacheAgent>(o);
  auto host = std::make_shared<HostCacheBackend>(0, 1 << 20);
  auto with_b200 = std::make_shared<CpuParameterService>(ServiceOptions("agent-service"));
  auto with_host = std::make_shared<CpuParameterService>(ServiceOptions("agent-service"));
  Take(with_b200->AttachAgent(0, agent), "attach b200 agent");
  Take(with_host->AttachAgent(0, host), "attach host backend");
  Take(with_b200->ConfigureAccess(0, AccessRoute::transfer_unique), "access b200");
  Take(with_host->ConfigureAccess(0, AccessRoute::transfer_unique), "access host");
  DistributedClient ca({with_b200}), cb({with_host});
  ca.SetCacheResolver([agent](auto work, auto layouts) {
    return agent->GatherHost(std::move(work), std::move(layouts)).get();
  });
  cb.SetCacheResolver([host](auto work, auto layouts) {
    return host->GatherHost(std::move(work), std::move(layouts)).get();
  });
  Take(ca.CreateTable(table), "create table b200");
  Take(cb.CreateTable(table), "create table host");
  Take(ca.Release(Take(ca.Lookup(Request(0, true)), "warm b200")), "release");
  Take(cb.Release(Take(cb.Lookup(Request(0, true)), "warm host")), "release");
  const std::vector<Key> keys{1, 2, 3, 5, 8, 13, 21, 34};
  const std::vector<RowKey> cached{{1, 1}, {1, 3}, {1, 8}, {1, 21}};
  auto ma = Take(with_b200->MoveRows(Move(cached, Placement::gpu)), "move to b200");
  auto mb = Take(with_host->MoveRows(Move(cached, Placement::gpu)), "move to host backend");
  Check(ma.size() == mb.size() && ma[0].placement == Placement::gpu, "admission publication");
  for (std::uint64_t seq = 1; seq <= 6; ++seq) {
    auto a = Take(ca.Lookup(Request(seq, false)), "lookup b200");
    auto b = Take(cb.Lookup(Request(seq, false)), "lookup host");
    CompareBlocks(a.features(), b.features(), "service lookup " + std::to_string(seq));
    auto gradients = a.features();
    Rng r{seq};
    for (auto& g : gradients)
      for (auto& v : g.values) v = r.Uniform(-1.0f, 1.0f);
    Take(ca.Push(a, gradients), "push b200");
    Take(cb.Push(b, gradients), "push host");
    auto sa = ServiceState(*with_b200, keys), sb = ServiceState(*with_host, keys);
    for (std::size_t i = 0; i < sa.size(); ++i)
      Check(sa[i].row_updates == sb[i].row_updates && SameBits(sa[i].weights, sb[i].weights) &&
                SameBits(sa[i].first_moment, sb[i].first_moment) &&
                SameBits(sa[i].second_moment, sb[i].second_moment),
            "service state differs at key " + std::to_string(keys[i]) + " after round " +
                std::to_string(seq));
  }
  // write the cached rows back to the CPU pool, then one more round
  Take(with_b200->MoveRows(Move(cached, Placement::cpu)), "evict from b200");
  Take(with_host->MoveRows(Move(cached, Placement::cpu)), "evict from host backend");
  Check(Take(agent->FreeSlots(1), "free slots") == 32, "slots not reclaimed after write-back");
  auto a = Take(ca.Lookup(Request(7, true)), "lookup b200");
  auto b = Take(cb.Lookup(Request(7, true)), "lookup host");
  CompareBlocks(a.features(), b.features(), "service lookup after write-back");
  Take(ca.Release(a), "release");
  Take(cb.Release(b), "release");
}

// ---- slot and budget limits, as the reference's CUDA backend enforces them
// (src/cuda/cache_backend.cu:353-371,378-404): a load that does not fit, or
// that would eat the plan's reserve, is refused whole and changes nothing.
void Capacity() {
  B200CacheOptions o;
  o.rows_per_table = 4;
  o.state_bytes = 4 * (std::uint64_t(kDim1) * 12 + 8) + 100;   // one table of 4 slots
  B200CacheAgent a(o);
  Take(a.Define(Table1()), "define");
  auto refused = a.Define(Table2()).get();
  Check(std::holds_alternative<Error>(refused) &&
            std::get<Error>(refused).code == Error::Code::capacity_exceeded,
        "a table over the state budget was accepted");
  Rng r{99};
  auto plan = [&](Key first, Key count, std::uint64_t reserve) {
    std::vector<LocatedRow> rows;
    std::vector<RowState> states;
    for (Key k = first; k < first + count; ++k) {
      rows.push_back({{1, k}, 0, Placement::loading, 0, 1, 0});
      states.push_back(RandomState(r, {1, k}, kDim1));
    }
    auto p = Plan(rows, Placement::gpu);
    p.reserve_slots = reserve;
    return std::make_pair(p, states);
  };
  auto [five, five_states] = plan(0, 5, 0);
  auto over = a.Load(five, five_states).get();
  Check(std::holds_alternative<Error>(over) &&
            std::get<Error>(over).code == Error::Code::capacity_exceeded,
        "a load over the slot count was accepted");
  Check(Take(a.FreeSlots(1), "free slots") == 4, "a refused load kept slots");
  auto [three, three_states] = plan(10, 3, 2);
  auto reserved = a.Load(three, three_states).get();
  Check(std::holds_alternative<Error>(reserved) &&
            std::get<Error>(reserved).code == Error::Code::capacity_exceeded,
        "a load into the reserve was accepted");
  auto [two, two_states] = plan(10, 2, 2);
  auto loaded = Take(a.Load(two, two_states), "load within the reserve");
  Check(Take(a.FreeSlots(1), "free slots") == 2, "slots after a load");
  auto back = Take(a.ReadBack(Plan(loaded, Placement::cpu)), "readback");
  Check(SameBits(back[1].weights, two_states[1].weights) && back[1].row_updates == two_states[1].row_updates,
        "loaded state differs");
}

// ---- calls from several threads: the agent runs them one at a time in
// submission order, so every thread's gathers equal the single-thread result
void Concurrent() {
  Rng r{4711};
  B200CacheOptions o;
  o.rows_per_table = 64;
  auto a = std::make_shared<B200CacheAgent>(o);
  for (auto t : {Table1(), Table2()}) Take(a->Define(t), "define");
  std::vector<LocatedRow> plan_rows;
  std::vector<RowState> states;
  for (Key k = 0; k < 40; ++k) {
    plan_rows.push_back({{1, k}, 0, Placement::loading, 0, 1, 0});
    states.push_back(RandomState(r, {1, k}, kDim1));
  }
  for (Key k = 100; k < 124; ++k) {
    plan_rows.push_back({{2, k}, 0, Placement::loading, 0, 1, 0});
    states.push_back(RandomState(r, {2, k}, kDim2));
  }
  auto loaded = Take(a->Load(Plan(plan_rows, Placement::gpu), states), "load");
  Residency ra;
  for (const auto& loc : loaded) ra[{loc.row.table, loc.row.key}] = loc;
  Rng fr{8}, wr{8};
  auto features = MakeFeatures(fr);
  auto work = MakeWork(features, ra, wr);
  const auto expected = Take(a->GatherHost(work, Layouts(features)), "gather");
  const auto state = Take(a->ReadBack(Plan(Rows(ra), Placement::cpu)), "readback");
  std::vector<std::string> failures(4);
  std::vector<std::thread> threads;
  for (int t = 0; t < 4; ++t)
    threads.emplace_back([&, t] {
      try {
        for (int i = 0; i < 25; ++i) {
          CompareBlocks(Take(a->GatherHost(work, Layouts(features)), "gather"), expected,
                        "concurrent gather");
          if (i % 5 == 0) {
            auto again = Take(a->ReadBack(Plan(Rows(ra), Placement::cpu)), "readback");
            Check(again.size() == state.size() && SameBits(again.back().weights, state.back().weights),
                  "concurrent readback");
          }
        }
      } catch (const std::exception& e) {
        failures[t] = e.what();
      }
    });
  for (auto& th : threads) th.join();
  for (const auto& f : failures) Check(f.empty(), f);
}

// ---- GatherDevice (GPU only): the device results equal the host backend's
// gather, are ready on a consumer stream after WaitOnStream, and outlive the
// agent that made them (tests/cuda_tests.cpp checks the same lifetime).
bool DeviceResults() {
  int devices = 0;
  if (cudaGetDeviceCount(&devices) != cudaSuccess || devices == 0) {
    cudaGetLastError();
    return false;
  }
  Rng r{2468};
  B200CacheOptions o;
  o.rows_per_table = 64;
  auto a = std::make_shared<B200CacheAgent>(o);
  HostCacheBackend b(0, 1 << 20);
  for (auto t : {Table1(), Table2()}) {
    Take(a->Define(t), "b200 define");
    Take(b.Define(t), "host define");
  }
  std::vector<LocatedRow> plan_rows;
  std::vector<RowState> states;
  for (Key k = 0; k < 25; ++k) {
    plan_rows.push_back({{1, k}, 0, Placement::loading, 0, 1, 0});
    states.push_back(RandomState(r, {1, k}, kDim1));
  }
  for (Key k = 100; k < 112; ++k) {
    plan_rows.push_back({{2, k}, 0, Placement::loading, 0, 1, 0});
    states.push_back(RandomState(r, {2, k}, kDim2));
  }
  auto la = Take(a->Load(Plan(plan_rows, Placement::gpu), states), "b200 load");
  auto lb = Take(b.Load(Plan(plan_rows, Placement::gpu), states), "host load");
  Residency ra, rb;
  for (std::size_t i = 0; i < la.size(); ++i) {
    ra[{la[i].row.table, la[i].row.key}] = la[i];
    rb[{lb[i].row.table, lb[i].row.key}] = lb[i];
  }
  Rng fr{31337};
  auto features = MakeFeatures(fr);
  Rng wa{3}, wb{3};
  auto work_a = MakeWork(features, ra, wa);
  auto work_b = MakeWork(features, rb, wb);
  auto device = Take(a->GatherDevice(work_a, Layouts(features)), "b200 device gather");
  auto expected = Take(b.GatherHost(work_b, Layouts(features)), "host gather");
  cudaStream_t consumer = nullptr;
  Check(cudaStreamCreateWithFlags(&consumer, cudaStreamNonBlocking) == cudaSuccess, "stream");
  std::vector<TensorBlock> got;
  for (const auto& d : device) {
    d.tensor->WaitOnStream(consumer);
    Check(d.tensor->elements() == d.shape[0] * d.shape[1], "device tensor size");
    got.push_back({d.feature, d.shape, d.tensor->CopyToHost()});
  }
  Check(cudaStreamSynchronize(consumer) == cudaSuccess, "consumer stream");
  cudaStreamDestroy(consumer);
  CompareBlocks(got, expected, "device gather");
  a.reset();                                     // the results outlive the agent
  got.clear();
  for (const auto& d : device) got.push_back({d.feature, d.shape, d.tensor->CopyToHost()});
  CompareBlocks(got, expected, "device gather after the agent is gone");
  return true;
}

// ---- the agent process's command layer over each backend
template <typename T>
T Both(std::future<Result<T>> a, std::future<Result<T>> b, const std::string& what) {
  auto x = Take(std::move(a), "b200 " + what);
  Take(std::move(b), "host " + what);
  return x;
}

void RuntimeReplay() {
  const TableDefinition table{1, 2, 1, 1, {0.1f, 0.9f, 0.999f, 1e-8f, 0.9f, 0.999f}, 0, 0, 42};
  B200CacheOptions o;
  o.rows_per_table = 2;                         // two slots, as the host budget below holds
  auto agent = std::make_shared<B200CacheAgent>(o);
  auto host = std::make_shared<HostCacheBackend>(0, 2 * (2 * 12 + 8));
  AgentRuntime ra("agent-runtime", agent), rb("agent-runtime", host);
  auto id = [](std::uint64_t n) { return AgentCommand{"agent-runtime", 0, n}; };
  Both(ra.Define(id(0), table), rb.Define(id(0), table), "define");
  Both(ra.Define(id(0), table), rb.Define(id(0), table), "define replay");
  const MigrationPlan load{"load", 0, {{{1, 4}, 0, Placement::loading, 0, 1, 0}}, Placement::gpu, 32, 0};
  const RowState state{{1, 4}, {0.125f, -0.25f}, {0.0f, 0.0f}, {0.0f, 0.0f}, 0};
  auto first_a = Take(ra.Load(id(1), load, {state}), "b200 load");
  auto first_b = Take(rb.Load(id(1), load, {state}), "host load");
  auto again_a = Take(ra.Load(id(1), load, {state}), "b200 load replay");
  Take(rb.Load(id(1), load, {state}), "host load replay");
  Check(first_a[0].slot == again_a[0].slot, "load replay allocated a second slot");
  Check(Take(agent->FreeSlots(1), "free slots") == 1, "load replay consumed a slot");
  UpdateContext c{{"agent-runtime", 0, 0, Phase::push}, 0, 1, 0, 0.1f, 0.9f, 0.999f};
  const RowGradients g{{{1, 4}}, {1.0f, -0.5f}};
  Both(ra.Apply(id(2), c, g), rb.Apply(id(2), c, g), "apply");
  Both(ra.Apply(id(2), c, g), rb.Apply(id(2), c, g), "apply replay");
  SameRejection(ra.Load(id(1), load, {state}), rb.Load(id(1), load, {state}),
                "retired load after an update");
  c.original_request.sequence = 1;
  c.optimizer_sequence = 1;
  c.beta1_power *= 0.9f;
  c.beta2_power *= 0.999f;
  const CompactGradients p{{{1, 4}}, 2, {0.5f, 0.25f, -1.0f, 2.0f}, {0, 3}, {0, 1, 0}, {1.0f, 0.5f, 0.25f}};
  Both(ra.ApplyCompact(id(3), c, p), rb.ApplyCompact(id(3), c, p), "compact apply");
  Both(ra.ApplyCompact(id(3), c, p), rb.ApplyCompact(id(3), c, p), "compact apply replay");
  const MigrationPlan evict_a{"evict", 0, first_a, Placement::cpu, 32, 0};
  const MigrationPlan evict_b{"evict", 0, first_b, Placement::cpu, 32, 0};
  auto sa = Take(ra.ReadBack(id(4), evict_a), "b200 readback");
  auto sb = Take(rb.ReadBack(id(4), evict_b), "host readback");
  auto replay = Take(ra.ReadBack(id(4), evict_a), "b200 readback replay");
  Check(sa[0].row_updates == 2 && sb[0].row_updates == 2, "replayed updates applied twice");
  Check(SameBits(sa[0].weights, sb[0].weights) && SameBits(sa[0].first_moment, sb[0].first_moment) &&
            SameBits(sa[0].second_moment, sb[0].second_moment) && SameBits(replay[0].weights, sa[0].weights),
        "runtime state differs from the host backend");
  Both(ra.CommitEviction(id(5), evict_a), rb.CommitEviction(id(5), evict_b), "eviction");
  Both(ra.CommitEviction(id(5), evict_a), rb.CommitEviction(id(5), evict_b), "eviction replay");
  Check(Take(agent->FreeSlots(1), "free slots") == 2, "eviction did not reclaim the slot");
  Both(ra.Define(id(7), table), rb.Define(id(7), table), "define after a skip");
  SameRejection(ra.Define(id(6), table), rb.Define(id(6), table), "command older than a skip");
}

}  // namespace

// A crash prints the stack (addresses resolve with addr2line against this
// binary and the libraries it loads) instead of ending the run silently.
void OnFatalSignal(int sig) {
  void* frames[64];
  const int n = backtrace(frames, 64);
  const char head[] = "agent_check: fatal signal, stack:\n";
  (void)!write(2, head, sizeof(head) - 1);
  backtrace_symbols_fd(frames, n, 2);
  _exit(128 + sig);
}

void Part(const char* name) { std::cerr << "agent_check: " << name << std::endl; }

int main() {
  std::signal(SIGSEGV, OnFatalSignal);
  std::signal(SIGABRT, OnFatalSignal);
  try {
    Part("backend contract");
    BackendContract();
    Part("service drop-in");
    ServiceDropIn();
    Part("agent runtime");
    RuntimeReplay();
    Part("capacity");
    Capacity();
    Part("concurrent calls");
    Concurrent();
    Part("device results");
    if (!DeviceResults()) std::cout << "agent_check: no GPU, device results not checked\n";
    Part("done");
    std::cout << "agent_check: PASS backend contract, service drop-in and agent runtime, "
                 "bit-exact vs HostCacheBackend\n";
    return 0;
  } catch (const std::exception& e) {
    std::cerr << "agent_check: FAIL " << e.what() << "\n";
    return 1;
  }
}
