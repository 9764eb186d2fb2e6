// B200CacheAgent: the reference's GPU cache-agent interface (eps::GpuCacheAgent,
// include/eps/cache_agent.hpp:18-23, over eps::CacheBackend,
// include/eps/cache_backend.hpp:12-29) implemented on libeps_b200.so's C ABI.
//
// It is a drop-in for eps::CudaCacheBackend (include/eps/cuda_cache_backend.hpp:21-37):
// a shard service attaches it with CpuParameterService::AttachAgent
// (include/eps/runtime.hpp:133), a worker resolves cached rows through its
// GatherHost / GatherDevice, and it compiles against the reference's public
// headers only (eps/cache_agent.hpp, eps/types.hpp).
//
// Model.  Rows that the shard service migrates to the agent (Load) receive a
// slot in a dense device table of `rows_per_table` slots per table, the
// [w | m | v] + u64-counter layout of the B200 store.  The agent keeps the
// residency map (row -> LocatedRow with generation and slot) on the host, as
// the reference's CUDA backend does (src/cuda/cache_backend.cu:190-200), and
// hands the store slot numbers as keys:
//   * GatherHost / GatherDevice: one eps_b200_lookup (shard partial, read
//     only) over all resident-row features; occurrences that the service does
//     not route to this agent (occurrence_to_unique == UINT64_MAX) become the
//     padding key, so pooled bags skip them and sequence positions read 0
//     (src/cuda/cache_backend.cu:81-94).  Rows that the service transfers from
//     its CPU pool (AccessRoute::transfer_unique) arrive as weights in the
//     request and are summed on the host in position order.
//   * ApplyHost / ApplyCompact: eps_b200_apply_rows / eps_b200_apply_compact
//     with the service's UpdateContext (external beta powers, all-or-nothing).
//   * Load / ReadBack: eps_b200_load_state / eps_b200_read_state.
// Every call runs on one ordered worker thread and returns a std::future, as
// the reference backends do (src/common/executor.hpp:11-50); errors come back
// as eps::Error with the C ABI's code - 1 (its codes are Error::Code + 1).
#pragma once

#include <cstdint>
#include <future>
#include <memory>
#include <vector>

#include "eps/cache_agent.hpp"

namespace eps {

// CudaCacheOptions (include/eps/cuda_cache_backend.hpp:5-13) minus the staging
// limits, which the B200 store does not have.
struct B200CacheOptions {
  AgentId agent = 0;
  int device = 0;
  std::uint64_t state_bytes = 64ULL << 20;        // device budget of all slot tables
  std::uint64_t rows_per_table = 4096;            // slots per table, 1 .. 2^31
  std::uint64_t outstanding_output_bytes = 64ULL << 20;  // live GatherDevice outputs
  std::uint32_t queue_limit = 128;                // queued calls before capacity_exceeded
};

class B200CacheAgent final : public GpuCacheAgent {
 public:
  // Creates the device store; throws std::runtime_error if that fails (no GPU,
  // no memory), as CudaCacheBackend's constructor throws on a CUDA error.
  explicit B200CacheAgent(B200CacheOptions options = {});
  ~B200CacheAgent() override;
  B200CacheAgent(const B200CacheAgent&) = delete;
  B200CacheAgent& operator=(const B200CacheAgent&) = delete;

  std::future<Result<Ack>> Define(TableDefinition table) override;
  std::future<Result<std::uint64_t>> FreeSlots(TableId table) override;
  std::future<Result<std::vector<LocatedRow>>> Load(MigrationPlan plan,
                                                    std::vector<RowState> states) override;
  std::future<Result<std::vector<TensorBlock>>> GatherHost(
      std::vector<AgentWork> work, std::vector<FeatureInput> layouts) override;
  std::future<Result<std::vector<DeviceTensorBlock>>> GatherDevice(
      std::vector<AgentWork> work, std::vector<FeatureInput> layouts) override;
  std::future<Result<Ack>> ApplyHost(UpdateContext context, RowGradients gradients) override;
  std::future<Result<Ack>> ApplyCompact(UpdateContext context, CompactGradients gradients) override;
  std::future<Result<std::vector<RowState>>> ReadBack(MigrationPlan plan) override;
  std::future<Result<Ack>> CommitEviction(MigrationPlan plan) override;

 private:
  struct Impl;
  std::unique_ptr<Impl> impl_;
};

}  // namespace eps
