// kernels.cuh -- device helpers and kernel launch wrappers (sm_100a).
//
// Every floating-point operation on the parity path uses an explicitly rounded
// intrinsic (__fadd_rn, __fmul_rn, __fdiv_rn, __fsqrt_rn): no FMA contraction
// can occur, so each value rounds exactly as the reference's x86-64 build
// (SSE2, no FMA) rounds it.  The library is also compiled with --fmad=false.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "device_types.h"

namespace eps_b200 {

template <int VEC>
__device__ __forceinline__ void load_vec(const float* p, float (&r)[VEC]) {
  if constexpr (VEC == 4) {
    const float4 x = *reinterpret_cast<const float4*>(p);
    r[0] = x.x; r[1] = x.y; r[2] = x.z; r[3] = x.w;
  } else if constexpr (VEC == 2) {
    const float2 x = *reinterpret_cast<const float2*>(p);
    r[0] = x.x; r[1] = x.y;
  } else {
    r[0] = *p;
  }
}

template <int VEC>
__device__ __forceinline__ void store_vec(float* p, const float (&r)[VEC]) {
  if constexpr (VEC == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(r[0], r[1], r[2], r[3]);
  } else if constexpr (VEC == 2) {
    *reinterpret_cast<float2*>(p) = make_float2(r[0], r[1]);
  } else {
    *p = r[0];
  }
}

// Streaming (evict-first) variants for data touched once per round.
template <int VEC>
__device__ __forceinline__ void load_vec_stream(const float* p, float (&r)[VEC]) {
  if constexpr (VEC == 4) {
    const float4 x = __ldcs(reinterpret_cast<const float4*>(p));
    r[0] = x.x; r[1] = x.y; r[2] = x.z; r[3] = x.w;
  } else if constexpr (VEC == 2) {
    const float2 x = __ldcs(reinterpret_cast<const float2*>(p));
    r[0] = x.x; r[1] = x.y;
  } else {
    r[0] = __ldcs(p);
  }
}

template <int VEC>
__device__ __forceinline__ void store_vec_stream(float* p, const float (&r)[VEC]) {
  if constexpr (VEC == 4) {
    __stcs(reinterpret_cast<float4*>(p), make_float4(r[0], r[1], r[2], r[3]));
  } else if constexpr (VEC == 2) {
    __stcs(reinterpret_cast<float2*>(p), make_float2(r[0], r[1]));
  } else {
    __stcs(p, r[0]);
  }
}

// Clamp with std::clamp semantics (src/common/optimizer_bounds.hpp:14-18).
__device__ __forceinline__ float clamp_weight(float v, int has, float lo, float hi) {
  if (!has) return v;
  return v < lo ? lo : (hi < v ? hi : v);
}

__device__ __forceinline__ unsigned abs_bits(float x) { return __float_as_uint(fabsf(x)); }

// Launch shape of the row kernels: a group of `group` lanes owns one row, each
// lane `vec` consecutive floats, `iters` times.  128-bit accesses (vec = 4) need
// every dimension divisible by 4 and 16-byte aligned buffers; then
// group = D/4 up to 32 lanes.  Otherwise one float per lane with 32 lanes.
struct Shape { int vec, group, iters; };
inline bool choose_shape(unsigned dmax, bool all4, bool align16, Shape* out) {
  if (all4 && align16) {
    if (dmax <= 32) { *out = {4, 8, 1}; return true; }
    if (dmax <= 64) { *out = {4, 16, 1}; return true; }
    if (dmax <= 128) { *out = {4, 32, 1}; return true; }
    if (dmax <= 256) { *out = {4, 32, 2}; return true; }
    if (dmax <= 512) { *out = {4, 32, 4}; return true; }
    return false;
  }
  if (dmax <= 32) { *out = {1, 32, 1}; return true; }
  if (dmax <= 64) { *out = {1, 32, 2}; return true; }
  if (dmax <= 128) { *out = {1, 32, 4}; return true; }
  return false;
}

// ---------------------------------------------------------------- launchers
struct LookupLaunch {
  const LookupFeature* features;   // device array
  unsigned int feature_count;
  unsigned long long bag_total;
  unsigned long long unit_total;   // gather work units over features (LookupFeature::units)
  unsigned long long emit_total;   // emit work units over features (LookupFeature::emit_units)
  unsigned int shard_count, shard_id;
  int client;                      // 1: merge + mean (DistributedClient), 0: shard partial
  unsigned int slot_bits;
  int key64;                       // composite key width
  unsigned long long pad_key;      // composite key of padding occurrences (table rank = table count)
  void* occ_key;                   // KeyT[occurrences]
  unsigned int* occ_src;           // [occurrences]
  float* row_scale;                // [gradient rows]
  unsigned int* error;             // LookupErrorBits
  int vec, group, iters;           // launch shape (see choose_shape)
  // emit only: the coalescing sort's digit histograms (hist[pass][256] of the
  // composite keys, zeroed), counted as the keys are written; null: not counted
  unsigned int* digit_hist;
  unsigned int digit_passes;
};
cudaError_t launch_lookup(const LookupLaunch& p, cudaStream_t stream);
// Occurrence list of a non-read-only lookup (one launch, before the gather).
cudaError_t launch_emit(const LookupLaunch& p, cudaStream_t stream);

// Shard partition of a lookup (multi-GPU round) and the client-side merge.
struct RouteLaunch {
  const LookupFeature* features;   // requester features; `rows` holds the table's key space
  unsigned int feature_count;
  unsigned int shard_count;        // 1 .. 32
  unsigned long long bag_total;    // B
  unsigned long long key_total;    // N
  unsigned long long cells;        // shard_count * B
  unsigned int tiles;              // route_tiles(cells)
  unsigned int* cnt;               // [cells] keys of bag g on shard o at o * B + g
  unsigned int* pk;                // [cells + 1] exclusive prefix of cnt
  unsigned int* pb;                // [cells + 1] exclusive prefix of (cnt > 0)
  unsigned int* tile_k;            // [tiles]
  unsigned int* tile_b;            // [tiles]
  unsigned int* bounds;            // [shard_count][feature_count + 1][2]
  unsigned int* error;             // LookupErrorBits
  unsigned long long* payload;     // scatter output (u64 words, shard-major)
  unsigned int* bag_map;           // [cells] kept bag -> bag index in its feature
  unsigned int* pos_map;           // [N] shard-ordered key -> position in its feature
  const float* partials;           // merge input, shard-major then feature-major
  unsigned long long* part_off;         // [shard_count * feature_count] float offsets
  float* const* outs;              // [feature_count] merge outputs
  const float* const* grads;       // [feature_count] gradient inputs of the gather
  float* send;                     // gather output (same layout as partials)
  unsigned int* nonfinite;         // gather: [0] set to 1 if a gradient value is not finite, [1] max |g| bits
  unsigned long long* row_pre;          // [shard_count * feature_count] row prefix
  unsigned long long* row_total_dev;    // rows of all blocks (device)
  long long* counts_out;                // [shard_count][5F + 1] count rows (route_layout)
  // Distinct rows of one-key groups.  A (shard, feature) group g = o * F + f of a
  // dense table whose kept bags hold one key each on shard o (or a sequence
  // feature) is deduplicated when it has fewer distinct keys than keys: the
  // owner gathers each distinct row once and the merge reads it by rank.
  unsigned long long* dd_keys;          // [dd_mask + 1] (key << 10 | g); ~0 = free
  unsigned int* dd_rank;                // [dd_mask + 1] the key's rank among g's distinct keys
  unsigned long long dd_mask;
  unsigned int* dd_count;               // [cells F-major: o * F + f] distinct keys of group g
  unsigned int* dd_used;                // [o * F + f] distinct keys if g is deduplicated, else 0
  unsigned long long* dd_off;           // [o * F + f] float offsets of the partials received
  unsigned long long* dd_words;         // [o * F + f + 1] prefix of the unique-key words (U + 2)
  unsigned int* dd_idx;                 // [N] shard-ordered key -> rank (deduplicated groups)
  int has_sequence;
  int vec, group, iters;           // launch shape (see choose_shape)
};
unsigned route_tiles(unsigned long long cells);
cudaError_t launch_route_count(const RouteLaunch& p, cudaStream_t stream);
unsigned route_count_launches(const RouteLaunch& p);
cudaError_t launch_route_scatter(const RouteLaunch& p, cudaStream_t stream);
cudaError_t launch_route_merge(const RouteLaunch& p, cudaStream_t stream);
cudaError_t launch_route_gather(const RouteLaunch& p, cudaStream_t stream);

struct SortLaunch {
  void* keys; void* keys_alt;      // KeyT
  unsigned int* vals; unsigned int* vals_alt;
  unsigned long long n;
  unsigned int bits;
  int key64;
  unsigned int* scratch;           // sort_scratch_bytes(n, bits), 256-byte aligned, zeroed
  unsigned int tiles;              // sort_tiles(n)
  unsigned int* error;             // set (kLookupSortFailed) if a look-back wait ran out
  int hist_ready;                  // the scratch's digit histograms are already counted
};
// Stable LSD radix sort; returns in *swapped whether the result is in the alt
// buffers.
cudaError_t launch_sort(const SortLaunch& p, cudaStream_t stream, int* swapped);
unsigned int sort_launch_count(const SortLaunch& p);
unsigned int sort_tiles(unsigned long long n);
size_t sort_scratch_header(unsigned passes);
size_t sort_scratch_bytes(unsigned long long n, unsigned bits);

// Segments (runs of equal keys) of the sorted occurrence keys.
struct SegmentLaunch {
  const void* keys;                // sorted KeyT[n]
  unsigned long long n;
  int key64;
  unsigned int* seg_start;         // [n + 1]: run starts, then n
  unsigned int* seg_total;         // number of runs U
  unsigned int* scratch;           // segment_scratch_bytes(n), zeroed
  unsigned int* error;
};
cudaError_t launch_segments(const SegmentLaunch& p, cudaStream_t stream);
unsigned segment_launch_count(unsigned long long n);
size_t segment_scratch_bytes(unsigned long long n);

// The push's row plan (RowRec / RowPlan), built from the segments at lookup time.
struct PlanLaunch {
  const void* keys;                // sorted KeyT[n]
  const unsigned int* srcs;        // sorted sources
  const unsigned int* seg_start;   // [U + 1]
  const unsigned int* seg_total;   // U (device)
  const LookupFeature* features;   // scale_base per feature
  unsigned int feature_count;
  const float* row_scale;
  unsigned long long n;
  int key64;
  unsigned int slot_bits, table_count;
  unsigned long long long_run;
  RowRec* rows;                    // [n]
  RowPlan* plan;                   // zeroed
  uint2* pieces;
  LongRecord* longs;
};
cudaError_t launch_row_plan(const PlanLaunch& p, cudaStream_t stream);

// Agent-style update with an external optimizer context (push.cu):
// CacheBackend::ApplyHost / ApplyCompact.
struct ApplyLaunch {
  PushTable table;                       // lr_t from the UpdateContext
  const unsigned long long* slots;       // [rows]
  unsigned long long rows;
  const float* values;                   // direct rows [rows][dim], or
  const float* source_values;            // compact: [sources][dim]
  const unsigned long long* row_offsets; // compact: [rows + 1]
  const unsigned long long* source_rows; // compact: [refs]
  const float* scales;                   // compact: [refs]
  int compact;
  unsigned int* reject;                  // RejectBits, zeroed by the caller
  int vec, group, iters;
};
cudaError_t launch_apply_rows(const ApplyLaunch& p, cudaStream_t stream);   // two launches

// Synchronous multi-worker round reduce (sync.cu).
struct SyncWorker {                  // layout of EpsB200WorkerGradients
  const unsigned long long* keys;
  const float* values;
  unsigned long long rows;
  unsigned long long sample_count;
};
struct SyncLaunch {
  const SyncWorker* workers;
  unsigned int worker_count;
  const unsigned long long* row_base;   // [workers + 1] prefix of rows
  const double* scale;                  // [workers]
  unsigned long long total_rows;
  unsigned int dim;
  unsigned long long key_space;
  unsigned int shard_count, shard_id;
  unsigned long long* keys;             // pack output: concatenated keys
  unsigned int* rows;                   // pack output: global row index
  const unsigned long long* sorted_keys;
  const unsigned int* sorted_rows;
  const unsigned int* seg_start;
  const unsigned int* seg_total;
  unsigned long long* keys_out;
  float* values_out;
  unsigned int* error;                  // 1 unsorted, 2 not owned, 4 non-finite, 16 overflow
                                        // (8: a sort wait ran out)
};
cudaError_t launch_sync_pack(const SyncLaunch& p, cudaStream_t stream);
cudaError_t launch_sync_accumulate(const SyncLaunch& p, cudaStream_t stream);

struct PushLaunch {
  const PushTable* tables;         // device, per table rank
  unsigned int table_count;
  const PushFeature* features;     // device, per feature index
  unsigned int feature_count;
  const float* row_scale;
  const void* keys;                // sorted composite keys
  const unsigned int* srcs;        // sorted sources
  unsigned long long n;
  unsigned int slot_bits;
  int key64;
  unsigned long long grad_values;  // total gradient values over features
  unsigned long long grad_max_values;  // largest feature's gradient values
  int grad_vec4;                   // every gradient buffer 16-byte aligned, size % 4 == 0
  const unsigned long long* grad_prefix;  // device: value prefix per feature
  const unsigned int* seg_start;   // [U + 1] run starts of the sorted keys
  const unsigned int* seg_total;   // U (device)
  const RowRec* rows;              // the row plan: rows[u] for u < U
  const RowPlan* plan;
  uint2* pieces;                   // [max_pieces] (start, count) of long-row pieces
  unsigned int max_pieces;
  float* part;                     // [max_pieces][dim_max] piece sums
  LongRecord* records;
  unsigned int dim_max;
  PushControl* control;
  const unsigned int* lookup_error;
  // optional device words of a sharded round: [0] nonzero rejects (non-finite
  // input), [1] an upper bound of every |g| (float bits) that replaces the scan
  const unsigned int* external_reject;
  unsigned long long long_run;     // segments longer than this are reduced in pieces
  int vec, group, iters;           // launch shape (see choose_shape)
  int ring_dim;                    // 32 / 64 / 128: rows updated through the async ring
                                   // (every table has this dimension, 16-byte aligned
                                   // gradients); 0: register path only
};
// Push = prescan (+ device-side mode decision), apply (stage A: piece sums and
// single-occurrence rows; stage B: long rows and rows with a piece sum, then the
// beta powers / sequence iff accepted; stage C: the apply pass of a CHECKED
// push); finalize launches a kernel only for a push without occurrences.
cudaError_t launch_push_prescan(const PushLaunch& p, cudaStream_t stream);
// part 0: piece sums (uniform shape only), 1: row updates, 2: long rows and
// the checked apply
cudaError_t launch_push_apply(const PushLaunch& p, cudaStream_t stream, int part);
unsigned launch_push_apply_count(const PushLaunch& p, int part);
unsigned launch_push_finalize_count(const PushLaunch& p);
cudaError_t launch_push_finalize(const PushLaunch& p, cudaStream_t stream);

struct InitLaunch {
  float* state; unsigned long long* updates;
  unsigned long long rows; unsigned int dim;
  unsigned int shard_count, shard_id;
  unsigned int table_id; unsigned long long seed;
  float init_min, init_max;
  int has_bounds; float bound_min, bound_max;
};
cudaError_t launch_init(const InitLaunch& p, cudaStream_t stream);

// Hashed tables (store.cu).  Resolves the keys of every hashed feature of a
// lookup: each occurrence's slot into LookupFeature::slots, creating rows for
// unseen keys (two launches: claim / insert, then entry -> slot).  `entries`
// is scratch of one u32 per occurrence of the lookup.
struct ResolveLaunch {
  const LookupFeature* features;   // device
  unsigned int feature_count;
  unsigned long long key_total;    // occurrences of the lookup (occ_base prefix)
  unsigned int shard_count, shard_id;
  unsigned int* entries;           // [key_total]
  unsigned int* error;             // LookupErrorBits
};
cudaError_t launch_resolve(const ResolveLaunch& p, cudaStream_t stream);   // two launches
// Keys of one hashed table -> slots (creating rows), for ReadState / Load.
// `index` is a host copy of the table's HashIndex (its pointers are device memory).
cudaError_t launch_resolve_keys(const HashIndex* index, const unsigned long long* keys,
                                unsigned long long n, unsigned int* entries, unsigned int* slots,
                                unsigned int* error, cudaStream_t stream);

// Row state gather/scatter for ReadState / Load (src/cuda/cache_backend.cu
// ReadStateKernel / ScatterState contract, slots from keys).
cudaError_t launch_read_rows(const float* state, const unsigned long long* updates,
                             unsigned int dim, unsigned long long rows,
                             unsigned int shard_count, const unsigned long long* keys,
                             unsigned long long n, float* packed, unsigned long long* upd_out,
                             unsigned int* error, cudaStream_t stream);
cudaError_t launch_write_rows(float* state, unsigned long long* updates, unsigned int dim,
                              unsigned long long rows, unsigned int shard_count,
                              const unsigned long long* keys, unsigned long long n,
                              const float* packed, const unsigned long long* upd_in,
                              DeviceTable* dtable, cudaStream_t stream);
// The same by resolved slots (hashed tables): slots[r] instead of keys[r] / shards.
cudaError_t launch_read_slots(const float* state, const unsigned long long* updates,
                              unsigned int dim, const unsigned int* slots, unsigned long long n,
                              float* packed, unsigned long long* upd_out, unsigned int* error,
                              cudaStream_t stream);
cudaError_t launch_write_slots(float* state, unsigned long long* updates, unsigned int dim,
                               const unsigned int* slots, unsigned long long n, const float* packed,
                               const unsigned long long* upd_in, DeviceTable* dtable,
                               cudaStream_t stream);

// Allocation-free lookup (eps_b200_lookup_noalloc): feature descriptors live in
// a fixed file-scope device array in noalloc.cu instead of an allocated block.
constexpr unsigned int kNoAllocFeatures = 256;
constexpr int kNoAllocMaxDevices = 64;
// Device address of this GPU's descriptor array; the first call on a GPU looks it
// up (with that GPU current) and caches it.
cudaError_t noalloc_feature_table(int device, LookupFeature** out);
// Writes `count` descriptors into that array on `stream` (by kernel parameters,
// so `desc` may be released once this returns); *launches receives the kernels
// launched.
cudaError_t noalloc_store_features(const LookupFeature* desc, unsigned count, cudaStream_t stream,
                                   unsigned* launches);

}  // namespace eps_b200
