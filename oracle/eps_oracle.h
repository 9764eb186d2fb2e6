/*
 * eps_oracle.h -- CPU restatement of the reference parameter server's hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load this library, and
 * only as the checker.  The product (libeps_b200.so) never links or calls it.
 *
 * Parity is pinned: tests/test_oracle.py checks this restatement against the
 * reference's own known-answer values (tests/core_tests.cpp:68-85,
 * tests/weight_bounds_tests.cpp:35-43) and against golden vectors produced by
 * the reference itself (oracle/_ref, tests/golden/make_golden.py).
 *
 * Citations are path:line inside the reference project.
 *
 * Model: one table is a dense key space [0, rows) held as the reference's row
 * layout [w(D) | m(D) | v(D)] f32 (src/store/shard_store.cpp:21-29) plus a
 * u64 update counter per row.  Rows exist from the start with the reference's
 * initializer (src/store/shard_store.cpp:104-110); the reference creates them
 * lazily on first touch with the same pure function, so the values agree.
 */
#ifndef EPS_ORACLE_H
#define EPS_ORACLE_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
  uint32_t id, dimension;
  float learning_rate, beta1, beta2, epsilon;
  float beta1_power, beta2_power;          /* current powers (types.hpp:76-86 initial) */
  uint64_t optimizer_sequence;
  int32_t has_bounds; float bound_min, bound_max;
  float init_min, init_max; uint64_t init_seed;
  uint64_t rows;
  float* state;        /* rows * 3 * dimension, [w|m|v] per row */
  uint64_t* updates;   /* rows */
} EoTable;

typedef struct {
  uint32_t table, feature, pooling;        /* pooling: 0 sum, 1 mean, 2 sequence */
  const uint64_t* keys; uint64_t key_count;
  const uint64_t* offsets; uint64_t offset_count;
} EoFeature;

/* src/store/shard_store.cpp:13-18 */
uint64_t eo_mix(uint64_t x);
/* Allocates state and initialises every row (src/store/shard_store.cpp:104-111). */
int eo_table_init(EoTable* t);
void eo_table_free(EoTable* t);
/* Initial weight of (key, d) (src/store/shard_store.cpp:104-110). */
float eo_initial_weight(const EoTable* t, uint64_t key, uint32_t d);

/* Client-level lookup over `shards` shards: per-shard unnormalised partials
 * (src/access/batch_access.cpp:53-80), merged in shard order and divided by
 * the bag length for mean (src/client/distributed_client.cpp:173-188,227-232).
 * outputs[f] has rows*dim floats, rows = bags or keys (sequence).
 * Returns 0 or an error code (Error::Code+1). */
int eo_lookup(EoTable* tables, uint32_t table_count, const EoFeature* features,
              uint32_t feature_count, uint32_t shards, float** outputs);

/* Shard-level partial of one shard (src/access/batch_access.cpp:53-80). */
int eo_shard_partial(EoTable* tables, uint32_t table_count, const EoFeature* f,
                     uint32_t shards, uint32_t shard, float* output);

/* Coalesce + segment-sum for one table (src/access/batch_access.cpp:82-125).
 * grads[f] are [rows_f, dim] feature gradients (pooled or sequence).
 * rows_out receives unique keys in first-occurrence order, values_out U*dim.
 * Capacity of rows_out must be >= total keys of the table.  *unique receives U.
 * Returns 0 or 1 (invalid_argument: non-finite input / reduction overflow). */
int eo_reduce_gradients(const EoTable* table, const EoFeature* features,
                        uint32_t feature_count, const float* const* grads,
                        uint64_t* rows_out, float* values_out, uint64_t* unique);

/* src/update/lazy_adam.cpp:7-23 ; returns 0 or 1 */
int eo_validate_lazy_adam(const EoTable* t, const uint64_t* rows, const float* values,
                          uint64_t unique);
/* src/update/lazy_adam.cpp:24-42 (advances powers and the optimizer sequence) */
void eo_apply_lazy_adam(EoTable* t, const uint64_t* rows, const float* values,
                        uint64_t unique);

/* Whole Push of one lookup (src/server/service.cpp:236-331 CPU rows path,
 * src/client/distributed_client.cpp:238-274 validation): all tables are
 * validated before any is written.  Returns 0 or 1; state unchanged on error. */
int eo_push(EoTable* tables, uint32_t table_count, const EoFeature* features,
            uint32_t feature_count, const float* const* grads);

/* ExpandCompactGradients (src/access/compact_gradients.cpp:27-39) */
int eo_expand_compact(uint32_t dim, uint64_t rows, const float* source_values,
                      uint64_t source_count, const uint64_t* row_offsets,
                      const uint64_t* source_rows, const float* scales, float* out);

/* Apply with an externally supplied context (src/cache/host_backend.cpp:119-146):
 * per-element finiteness check, no power advance. Returns 0 or 1. */
int eo_apply_host(EoTable* t, float learning_rate, float beta1_power, float beta2_power,
                  const uint64_t* rows, const float* values, uint64_t unique);

/* Shard routing (src/access/prepared_lookup.cpp:52-66): for one feature, the
 * keys routed to `shard` in (bag, position) order, their original positions
 * and the shard-local offsets.  Returns the routed key count. */
uint64_t eo_partition(const EoFeature* f, uint32_t shards, uint32_t shard,
                      uint64_t* keys_out, uint64_t* positions_out, uint64_t* offsets_out);

/* Padding removal (src/access/prepare_queue.cpp:64-78): returns new key count. */
uint64_t eo_drop_padding(const uint64_t* keys, const uint64_t* offsets, uint64_t bags,
                         uint64_t padding_key, uint64_t* keys_out, uint64_t* offsets_out,
                         uint64_t* positions_out);

/* SynchronousGradientCollector::Reduce (src/training/synchronous_gradients.cpp:91-126)
 * for one table: workers' sorted unique keys + float rows, reduction 0 sum,
 * 1 worker_mean, 2 sample_mean.  Writes the ascending union of keys and the
 * float of the worker-ordered double sums; returns the key count, or
 * UINT64_MAX if a reduced value is not finite. */
uint64_t eo_sync_reduce(uint32_t dim, uint32_t workers, const uint64_t* const* keys,
                        const float* const* values, const uint64_t* rows,
                        const uint64_t* sample_counts, int reduction, uint64_t* keys_out,
                        float* values_out);

#ifdef __cplusplus
}
#endif
#endif
