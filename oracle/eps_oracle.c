/*
 * eps_oracle.c -- CPU restatement of the reference hot path (TEST INFRASTRUCTURE).
 *
 * Only the test suite, __graft_entry__.smoke() and bench.py's CPU baseline leg
 * load this file's library, as the checker.  The product never links it.
 *
 * Floating point follows the reference as built by its CMake (x86-64 SSE2, no
 * FMA contraction): this file is compiled with -ffp-contract=off and no -march,
 * so every float expression rounds exactly as the reference's does.
 */
#include "eps_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

enum { EO_OK = 0, EO_INVALID = 1, EO_CAPACITY = 5 };

/* src/store/shard_store.cpp:13-18 (splitmix64 finaliser) */
uint64_t eo_mix(uint64_t x) {
  x += 0x9e3779b97f4a7c15ULL;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ULL;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebULL;
  return x ^ (x >> 31);
}

/* std::clamp semantics of BoundWeight (src/common/optimizer_bounds.hpp:14-18) */
static float bound(const EoTable* t, float v) {
  if (!t->has_bounds) return v;
  return v < t->bound_min ? t->bound_min : (t->bound_max < v ? t->bound_max : v);
}

/* src/store/shard_store.cpp:104-110 */
float eo_initial_weight(const EoTable* t, uint64_t key, uint32_t d) {
  const uint64_t bits = eo_mix(key ^ eo_mix(t->init_seed) ^ eo_mix((uint64_t)t->id) ^
                               eo_mix((uint64_t)d));
  const double u = (double)(bits >> 11) * 0x1.0p-53;
  const float w = (float)((1 - u) * (double)t->init_min + u * (double)t->init_max);
  return bound(t, w);
}

int eo_table_init(EoTable* t) {
  const uint64_t dim = t->dimension;
  t->state = (float*)malloc(t->rows * dim * 3 * sizeof(float));
  t->updates = (uint64_t*)calloc(t->rows, sizeof(uint64_t));
  if (!t->state || !t->updates) { eo_table_free(t); return EO_CAPACITY; }
  for (uint64_t key = 0; key < t->rows; ++key) {
    float* row = t->state + key * dim * 3;
    for (uint32_t d = 0; d < dim; ++d) {
      row[d] = eo_initial_weight(t, key, d);
      row[dim + d] = 0.0f;
      row[2 * dim + d] = 0.0f;
    }
  }
  return EO_OK;
}

void eo_table_free(EoTable* t) {
  free(t->state); free(t->updates);
  t->state = NULL; t->updates = NULL;
}

static EoTable* find_table(EoTable* tables, uint32_t n, uint32_t id) {
  for (uint32_t i = 0; i < n; ++i) if (tables[i].id == id) return &tables[i];
  return NULL;
}

/* ValidateFeature (src/access/batch_access.cpp:10-23) at client level, where the
 * original lengths are the offset differences (prepared_lookup.cpp:24-25). */
static int valid_feature(const EoTable* t, const EoFeature* f) {
  if (!t || f->pooling > 2 || f->offset_count == 0) return 0;
  if (f->offsets[0] != 0 || f->offsets[f->offset_count - 1] != f->key_count) return 0;
  for (uint64_t b = 1; b < f->offset_count; ++b)
    if (f->offsets[b] < f->offsets[b - 1]) return 0;
  for (uint64_t i = 0; i < f->key_count; ++i)
    if (f->keys[i] >= t->rows) return 0;
  return 1;
}

static uint64_t output_rows(const EoFeature* f) {
  return f->pooling == 2 ? f->key_count : f->offset_count - 1;
}

/* src/access/batch_access.cpp:67-78: unnormalised sum (or per-position row) of
 * this shard's keys, added in position order into a zeroed contribution. */
int eo_shard_partial(EoTable* tables, uint32_t table_count, const EoFeature* f,
                     uint32_t shards, uint32_t shard, float* output) {
  EoTable* t = find_table(tables, table_count, f->table);
  if (!valid_feature(t, f)) return EO_INVALID;
  const uint32_t dim = t->dimension;
  memset(output, 0, output_rows(f) * dim * sizeof(float));
  for (uint64_t b = 0; b + 1 < f->offset_count; ++b) {
    for (uint64_t i = f->offsets[b]; i < f->offsets[b + 1]; ++i) {
      if (f->keys[i] % shards != shard) continue;
      const float* w = t->state + f->keys[i] * dim * 3;
      float* dest = output + (f->pooling == 2 ? i : b) * dim;
      for (uint32_t d = 0; d < dim; ++d) dest[d] += w[d];
    }
  }
  return EO_OK;
}

int eo_lookup(EoTable* tables, uint32_t table_count, const EoFeature* features,
              uint32_t feature_count, uint32_t shards, float** outputs) {
  if (shards == 0) return EO_INVALID;
  for (uint32_t fi = 0; fi < feature_count; ++fi) {
    const EoFeature* f = &features[fi];
    EoTable* t = find_table(tables, table_count, f->table);
    if (!valid_feature(t, f)) return EO_INVALID;
    const uint32_t dim = t->dimension;
    const uint64_t n = output_rows(f) * dim;
    float* part = (float*)malloc((n ? n : 1) * sizeof(float));
    if (!part) return EO_CAPACITY;
    memset(outputs[fi], 0, n * sizeof(float));
    /* src/client/distributed_client.cpp:173-188: merge shard partials in shard order */
    for (uint32_t s = 0; s < shards; ++s) {
      eo_shard_partial(tables, table_count, f, shards, s, part);
      if (f->pooling == 2) {
        /* sequence rows are copied to their positions; the routed position of
         * every key is unique, so copy == add-to-zero except for -0.0 */
        for (uint64_t i = 0; i < f->key_count; ++i)
          if (f->keys[i] % shards == s)
            memcpy(outputs[fi] + i * dim, part + i * dim, dim * sizeof(float));
      } else {
        for (uint64_t i = 0; i < n; ++i) outputs[fi][i] += part[i];
      }
    }
    free(part);
    /* src/client/distributed_client.cpp:227-232 */
    if (f->pooling == 1) {
      for (uint64_t b = 0; b + 1 < f->offset_count; ++b) {
        const uint64_t len = f->offsets[b + 1] - f->offsets[b];
        if (len)
          for (uint32_t d = 0; d < dim; ++d) outputs[fi][b * dim + d] /= (float)len;
      }
    }
  }
  return EO_OK;
}

/* --- open-addressing key -> index map (first-occurrence order) ------------- */
typedef struct { uint64_t* keys; uint64_t* vals; uint64_t cap; } Map;
static int map_init(Map* m, uint64_t n) {
  m->cap = 16; while (m->cap < 2 * n + 16) m->cap <<= 1;
  m->keys = (uint64_t*)malloc(m->cap * sizeof(uint64_t));
  m->vals = (uint64_t*)malloc(m->cap * sizeof(uint64_t));
  if (!m->keys || !m->vals) return 0;
  memset(m->vals, 0xff, m->cap * sizeof(uint64_t));
  return 1;
}
static void map_free(Map* m) { free(m->keys); free(m->vals); }
/* returns index; *inserted set when new */
static uint64_t map_get(Map* m, uint64_t key, uint64_t next, int* inserted) {
  uint64_t h = eo_mix(key) & (m->cap - 1);
  for (;;) {
    if (m->vals[h] == UINT64_MAX) { m->keys[h] = key; m->vals[h] = next; *inserted = 1; return next; }
    if (m->keys[h] == key) { *inserted = 0; return m->vals[h]; }
    h = (h + 1) & (m->cap - 1);
  }
}

/* src/access/batch_access.cpp:82-125 for the features of one table. */
int eo_reduce_gradients(const EoTable* table, const EoFeature* features,
                        uint32_t feature_count, const float* const* grads,
                        uint64_t* rows_out, float* values_out, uint64_t* unique) {
  const uint32_t dim = table->dimension;
  uint64_t total = 0;
  for (uint32_t fi = 0; fi < feature_count; ++fi) {
    if (features[fi].table != table->id) continue;
    total += features[fi].key_count;
    /* batch_access.cpp:97: every gradient value must be finite */
    const uint64_t n = output_rows(&features[fi]) * dim;
    for (uint64_t i = 0; i < n; ++i) if (!isfinite(grads[fi][i])) return EO_INVALID;
  }
  Map map;
  if (!map_init(&map, total)) { map_free(&map); return EO_CAPACITY; }
  uint64_t u = 0;
  for (uint32_t fi = 0; fi < feature_count; ++fi) {
    const EoFeature* f = &features[fi];
    if (f->table != table->id) continue;
    for (uint64_t b = 0; b + 1 < f->offset_count; ++b) {
      const uint64_t len = f->offsets[b + 1] - f->offsets[b];
      /* batch_access.cpp:107-108: scale = 1.0f / valid_length for mean */
      const float scale = (f->pooling == 1 && len) ? 1.0f / (float)len : 1.0f;
      for (uint64_t i = f->offsets[b]; i < f->offsets[b + 1]; ++i) {
        int inserted;
        const uint64_t at = map_get(&map, f->keys[i], u, &inserted);
        if (inserted) {
          rows_out[u] = f->keys[i];
          memset(values_out + u * dim, 0, dim * sizeof(float));
          ++u;
        }
        const float* src = grads[fi] + (f->pooling == 2 ? i : b) * dim;
        float* dest = values_out + at * dim;
        for (uint32_t d = 0; d < dim; ++d) dest[d] += src[d] * scale;
      }
    }
  }
  map_free(&map);
  *unique = u;
  /* batch_access.cpp:122-123 */
  for (uint64_t i = 0; i < u * dim; ++i) if (!isfinite(values_out[i])) return EO_INVALID;
  return EO_OK;
}

static float bias_corrected(float lr, float b1p, float b2p) {
  /* src/update/lazy_adam.cpp:11,27: evaluated in float, left to right */
  return lr * sqrtf(1 - b2p) / (1 - b1p);
}

/* src/update/lazy_adam.cpp:7-23 */
int eo_validate_lazy_adam(const EoTable* t, const uint64_t* rows, const float* values,
                          uint64_t unique) {
  const uint32_t dim = t->dimension;
  const float lr = bias_corrected(t->learning_rate, t->beta1_power, t->beta2_power);
  if (!isfinite(lr)) return EO_INVALID;
  for (uint64_t i = 0; i < unique; ++i) {
    const float* row = t->state + rows[i] * dim * 3;
    for (uint32_t d = 0; d < dim; ++d) {
      const float g = values[i * dim + d];
      const float m = t->beta1 * row[dim + d] + (1 - t->beta1) * g;
      const float v = t->beta2 * row[2 * dim + d] + (1 - t->beta2) * g * g;
      const float w = row[d] - lr * m / (sqrtf(v) + t->epsilon);
      if (!isfinite(m) || !isfinite(v) || !isfinite(w)) return EO_INVALID;
    }
  }
  return EO_OK;
}

/* src/update/lazy_adam.cpp:24-42 */
void eo_apply_lazy_adam(EoTable* t, const uint64_t* rows, const float* values,
                        uint64_t unique) {
  const uint32_t dim = t->dimension;
  const float lr = bias_corrected(t->learning_rate, t->beta1_power, t->beta2_power);
  for (uint64_t i = 0; i < unique; ++i) {
    float* row = t->state + rows[i] * dim * 3;
    for (uint32_t d = 0; d < dim; ++d) {
      const float g = values[i * dim + d];
      row[dim + d] = t->beta1 * row[dim + d] + (1 - t->beta1) * g;
      row[2 * dim + d] = t->beta2 * row[2 * dim + d] + (1 - t->beta2) * g * g;
      row[d] -= lr * row[dim + d] / (sqrtf(row[2 * dim + d]) + t->epsilon);
      row[d] = bound(t, row[d]);
    }
    ++t->updates[rows[i]];
  }
  ++t->optimizer_sequence;
  t->beta1_power *= t->beta1;
  t->beta2_power *= t->beta2;
}

int eo_push(EoTable* tables, uint32_t table_count, const EoFeature* features,
            uint32_t feature_count, const float* const* grads) {
  /* src/client/distributed_client.cpp:246-250: all gradients finite first */
  for (uint32_t fi = 0; fi < feature_count; ++fi) {
    EoTable* t = find_table(tables, table_count, features[fi].table);
    if (!valid_feature(t, &features[fi])) return EO_INVALID;
    const uint64_t n = output_rows(&features[fi]) * t->dimension;
    for (uint64_t i = 0; i < n; ++i) if (!isfinite(grads[fi][i])) return EO_INVALID;
  }
  /* tables that appear in the Push, in ascending id (std::map order,
   * src/server/service.cpp:252-267) */
  uint32_t* ids = (uint32_t*)malloc((feature_count + 1) * sizeof(uint32_t));
  uint32_t nids = 0;
  for (uint32_t fi = 0; fi < feature_count; ++fi) {
    uint32_t id = features[fi].table, seen = 0;
    for (uint32_t k = 0; k < nids; ++k) seen |= ids[k] == id;
    if (!seen) ids[nids++] = id;
  }
  for (uint32_t a = 0; a < nids; ++a)
    for (uint32_t b = a + 1; b < nids; ++b)
      if (ids[b] < ids[a]) { uint32_t x = ids[a]; ids[a] = ids[b]; ids[b] = x; }
  uint64_t** rows = (uint64_t**)calloc(nids, sizeof(uint64_t*));
  float** values = (float**)calloc(nids, sizeof(float*));
  uint64_t* unique = (uint64_t*)calloc(nids, sizeof(uint64_t));
  int rc = EO_OK;
  for (uint32_t k = 0; k < nids && rc == EO_OK; ++k) {
    EoTable* t = find_table(tables, table_count, ids[k]);
    uint64_t total = 0;
    for (uint32_t fi = 0; fi < feature_count; ++fi)
      if (features[fi].table == ids[k]) total += features[fi].key_count;
    rows[k] = (uint64_t*)malloc((total + 1) * sizeof(uint64_t));
    values[k] = (float*)malloc((total + 1) * t->dimension * sizeof(float));
    if (!rows[k] || !values[k]) { rc = EO_CAPACITY; break; }
    rc = eo_reduce_gradients(t, features, feature_count, grads, rows[k], values[k], &unique[k]);
  }
  /* src/server/service.cpp:268: validate every table before applying any */
  for (uint32_t k = 0; k < nids && rc == EO_OK; ++k)
    rc = eo_validate_lazy_adam(find_table(tables, table_count, ids[k]), rows[k], values[k], unique[k]);
  if (rc == EO_OK)
    for (uint32_t k = 0; k < nids; ++k)
      eo_apply_lazy_adam(find_table(tables, table_count, ids[k]), rows[k], values[k], unique[k]);
  for (uint32_t k = 0; k < nids; ++k) { free(rows[k]); free(values[k]); }
  free(rows); free(values); free(unique); free(ids);
  return rc;
}

/* src/access/compact_gradients.cpp:27-39 */
int eo_expand_compact(uint32_t dim, uint64_t rows, const float* source_values,
                      uint64_t source_count, const uint64_t* row_offsets,
                      const uint64_t* source_rows, const float* scales, float* out) {
  for (uint64_t r = 0; r < rows; ++r)
    for (uint64_t ref = row_offsets[r]; ref < row_offsets[r + 1]; ++ref)
      if (source_rows[ref] >= source_count) return EO_INVALID;
  for (uint64_t r = 0; r < rows; ++r) {
    for (uint32_t d = 0; d < dim; ++d) {
      float sum = 0;
      for (uint64_t ref = row_offsets[r]; ref < row_offsets[r + 1]; ++ref)
        sum += source_values[source_rows[ref] * dim + d] * scales[ref];
      if (!isfinite(sum)) return EO_INVALID;
      out[r * dim + d] = sum;
    }
  }
  return EO_OK;
}

/* src/cache/host_backend.cpp:192-218 */
int eo_apply_host(EoTable* t, float learning_rate, float beta1_power, float beta2_power,
                  const uint64_t* rows, const float* values, uint64_t unique) {
  const uint32_t dim = t->dimension;
  const float lr = bias_corrected(learning_rate, beta1_power, beta2_power);
  float* staged = (float*)malloc((unique ? unique : 1) * dim * 3 * sizeof(float));
  if (!staged) return EO_CAPACITY;
  for (uint64_t i = 0; i < unique; ++i) {
    const float* row = t->state + rows[i] * dim * 3;
    float* out = staged + i * dim * 3;
    for (uint32_t d = 0; d < dim; ++d) {
      const float g = values[i * dim + d];
      const float m = t->beta1 * row[dim + d] + (1 - t->beta1) * g;
      const float v = t->beta2 * row[2 * dim + d] + (1 - t->beta2) * g * g;
      const float w = row[d] - lr * m / (sqrtf(v) + t->epsilon);
      if (!isfinite(g) || !isfinite(w) || !isfinite(m) || !isfinite(v)) { free(staged); return EO_INVALID; }
      out[d] = bound(t, w); out[dim + d] = m; out[2 * dim + d] = v;
    }
  }
  for (uint64_t i = 0; i < unique; ++i) {
    memcpy(t->state + rows[i] * dim * 3, staged + i * dim * 3, dim * 3 * sizeof(float));
    ++t->updates[rows[i]];
  }
  free(staged);
  return EO_OK;
}

/* src/access/prepared_lookup.cpp:52-66 */
uint64_t eo_partition(const EoFeature* f, uint32_t shards, uint32_t shard,
                      uint64_t* keys_out, uint64_t* positions_out, uint64_t* offsets_out) {
  uint64_t n = 0;
  offsets_out[0] = 0;
  for (uint64_t b = 0; b + 1 < f->offset_count; ++b) {
    for (uint64_t i = f->offsets[b]; i < f->offsets[b + 1]; ++i)
      if (f->keys[i] % shards == shard) { keys_out[n] = f->keys[i]; positions_out[n] = i; ++n; }
    offsets_out[b + 1] = n;
  }
  return n;
}

/* src/access/prepare_queue.cpp:64-78 */
uint64_t eo_drop_padding(const uint64_t* keys, const uint64_t* offsets, uint64_t bags,
                         uint64_t padding_key, uint64_t* keys_out, uint64_t* offsets_out,
                         uint64_t* positions_out) {
  uint64_t n = 0;
  offsets_out[0] = 0;
  for (uint64_t b = 0; b < bags; ++b) {
    for (uint64_t i = offsets[b]; i < offsets[b + 1]; ++i)
      if (keys[i] != padding_key) { keys_out[n] = keys[i]; positions_out[n] = i; ++n; }
    offsets_out[b + 1] = n;
  }
  return n;
}

static int eo_cmp_u64(const void* a, const void* b) {
  const uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
  return x < y ? -1 : x > y;
}

/* src/training/synchronous_gradients.cpp:91-126: denominator (:92-97), per-worker
 * scale (:104), accumulation in worker order in double (:105-110), ascending keys
 * of the std::map and the float conversion with its overflow check (:113-121). */
uint64_t eo_sync_reduce(uint32_t dim, uint32_t workers, const uint64_t* const* keys,
                        const float* const* values, const uint64_t* rows,
                        const uint64_t* sample_counts, int reduction, uint64_t* keys_out,
                        float* values_out) {
  double denominator = 1;
  if (reduction == 1) denominator = workers;
  else if (reduction == 2) {
    denominator = 0;
    for (uint32_t w = 0; w < workers; ++w) denominator += (double)sample_counts[w];
  }
  uint64_t total = 0;
  for (uint32_t w = 0; w < workers; ++w) total += rows[w];
  uint64_t* all = (uint64_t*)malloc((total ? total : 1) * sizeof(uint64_t));
  uint64_t n = 0;
  for (uint32_t w = 0; w < workers; ++w)
    for (uint64_t r = 0; r < rows[w]; ++r) all[n++] = keys[w][r];
  qsort(all, n, sizeof(uint64_t), eo_cmp_u64);
  uint64_t u = 0;
  for (uint64_t i = 0; i < n; ++i)
    if (i == 0 || all[i] != all[i - 1]) all[u++] = all[i];
  double* acc = (double*)malloc((dim ? dim : 1) * sizeof(double));
  int overflow = 0;
  for (uint64_t k = 0; k < u; ++k) {
    for (uint32_t d = 0; d < dim; ++d) acc[d] = 0.0;
    for (uint32_t w = 0; w < workers; ++w) {
      const double scale = (reduction == 2 ? (double)sample_counts[w] : 1.) / denominator;
      uint64_t lo = 0, hi = rows[w];
      while (lo < hi) { const uint64_t mid = (lo + hi) / 2; if (keys[w][mid] < all[k]) lo = mid + 1; else hi = mid; }
      if (lo < rows[w] && keys[w][lo] == all[k])
        for (uint32_t d = 0; d < dim; ++d) acc[d] += (double)values[w][lo * dim + d] * scale;
    }
    keys_out[k] = all[k];
    for (uint32_t d = 0; d < dim; ++d) {
      const float f = (float)acc[d];
      if (!isfinite(f)) overflow = 1;
      values_out[k * dim + d] = f;
    }
  }
  free(acc);
  free(all);
  return overflow ? UINT64_MAX : u;
}
