// fake_b200_abi.cpp -- TEST INFRASTRUCTURE ONLY: a CPU stand-in for the part of
// libeps_b200.so's C ABI (include/eps_b200.h) that the GpuCacheAgent adapter
// (distributed-recommendation-model-training-system_b200/agent/) calls, so that
// the adapter's host logic -- residency map, slots, generations, budgets, the
// occurrence-to-padding translation, error mapping -- can be checked against
// the reference's own HostCacheBackend on a machine without a GPU.  It links
// the oracle (eps_oracle.c) for the optimizer arithmetic and is never loaded by
// the package or the product library.
//
// Covered entry points and semantics (those of the real library):
//   create / destroy / abi_version / synchronize
//   create_table      dense key space, reference initializer
//   lookup            host inputs and outputs, read_only, shard partial; padding
//                     keys skipped (pooled) or read as 0 (sequence); sums start
//                     at 0.0f in position order; keys >= key_space rejected
//   load_state        finite state, v >= 0, all-or-nothing
//   read_state
//   apply_rows        host values, external powers (eo_apply_host), all-or-nothing
//   apply_compact     packet checks of ValidateCompactGradients, ExpandCompactGradients,
//                     then apply_rows
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <set>
#include <string>
#include <vector>

#include "eps_b200.h"
#include "eps_oracle.h"

struct EpsB200Store {
  EpsB200Options options;
  std::map<uint32_t, EoTable> tables;
  std::map<uint32_t, EpsB200Table> definitions;
};

namespace {

int Fail(EpsB200Status* st, int code, const char* message) {
  if (st) {
    st->code = code;
    std::snprintf(st->message, sizeof(st->message), "%s", message);
  }
  return code;
}
int Ok(EpsB200Status* st) {
  if (st) {
    st->code = 0;
    st->message[0] = 0;
  }
  return 0;
}
EoTable* Find(EpsB200Store* s, uint32_t id) {
  auto it = s->tables.find(id);
  return it == s->tables.end() ? nullptr : &it->second;
}

}  // namespace

extern "C" {

uint32_t eps_b200_abi_version(void) { return EPS_B200_ABI; }

int eps_b200_create(const EpsB200Options* options, EpsB200Store** out, EpsB200Status* st) {
  if (!options || !out || !options->shard_count || options->shard_id >= options->shard_count)
    return Fail(st, EPS_B200_INVALID_ARGUMENT, "invalid native options");
  *out = new EpsB200Store{*options, {}, {}};
  return Ok(st);
}

void eps_b200_destroy(EpsB200Store* s) {
  if (!s) return;
  for (auto& [id, t] : s->tables) eo_table_free(&t);
  delete s;
}

int eps_b200_synchronize(EpsB200Store*, EpsB200Status* st) { return Ok(st); }

int eps_b200_create_table(EpsB200Store* s, const EpsB200Table* d, EpsB200Status* st) {
  if (!s || !d || !d->dimension || !d->key_space || d->shard_count != s->options.shard_count)
    return Fail(st, EPS_B200_INVALID_ARGUMENT, "invalid table");
  if (s->tables.count(d->id)) return Ok(st);
  EoTable t{};
  t.id = d->id;
  t.dimension = d->dimension;
  t.learning_rate = d->learning_rate;
  t.beta1 = d->beta1;
  t.beta2 = d->beta2;
  t.epsilon = d->epsilon;
  t.beta1_power = d->initial_beta1_power;
  t.beta2_power = d->initial_beta2_power;
  t.has_bounds = d->has_weight_bounds;
  t.bound_min = d->weight_min;
  t.bound_max = d->weight_max;
  t.init_min = d->initialization_min;
  t.init_max = d->initialization_max;
  t.init_seed = d->initialization_seed;
  t.rows = d->key_space;
  if (eo_table_init(&t)) return Fail(st, EPS_B200_CAPACITY_EXCEEDED, "table allocation failed");
  s->tables.emplace(d->id, t);
  s->definitions.emplace(d->id, *d);
  return Ok(st);
}

int eps_b200_lookup(EpsB200Store* s, const EpsB200Feature* features, uint64_t count,
                    int32_t input_on_device, int32_t read_only, int32_t shard_partial,
                    EpsB200Buffer* outputs, void*, uint64_t*, EpsB200Status* st) {
  if (!s || !features || !outputs || !count || input_on_device || !read_only ||
      !(shard_partial || s->options.shard_count == 1))
    return Fail(st, EPS_B200_INVALID_ARGUMENT, "unsupported lookup form in the fake");
  std::set<uint32_t> ids;
  for (uint64_t i = 0; i < count; ++i) {
    const auto& f = features[i];
    EoTable* t = Find(s, f.table);
    if (!t || !ids.insert(f.feature).second || f.pooling > 2 || f.offset_count < 1 ||
        f.offsets[0] != 0 || f.offsets[f.offset_count - 1] != f.key_count || f.valid_lengths)
      return Fail(st, EPS_B200_INVALID_ARGUMENT, "invalid feature");
    for (uint64_t b = 0; b + 1 < f.offset_count; ++b)
      if (f.offsets[b] > f.offsets[b + 1]) return Fail(st, EPS_B200_INVALID_ARGUMENT, "invalid bag offsets");
    const uint64_t rows = f.pooling == 2 ? f.key_count : f.offset_count - 1;
    const auto& o = outputs[i];
    if (o.feature != f.feature || o.rows != rows || o.columns != t->dimension || o.device >= 0)
      return Fail(st, EPS_B200_INVALID_ARGUMENT, "output buffer layout mismatch");
    for (uint64_t k = 0; k < f.key_count; ++k)
      if (!(f.has_padding && f.keys[k] == f.padding_key) && f.keys[k] >= t->rows)
        return Fail(st, EPS_B200_INVALID_ARGUMENT, "unknown parameter row");
  }
  for (uint64_t i = 0; i < count; ++i) {
    const auto& f = features[i];
    EoTable* t = Find(s, f.table);
    const uint32_t D = t->dimension;
    float* out = static_cast<float*>(outputs[i].data);
    const uint64_t rows = f.pooling == 2 ? f.key_count : f.offset_count - 1;
    for (uint64_t r = 0; r < rows * D; ++r) out[r] = 0.0f;
    for (uint64_t b = 0; b + 1 < f.offset_count; ++b)
      for (uint64_t k = f.offsets[b]; k < f.offsets[b + 1]; ++k) {
        if (f.has_padding && f.keys[k] == f.padding_key) continue;
        const float* w = t->state + f.keys[k] * 3ull * D;
        float* row = out + (f.pooling == 2 ? k : b) * D;
        for (uint32_t d = 0; d < D; ++d) row[d] += w[d];
      }
  }
  return Ok(st);
}

int eps_b200_load_state(EpsB200Store* s, uint32_t table, const uint64_t* keys, uint64_t count,
                        const float* w, const float* m, const float* v, const uint64_t* updates,
                        EpsB200Status* st) {
  EoTable* t = s ? Find(s, table) : nullptr;
  if (!t) return Fail(st, EPS_B200_INVALID_ARGUMENT, "unknown table");
  const uint32_t D = t->dimension;
  for (uint64_t i = 0; i < count; ++i) {
    if (keys[i] >= t->rows) return Fail(st, EPS_B200_INVALID_ARGUMENT, "unknown parameter row");
    for (uint32_t d = 0; d < D; ++d)
      if (!std::isfinite(w[i * D + d]) || !std::isfinite(m[i * D + d]) ||
          !std::isfinite(v[i * D + d]) || v[i * D + d] < 0)
        return Fail(st, EPS_B200_INVALID_ARGUMENT, "invalid row state");
  }
  for (uint64_t i = 0; i < count; ++i) {
    float* row = t->state + keys[i] * 3ull * D;
    std::memcpy(row, w + i * D, D * 4);
    std::memcpy(row + D, m + i * D, D * 4);
    std::memcpy(row + 2 * D, v + i * D, D * 4);
    t->updates[keys[i]] = updates ? updates[i] : 0;
  }
  return Ok(st);
}

int eps_b200_read_state(EpsB200Store* s, uint32_t table, const uint64_t* keys, uint64_t count,
                        float* w, float* m, float* v, uint64_t* updates, EpsB200Status* st) {
  EoTable* t = s ? Find(s, table) : nullptr;
  if (!t) return Fail(st, EPS_B200_INVALID_ARGUMENT, "unknown table");
  const uint32_t D = t->dimension;
  for (uint64_t i = 0; i < count; ++i)
    if (keys[i] >= t->rows) return Fail(st, EPS_B200_INVALID_ARGUMENT, "unknown parameter row");
  for (uint64_t i = 0; i < count; ++i) {
    const float* row = t->state + keys[i] * 3ull * D;
    if (w) std::memcpy(w + i * D, row, D * 4);
    if (m) std::memcpy(m + i * D, row + D, D * 4);
    if (v) std::memcpy(v + i * D, row + 2 * D, D * 4);
    if (updates) updates[i] = t->updates[keys[i]];
  }
  return Ok(st);
}

int eps_b200_apply_rows(EpsB200Store* s, const EpsB200UpdateContext* c, const uint64_t* keys,
                        uint64_t rows, const float* values, int32_t values_on_device, void*,
                        EpsB200Status* st) {
  EoTable* t = s && c ? Find(s, c->table) : nullptr;
  if (!t || values_on_device) return Fail(st, EPS_B200_INVALID_ARGUMENT, "invalid update");
  std::set<uint64_t> unique;
  for (uint64_t i = 0; i < rows; ++i)
    if (keys[i] >= t->rows || !unique.insert(keys[i]).second)
      return Fail(st, EPS_B200_INVALID_ARGUMENT, "invalid gradient rows");
  if (eo_apply_host(t, c->learning_rate, c->beta1_power, c->beta2_power, keys, values, rows))
    return Fail(st, EPS_B200_INVALID_ARGUMENT, "cached optimizer overflow");
  return Ok(st);
}

int eps_b200_apply_compact(EpsB200Store* s, const EpsB200UpdateContext* c,
                           const EpsB200CompactGradients* g, void* stream, EpsB200Status* st) {
  EoTable* t = s && c && g ? Find(s, c->table) : nullptr;
  if (!t || g->dimension != t->dimension || g->row_offsets[0] != 0 ||
      g->row_offsets[g->rows] != g->refs)
    return Fail(st, EPS_B200_INVALID_ARGUMENT, "invalid compact gradient packet");
  for (uint64_t r = 0; r < g->rows; ++r)
    if (g->row_offsets[r] > g->row_offsets[r + 1])
      return Fail(st, EPS_B200_INVALID_ARGUMENT, "invalid compact gradient packet");
  for (uint64_t k = 0; k < g->refs; ++k)
    if (g->source_rows[k] >= g->sources || !std::isfinite(g->scales[k]) || g->scales[k] < 0)
      return Fail(st, EPS_B200_INVALID_ARGUMENT, "invalid compact gradient packet");
  for (uint64_t j = 0; j < g->sources * g->dimension; ++j)
    if (!std::isfinite(g->source_values[j]))
      return Fail(st, EPS_B200_INVALID_ARGUMENT, "non-finite compact gradient value");
  std::vector<float> expanded(g->rows * g->dimension);
  if (eo_expand_compact(g->dimension, g->rows, g->source_values, g->sources, g->row_offsets,
                        g->source_rows, g->scales, expanded.data()))
    return Fail(st, EPS_B200_INVALID_ARGUMENT, "invalid compact gradient packet");
  return eps_b200_apply_rows(s, c, g->keys, g->rows, expanded.data(), 0, stream, st);
}

}  // extern "C"
