// store.cu -- device row store: initialisation, row read-back and row load.
//
// Initialisation applies the reference initializer to every slot up front
// (src/store/shard_store.cpp:104-111):
//   bits = Mix(key ^ Mix(seed) ^ Mix(table) ^ Mix(d));  u = (bits >> 11) * 2^-53
//   w = clamp((float)((1-u)*min + u*max)),  m = v = 0,  updates = 0
// The reference creates a row lazily on its first lookup with the same pure
// function of (seed, table, key, d), so the values are identical; the double
// arithmetic uses explicitly rounded intrinsics (no FMA), as on x86-64.
#include "kernels.cuh"

namespace eps_b200 {
namespace {

// splitmix64 finaliser (src/store/shard_store.cpp:13-18)
__device__ __forceinline__ unsigned long long mix64(unsigned long long x) {
  x += 0x9e3779b97f4a7c15ULL;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ULL;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebULL;
  return x ^ (x >> 31);
}

__global__ void __launch_bounds__(256) init_kernel(InitLaunch p) {
  extern __shared__ unsigned long long s_mixd[];   // Mix(d) for d < D
  const unsigned D = p.dim;
  for (unsigned d = threadIdx.x; d < D; d += blockDim.x) s_mixd[d] = mix64((unsigned long long)d);
  __syncthreads();
  const unsigned long long base = mix64(p.seed) ^ mix64((unsigned long long)p.table_id);
  const unsigned long long total = p.rows * D;
  const double lo = (double)p.init_min, hi = (double)p.init_max;
  for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < total;
       i += (unsigned long long)gridDim.x * blockDim.x) {
    const unsigned long long slot = i / D;
    const unsigned d = (unsigned)(i - slot * D);
    const unsigned long long key = slot * p.shard_count + p.shard_id;
    const unsigned long long bits = mix64(key ^ base ^ s_mixd[d]);
    const double u = __dmul_rn((double)(bits >> 11), 0x1.0p-53);
    const double x = __dadd_rn(__dmul_rn(__dsub_rn(1.0, u), lo), __dmul_rn(u, hi));
    const float w = clamp_weight(__double2float_rn(x), p.has_bounds, p.bound_min, p.bound_max);
    float* row = p.state + slot * 3ull * D;
    row[d] = w;
    row[D + d] = 0.0f;
    row[2 * D + d] = 0.0f;
  }
  for (unsigned long long r = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; r < p.rows;
       r += (unsigned long long)gridDim.x * blockDim.x)
    p.updates[r] = 0ull;
}

__global__ void read_rows_kernel(const float* state, const unsigned long long* updates,
                                 unsigned D, unsigned long long rows, unsigned shards,
                                 const unsigned long long* keys, unsigned long long n,
                                 float* packed, unsigned long long* upd_out, unsigned* error) {
  const unsigned long long total = n * 3ull * D;
  for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < total;
       i += (unsigned long long)gridDim.x * blockDim.x) {
    const unsigned long long r = i / (3ull * D);
    const unsigned long long c = i - r * 3ull * D;
    const unsigned long long slot = keys[r] / shards;
    if (slot < rows) {
      packed[i] = state[slot * 3ull * D + c];
      if (c == 0) upd_out[r] = updates[slot];
    } else {
      packed[i] = 0.0f;
      if (c == 0) { upd_out[r] = 0; atomicOr(error, kLookupBadKey); }
    }
  }
}

__global__ void write_rows_kernel(float* state, unsigned long long* updates, unsigned D,
                                  unsigned long long rows, unsigned shards,
                                  const unsigned long long* keys, unsigned long long n,
                                  const float* packed, const unsigned long long* upd_in,
                                  DeviceTable* dtable) {
  const unsigned long long total = n * 3ull * D;
  unsigned mx = 0;
  for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < total;
       i += (unsigned long long)gridDim.x * blockDim.x) {
    const unsigned long long r = i / (3ull * D);
    const unsigned long long c = i - r * 3ull * D;
    const unsigned long long slot = keys[r] / shards;
    if (slot >= rows) continue;   // the host validated keys before the launch
    const float x = packed[i];
    state[slot * 3ull * D + c] = x;
    mx = max(mx, abs_bits(x));
    if (c == 0) updates[slot] = upd_in[r];
  }
  mx = __reduce_max_sync(0xffffffffu, mx);
  if ((threadIdx.x & 31) == 0 && mx) atomicMax(&dtable->state_absmax_bits, mx);
}

// ------------------------------------------------------------ hashed tables
// The initial value of one row (the function init_kernel applies), written by
// the thread that created the row.
__device__ void init_row(const HashIndex& H, unsigned long long slot, unsigned long long key) {
  const unsigned D = H.dim;
  const unsigned long long base = mix64(H.seed) ^ mix64((unsigned long long)H.table_id);
  const double lo = (double)H.init_min, hi = (double)H.init_max;
  float* row = H.state + slot * 3ull * D;
  for (unsigned d = 0; d < D; ++d) {
    const unsigned long long bits = mix64(key ^ base ^ mix64((unsigned long long)d));
    const double u = __dmul_rn((double)(bits >> 11), 0x1.0p-53);
    const double x = __dadd_rn(__dmul_rn(__dsub_rn(1.0, u), lo), __dmul_rn(u, hi));
    row[d] = clamp_weight(__double2float_rn(x), H.has_bounds, H.bound_min, H.bound_max);
    row[D + d] = 0.0f;
    row[2 * D + d] = 0.0f;
  }
  H.updates[slot] = 0ull;
}

// The index entry of `key`, claimed if absent (linear probing; the probe count
// is bounded by the index size); the claiming thread takes the next slot and
// creates the row.  Returns kNoSlot when the index is full.
__device__ unsigned claim_entry(const HashIndex& H, unsigned long long key, unsigned* err) {
  unsigned long long h;
  bool inserted = false;
  if (key == kEmptyKey) {                 // the one key that cannot mark a free entry
    h = H.mask + 1;
    inserted = atomicCAS(H.top, 0u, 1u) == 0u;
  } else {
    h = mix64(key) & H.mask;
    unsigned long long probe = 0;
    for (; probe <= H.mask; ++probe) {
      const unsigned long long old = atomicCAS(H.keys + h, kEmptyKey, key);
      if (old == kEmptyKey) { inserted = true; break; }
      if (old == key) break;
      h = (h + 1) & H.mask;
    }
    if (probe > H.mask) { *err |= kLookupCapacity; return kNoSlot; }
  }
  if (inserted) {
    const unsigned long long slot = atomicAdd(H.used, 1ull);
    if (slot < H.capacity) {
      init_row(H, slot, key);
      H.slot_keys[slot] = key;
      H.slots[h] = (unsigned)slot;
    } else {
      *err |= kLookupCapacity;            // the entry keeps kNoSlot: the table is full
    }
  }
  return (unsigned)h;
}

// Pass 1: claim every occurrence's entry (padding and other shards' keys marked).
__global__ void __launch_bounds__(256) resolve_claim(ResolveLaunch p) {
  __shared__ unsigned long long s_occ[kMaxFeatures + 1];
  const unsigned fc = p.feature_count;
  for (unsigned i = threadIdx.x; i < fc; i += blockDim.x) s_occ[i] = p.features[i].occ_base;
  if (threadIdx.x == 0) s_occ[fc] = p.key_total;
  __syncthreads();
  unsigned err = 0;
  for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x;
       i < p.key_total; i += (unsigned long long)gridDim.x * blockDim.x) {
    unsigned lo = 0, hi = fc;
    while (hi - lo > 1) { const unsigned mid = (lo + hi) >> 1; if (s_occ[mid] <= i) lo = mid; else hi = mid; }
    const LookupFeature& F = p.features[lo];
    if (!F.hash) continue;
    const unsigned long long key = F.keys[i - s_occ[lo]];
    unsigned e;
    if (F.has_padding && key == F.padding_key) e = kPadSlot;
    else if (p.shard_count > 1 && key % p.shard_count != p.shard_id) { e = kNoSlot; err |= kLookupBadKey; }
    else e = claim_entry(*F.hash, key, &err);
    p.entries[i] = e;
  }
  err = __reduce_or_sync(0xffffffffu, err);
  if (err && (threadIdx.x & 31) == 0) atomicOr(p.error, err);
}

// Pass 2 (after every claim): entry -> slot, in place.
__global__ void __launch_bounds__(256) resolve_slots(ResolveLaunch p) {
  __shared__ unsigned long long s_occ[kMaxFeatures + 1];
  const unsigned fc = p.feature_count;
  for (unsigned i = threadIdx.x; i < fc; i += blockDim.x) s_occ[i] = p.features[i].occ_base;
  if (threadIdx.x == 0) s_occ[fc] = p.key_total;
  __syncthreads();
  unsigned err = 0;
  for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x;
       i < p.key_total; i += (unsigned long long)gridDim.x * blockDim.x) {
    unsigned lo = 0, hi = fc;
    while (hi - lo > 1) { const unsigned mid = (lo + hi) >> 1; if (s_occ[mid] <= i) lo = mid; else hi = mid; }
    const LookupFeature& F = p.features[lo];
    if (!F.hash) continue;
    const unsigned e = p.entries[i];
    unsigned slot = e;
    if (e != kPadSlot && e != kNoSlot) {
      slot = F.hash->slots[e];
      if (slot == kNoSlot) err |= kLookupCapacity;
    }
    p.entries[i] = slot;
  }
  err = __reduce_or_sync(0xffffffffu, err);
  if (err && (threadIdx.x & 31) == 0) atomicOr(p.error, err);
}

__global__ void __launch_bounds__(256) resolve_keys_claim(HashIndex H, const unsigned long long* keys,
                                                          unsigned long long n, unsigned* entries,
                                                          unsigned* error) {
  unsigned err = 0;
  for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < n;
       i += (unsigned long long)gridDim.x * blockDim.x)
    entries[i] = claim_entry(H, keys[i], &err);
  err = __reduce_or_sync(0xffffffffu, err);
  if (err && (threadIdx.x & 31) == 0) atomicOr(error, err);
}

__global__ void __launch_bounds__(256) resolve_keys_slots(const unsigned* index_slots,
                                                          const unsigned* entries,
                                                          unsigned long long n, unsigned* slots,
                                                          unsigned* error) {
  unsigned err = 0;
  for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < n;
       i += (unsigned long long)gridDim.x * blockDim.x) {
    const unsigned e = entries[i];
    const unsigned slot = e == kNoSlot ? kNoSlot : index_slots[e];
    if (slot == kNoSlot) err |= kLookupCapacity;
    slots[i] = slot;
  }
  err = __reduce_or_sync(0xffffffffu, err);
  if (err && (threadIdx.x & 31) == 0) atomicOr(error, err);
}

__global__ void read_slots_kernel(const float* state, const unsigned long long* updates, unsigned D,
                                  const unsigned* slots, unsigned long long n, float* packed,
                                  unsigned long long* upd_out) {
  const unsigned long long total = n * 3ull * D;
  for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < total;
       i += (unsigned long long)gridDim.x * blockDim.x) {
    const unsigned long long r = i / (3ull * D);
    const unsigned long long c = i - r * 3ull * D;
    const unsigned slot = slots[r];
    if (slot != kNoSlot) {
      packed[i] = state[slot * 3ull * D + c];
      if (c == 0) upd_out[r] = updates[slot];
    } else {
      packed[i] = 0.0f;
      if (c == 0) upd_out[r] = 0;
    }
  }
}

__global__ void write_slots_kernel(float* state, unsigned long long* updates, unsigned D,
                                   const unsigned* slots, unsigned long long n, const float* packed,
                                   const unsigned long long* upd_in, DeviceTable* dtable) {
  const unsigned long long total = n * 3ull * D;
  unsigned mx = 0;
  for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < total;
       i += (unsigned long long)gridDim.x * blockDim.x) {
    const unsigned long long r = i / (3ull * D);
    const unsigned long long c = i - r * 3ull * D;
    const unsigned slot = slots[r];
    if (slot == kNoSlot) continue;        // reported by the resolve
    const float x = packed[i];
    state[slot * 3ull * D + c] = x;
    mx = max(mx, abs_bits(x));
    if (c == 0) updates[slot] = upd_in[r];
  }
  mx = __reduce_max_sync(0xffffffffu, mx);
  if ((threadIdx.x & 31) == 0 && mx) atomicMax(&dtable->state_absmax_bits, mx);
}

unsigned grid_for(unsigned long long work) {
  const unsigned long long g = (work + 255) / 256;
  return (unsigned)(g < 148ull * 32 ? (g ? g : 1) : 148ull * 32);
}
}  // namespace

cudaError_t launch_init(const InitLaunch& p, cudaStream_t stream) {
  if (p.rows == 0) return cudaSuccess;
  init_kernel<<<grid_for(p.rows * p.dim), 256, p.dim * sizeof(unsigned long long), stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_read_rows(const float* state, const unsigned long long* updates,
                             unsigned int dim, unsigned long long rows,
                             unsigned int shard_count, const unsigned long long* keys,
                             unsigned long long n, float* packed, unsigned long long* upd_out,
                             unsigned int* error, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  read_rows_kernel<<<grid_for(n * 3ull * dim), 256, 0, stream>>>(
      state, updates, dim, rows, shard_count, keys, n, packed, upd_out, error);
  return cudaGetLastError();
}

cudaError_t launch_write_rows(float* state, unsigned long long* updates, unsigned int dim,
                              unsigned long long rows, unsigned int shard_count,
                              const unsigned long long* keys, unsigned long long n,
                              const float* packed, const unsigned long long* upd_in,
                              DeviceTable* dtable, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  write_rows_kernel<<<grid_for(n * 3ull * dim), 256, 0, stream>>>(
      state, updates, dim, rows, shard_count, keys, n, packed, upd_in, dtable);
  return cudaGetLastError();
}

}  // namespace eps_b200

namespace eps_b200 {

cudaError_t launch_resolve(const ResolveLaunch& p, cudaStream_t stream) {
  if (p.key_total == 0) return cudaSuccess;
  resolve_claim<<<grid_for(p.key_total), 256, 0, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  resolve_slots<<<grid_for(p.key_total), 256, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_resolve_keys(const HashIndex* index, const unsigned long long* keys,
                                unsigned long long n, unsigned int* entries, unsigned int* slots,
                                unsigned int* error, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  resolve_keys_claim<<<grid_for(n), 256, 0, stream>>>(*index, keys, n, entries, error);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  resolve_keys_slots<<<grid_for(n), 256, 0, stream>>>(index->slots, entries, n, slots, error);
  return cudaGetLastError();
}

cudaError_t launch_read_slots(const float* state, const unsigned long long* updates,
                              unsigned int dim, const unsigned int* slots, unsigned long long n,
                              float* packed, unsigned long long* upd_out, unsigned int* error,
                              cudaStream_t stream) {
  (void)error;
  if (n == 0) return cudaSuccess;
  read_slots_kernel<<<grid_for(n * 3ull * dim), 256, 0, stream>>>(state, updates, dim, slots, n,
                                                                   packed, upd_out);
  return cudaGetLastError();
}

cudaError_t launch_write_slots(float* state, unsigned long long* updates, unsigned int dim,
                               const unsigned int* slots, unsigned long long n, const float* packed,
                               const unsigned long long* upd_in, DeviceTable* dtable,
                               cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  write_slots_kernel<<<grid_for(n * 3ull * dim), 256, 0, stream>>>(state, updates, dim, slots, n,
                                                                    packed, upd_in, dtable);
  return cudaGetLastError();
}

}  // namespace eps_b200
