// route.cu -- the shard-partition step of a multi-GPU round and the client-side
// merge, on the device.
//
// Reference semantics followed:
//   * PrepareLookupInputs, src/access/prepared_lookup.cpp:47-83: every key goes to
//     shard key % n in (bag, position) order; every shard receives every bag of
//     every feature (offsets per shard) and the GLOBAL valid lengths, which must
//     equal the offset differences (:24-25).
//   * DistributedClient merge, src/client/distributed_client.cpp:173-188: the
//     zeroed output receives the shard partials in shard order; sequence rows are
//     scattered by position; mean bags are divided once by (float)valid_length
//     after the merge (:227-232).
//   * Push split, src/client/distributed_client.cpp:252-265: each shard receives
//     the full bag gradients of pooled features and the position rows of its
//     keys for sequence features.
//
// Adapter padding (PrepareAdapterInput, src/access/prepare_queue.cpp:58-85, which
// runs before PrepareLookupInputs): keys equal to a feature's padding key go to
// no shard; a padded feature's valid length is the bag's kept (non-padding)
// key count, and its sequence positions holding padding read zeros.
//
// Bags without a key on a shard contribute an all-zero partial (0 + nothing) and
// no gradient term, so they are dropped from that shard's part: a merge that
// skips them adds +0.0f fewer times, which leaves every value unchanged (a
// partial is never -0.0f: 0 + w rounds an exact cancellation to +0.0f).
//
// Index spaces (n shards, B = bags of all features, N = keys of all features):
//   cell (o, g) = o * B + g, g = feature bag base + bag: count of bag g's keys on
//   shard o.  pk / pb = exclusive prefix over cells of the key counts / of
//   (count > 0), so shard o's keys are [pk[o*B], pk[(o+1)*B]) in (feature, bag,
//   position) order and its kept bags [pb[o*B], pb[(o+1)*B]).
//   Payload sent to shard o (u64): [keys | offsets (kept + 1 per feature) |
//   valid lengths (kept)], feature-major inside each region.
#include "kernels.cuh"

namespace eps_b200 {
namespace {

constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;

__device__ __forceinline__ unsigned feature_of(const unsigned long long* s_base, unsigned fc,
                                               unsigned long long g) {
  unsigned lo = 0, hi = fc;
  while (hi - lo > 1) { const unsigned mid = (lo + hi) >> 1; if (s_base[mid] <= g) lo = mid; else hi = mid; }
  return lo;
}

// ---------------------------------------------------------- distinct rows
// A group (shard o, feature f) whose kept bags hold exactly one key each on
// shard o -- or a sequence feature's keys on o -- has a partial per kept bag
// that is just 0 + the key's row.  When such a group (dense table) has fewer
// distinct keys than keys, the owner returns each distinct row once and the
// merge reads a bag's row by its key's rank: the bytes change, the values and
// their order of addition do not.  The ranks come from a hash set of
// (key << 10 | group) built while the batch is prepared.
constexpr unsigned long long kDedupFree = ~0ull;

__device__ __forceinline__ unsigned long long dd_mix(unsigned long long x) {
  // MurmurHash3's 64-bit finaliser
  x ^= x >> 33;
  x *= 0xff51afd7ed558ccdull;
  x ^= x >> 33;
  x *= 0xc4ceb9fe1a85ec53ull;
  x ^= x >> 33;
  return x;
}

// keys and kept bags of group (o, f), from route_bounds
__device__ __forceinline__ void group_counts(const RouteLaunch& p, unsigned o, unsigned f,
                                             unsigned& keys, unsigned& kept) {
  const unsigned* a = p.bounds + 2 * (o * (p.feature_count + 1) + f);
  keys = a[2] - a[0];
  kept = a[3] - a[1];
}

__device__ __forceinline__ bool dedup_eligible(const RouteLaunch& p, const LookupFeature* F,
                                               unsigned o, unsigned f) {
  unsigned keys, kept;
  group_counts(p, o, f, keys, kept);
  return p.dd_mask && F->rows <= (1ull << 53) && keys > 0 && (F->pooling == 2 || keys == kept);
}

__device__ __forceinline__ void dd_claim(const RouteLaunch& p, unsigned long long comp, unsigned g) {
  unsigned long long h = dd_mix(comp) & p.dd_mask;
  for (unsigned long long probe = 0; probe <= p.dd_mask; ++probe) {
    const unsigned long long old = atomicCAS(p.dd_keys + h, kDedupFree, comp);
    if (old == kDedupFree) { p.dd_rank[h] = atomicAdd(p.dd_count + g, 1u); return; }
    if (old == comp) return;
    h = (h + 1) & p.dd_mask;
  }
}

__device__ __forceinline__ unsigned dd_find(const RouteLaunch& p, unsigned long long comp) {
  unsigned long long h = dd_mix(comp) & p.dd_mask;
  for (unsigned long long probe = 0; probe <= p.dd_mask; ++probe) {
    const unsigned long long k = p.dd_keys[h];
    if (k == comp) return p.dd_rank[h];
    if (k == kDedupFree) return 0u;      // not reached: every key was claimed
    h = (h + 1) & p.dd_mask;
  }
  return 0u;
}

// ------------------------------------------------------------------ count
// One warp per bag: validates the bag and counts its keys per shard (lane o
// holds shard o's count; n <= 32).
__global__ void __launch_bounds__(256) route_count(RouteLaunch p) {
  __shared__ unsigned long long s_base[kMaxFeatures + 1];
  const unsigned fc = p.feature_count;
  for (unsigned i = threadIdx.x; i < fc; i += blockDim.x) s_base[i] = p.features[i].bag_base;
  if (threadIdx.x == 0) s_base[fc] = p.bag_total;
  __syncthreads();
  const unsigned lane = threadIdx.x & 31;
  const unsigned long long warp = (blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x) >> 5;
  const unsigned long long nwarps = (gridDim.x * (unsigned long long)blockDim.x) >> 5;
  const unsigned n = p.shard_count;
  unsigned err = 0;
  for (unsigned long long g = warp; g < p.bag_total; g += nwarps) {
    const LookupFeature* F = p.features + feature_of(s_base, fc, g);
    const unsigned long long b = g - F->bag_base;
    const unsigned long long key_count = F->key_count;
    unsigned long long o2 = 0;
    if (lane < 2) o2 = F->offsets[b + lane];
    unsigned long long s = __shfl_sync(~0u, o2, 0), e = __shfl_sync(~0u, o2, 1);
    if (b == 0 && s != 0) err |= kLookupBadOffsets;
    if (b + 1 == F->bag_count && e != key_count) err |= kLookupBadOffsets;
    if (s > e || e > key_count) { err |= kLookupBadOffsets; s = e = 0; }
    if (F->lengths && F->lengths[b] != e - s) err |= kLookupShortLength;
    const unsigned long long key_space = F->rows;
    const bool has_pad = F->has_padding != 0;
    const unsigned long long pad_key = F->padding_key;
    unsigned count = 0;
    for (unsigned long long c0 = s; c0 < e; c0 += 32) {
      const unsigned long long i = c0 + lane;
      unsigned owner = ~0u;
      if (i < e) {
        const unsigned long long key = F->keys[i];
        if (has_pad && key == pad_key) owner = ~0u;          // dropped, goes nowhere
        else if (key < key_space) owner = (unsigned)(key % n);
        else err |= kLookupBadKey;
      }
      for (unsigned o = 0; o < n; ++o) {
        const unsigned m = __ballot_sync(~0u, owner == o);
        if (lane == o) count += __popc(m);
      }
    }
    if (lane < n) p.cnt[lane * p.bag_total + g] = count;
  }
  err = __reduce_or_sync(~0u, err);
  if (err && lane == 0) atomicOr(p.error, err);
}

// One warp per bag (after route_bounds): every key of an eligible group joins
// the group's distinct-key set; the key that inserts an entry takes the next rank.
__global__ void __launch_bounds__(256) route_dedup_claim(RouteLaunch p) {
  __shared__ unsigned long long s_base[kMaxFeatures + 1];
  const unsigned fc = p.feature_count;
  for (unsigned i = threadIdx.x; i < fc; i += blockDim.x) s_base[i] = p.features[i].bag_base;
  if (threadIdx.x == 0) s_base[fc] = p.bag_total;
  __syncthreads();
  const unsigned lane = threadIdx.x & 31;
  const unsigned long long warp = (blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x) >> 5;
  const unsigned long long nwarps = (gridDim.x * (unsigned long long)blockDim.x) >> 5;
  const unsigned n = p.shard_count;
  for (unsigned long long g = warp; g < p.bag_total; g += nwarps) {
    const unsigned f = feature_of(s_base, fc, g);
    const LookupFeature* F = p.features + f;
    const unsigned long long b = g - F->bag_base;
    unsigned long long o2 = 0;
    if (lane < 2) o2 = F->offsets[b + lane];
    const unsigned long long s = __shfl_sync(~0u, o2, 0), e = __shfl_sync(~0u, o2, 1);
    if (s > e || e > F->key_count) continue;      // reported by route_count
    const bool has_pad = F->has_padding != 0;
    for (unsigned long long c0 = s; c0 < e; c0 += 32) {
      const unsigned long long i = c0 + lane;
      if (i >= e) continue;
      const unsigned long long key = F->keys[i];
      if ((has_pad && key == F->padding_key) || key >= F->rows) continue;
      const unsigned o = (unsigned)(key % n);
      if (dedup_eligible(p, F, o, f)) dd_claim(p, (key << 10) | (o * fc + f), o * fc + f);
    }
  }
}

// --------------------------------------------------------- three-phase scan
__device__ __forceinline__ void load_cells(const RouteLaunch& p, unsigned long long tile, unsigned (&k)[kScanItems],
                                           unsigned (&b)[kScanItems]) {
  const unsigned long long base = tile * kScanTile + threadIdx.x * (unsigned long long)kScanItems;
#pragma unroll
  for (int j = 0; j < kScanItems; ++j) {
    const unsigned long long idx = base + j;
    const unsigned c = idx < p.cells ? p.cnt[idx] : 0u;
    k[j] = c;
    b[j] = c ? 1u : 0u;
  }
}

// Block-wide exclusive scan of one value per thread; returns the block total.
__device__ __forceinline__ unsigned block_exclusive(unsigned x, unsigned* s_warp, unsigned& total) {
  const unsigned lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  unsigned inc = x;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const unsigned y = __shfl_up_sync(~0u, inc, d);
    if (lane >= d) inc += y;
  }
  if (lane == 31) s_warp[w] = inc;
  __syncthreads();
  if (w == 0) {
    unsigned v = lane < blockDim.x / 32 ? s_warp[lane] : 0u;
    unsigned vi = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const unsigned y = __shfl_up_sync(~0u, vi, d);
      if (lane >= d) vi += y;
    }
    if (lane < blockDim.x / 32) s_warp[lane] = vi - v;
    if (lane == 31) s_warp[32] = vi;
  }
  __syncthreads();
  const unsigned r = s_warp[w] + inc - x;
  total = s_warp[32];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kScanThreads) route_tile_sums(RouteLaunch p) {
  __shared__ unsigned s_warp[33];
  unsigned k[kScanItems], b[kScanItems];
  load_cells(p, blockIdx.x, k, b);
  unsigned sk = 0, sb = 0;
#pragma unroll
  for (int j = 0; j < kScanItems; ++j) { sk += k[j]; sb += b[j]; }
  unsigned tk, tb;
  block_exclusive(sk, s_warp, tk);
  block_exclusive(sb, s_warp, tb);
  if (threadIdx.x == 0) { p.tile_k[blockIdx.x] = tk; p.tile_b[blockIdx.x] = tb; }
}

// One block: exclusive prefixes of the tile sums (in place) and the totals.
__global__ void __launch_bounds__(1024) route_tile_scan(RouteLaunch p) {
  __shared__ unsigned s_warp[33];
  unsigned carry_k = 0, carry_b = 0;
  for (unsigned base = 0; base < p.tiles; base += blockDim.x) {
    const unsigned t = base + threadIdx.x;
    const unsigned xk = t < p.tiles ? p.tile_k[t] : 0u, xb = t < p.tiles ? p.tile_b[t] : 0u;
    unsigned tk, tb;
    const unsigned ek = block_exclusive(xk, s_warp, tk);
    const unsigned eb = block_exclusive(xb, s_warp, tb);
    if (t < p.tiles) { p.tile_k[t] = carry_k + ek; p.tile_b[t] = carry_b + eb; }
    carry_k += tk;
    carry_b += tb;
  }
  if (threadIdx.x == 0) { p.pk[p.cells] = carry_k; p.pb[p.cells] = carry_b; }
}

__global__ void __launch_bounds__(kScanThreads) route_tile_apply(RouteLaunch p) {
  __shared__ unsigned s_warp[33];
  unsigned k[kScanItems], b[kScanItems];
  load_cells(p, blockIdx.x, k, b);
  unsigned sk = 0, sb = 0;
#pragma unroll
  for (int j = 0; j < kScanItems; ++j) { sk += k[j]; sb += b[j]; }
  unsigned tk, tb;
  unsigned ek = block_exclusive(sk, s_warp, tk) + p.tile_k[blockIdx.x];
  unsigned eb = block_exclusive(sb, s_warp, tb) + p.tile_b[blockIdx.x];
  const unsigned long long base = blockIdx.x * (unsigned long long)kScanTile + threadIdx.x * (unsigned long long)kScanItems;
#pragma unroll
  for (int j = 0; j < kScanItems; ++j) {
    const unsigned long long idx = base + j;
    if (idx < p.cells) { p.pk[idx] = ek; p.pb[idx] = eb; }
    ek += k[j];
    eb += b[j];
  }
}

// bounds[(o * (F + 1) + f) * 2 + {0,1}] = pk, pb at the first cell of (o, f);
// f = F gives the first cell of shard o + 1.
__global__ void route_bounds(RouteLaunch p) {
  const unsigned F = p.feature_count;
  const unsigned t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= p.shard_count * (F + 1)) return;
  const unsigned o = t / (F + 1), f = t % (F + 1);
  const unsigned long long idx = f < F ? o * p.bag_total + p.features[f].bag_base : (o + 1ull) * p.bag_total;
  p.bounds[2 * t] = p.pk[idx];
  p.bounds[2 * t + 1] = p.pb[idx];
}

// One block: the (shard, feature) row blocks of the gradient exchange (part_off:
// float offsets, row_pre: row prefix, shard-major), of the partials received
// (dd_off: distinct rows for deduplicated groups), the unique-key words of the
// payload (dd_words) and the count rows sent to every shard before the payload:
// [keys(F) kept(F) interleaved as (keys, kept) per feature | table ids (F) |
// poolings (F) | distinct keys (F, 0 = not deduplicated) | error], int64.
__global__ void __launch_bounds__(1024) route_layout(RouteLaunch p) {
  __shared__ unsigned s_warp[33];
  __shared__ unsigned long long s_carry[4];
  const unsigned F = p.feature_count, cells = p.shard_count * F;
  if (threadIdx.x < 4) s_carry[threadIdx.x] = 0;
  __syncthreads();
  const unsigned err = *(volatile const unsigned*)p.error;
  for (unsigned base = 0; base < cells; base += blockDim.x) {
    const unsigned c = base + threadIdx.x;
    unsigned rows = 0, floats = 0, dfloats = 0, words = 0;
    if (c < cells) {
      const unsigned o = c / F, f = c % F;
      unsigned keys, kept;
      group_counts(p, o, f, keys, kept);
      const LookupFeature* X = p.features + f;
      rows = X->pooling == 2 ? keys : kept;
      floats = rows * X->dim;
      const bool dd = dedup_eligible(p, X, o, f) && p.dd_count[c] < keys;
      const unsigned U = dd ? p.dd_count[c] : 0u;
      p.dd_used[c] = U;
      dfloats = (dd ? U : rows) * X->dim;
      words = dd ? U + 2 : 0u;
      long long* row = p.counts_out + (unsigned long long)o * (5 * F + 1);
      row[2 * f] = keys;
      row[2 * f + 1] = kept;
      row[2 * F + f] = X->table_rank;        // the table id, in a route's descriptors
      row[3 * F + f] = X->pooling;
      row[4 * F + f] = U;
      if (f == 0) row[5 * F] = err;
    }
    unsigned tr, tf, td, tw;
    const unsigned er = block_exclusive(rows, s_warp, tr);
    const unsigned ef = block_exclusive(floats, s_warp, tf);
    const unsigned ed = block_exclusive(dfloats, s_warp, td);
    const unsigned ew = block_exclusive(words, s_warp, tw);
    if (c < cells) {
      p.row_pre[c] = s_carry[0] + er;
      p.part_off[c] = s_carry[1] + ef;
      p.dd_off[c] = s_carry[2] + ed;
      p.dd_words[c] = s_carry[3] + ew;
    }
    __syncthreads();
    if (threadIdx.x == 0) { s_carry[0] += tr; s_carry[1] += tf; s_carry[2] += td; s_carry[3] += tw; }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    *p.row_total_dev = s_carry[0];
    p.dd_words[cells] = s_carry[3];
  }
}

// ---------------------------------------------------------------- scatter
__device__ __forceinline__ unsigned long long extra_of(const RouteLaunch& p, unsigned o) {
  // u64 words before shard o's keys that are not keys: the offsets, lengths and
  // unique-key regions of shards 0 .. o-1 (2 per kept bag + 1 per feature, and
  // U + 2 per deduplicated group)
  return 2ull * p.pb[o * p.bag_total] + (unsigned long long)o * p.feature_count +
         p.dd_words[o * p.feature_count];
}

__global__ void __launch_bounds__(256) route_scatter(RouteLaunch p) {
  __shared__ unsigned long long s_base[kMaxFeatures + 1];
  const unsigned fc = p.feature_count;
  for (unsigned i = threadIdx.x; i < fc; i += blockDim.x) s_base[i] = p.features[i].bag_base;
  if (threadIdx.x == 0) s_base[fc] = p.bag_total;
  __syncthreads();
  const unsigned n = p.shard_count;
  const unsigned long long B = p.bag_total;
  // leading zero of every (shard, feature) offsets region, and the offsets
  // [0, U] heading a deduplicated group's unique keys
  {
    const unsigned long long t = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x;
    if (t < (unsigned long long)n * fc) {
      const unsigned o = (unsigned)(t / fc), f = (unsigned)(t % fc);
      const unsigned long long keys_end = p.pk[(o + 1ull) * B] + extra_of(p, o);
      const unsigned long long at = keys_end + (p.pb[o * B + s_base[f]] - p.pb[o * B]) + f;
      p.payload[at] = 0ull;
      const unsigned U = p.dd_used[t];
      if (U) {
        const unsigned long long kept_o = p.pb[(o + 1ull) * B] - p.pb[o * B];
        const unsigned long long u_at = keys_end + 2 * kept_o + fc + (p.dd_words[t] - p.dd_words[o * fc]);
        p.payload[u_at] = 0ull;
        p.payload[u_at + 1] = U;
      }
    }
  }
  const unsigned lane = threadIdx.x & 31;
  const unsigned long long warp = (blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x) >> 5;
  const unsigned long long nwarps = (gridDim.x * (unsigned long long)blockDim.x) >> 5;
  const unsigned lt = (1u << lane) - 1u;
  // per-lane constants of shard `lane`
  unsigned long long my_extra = 0, my_keys_end = 0, my_lens_at = 0, my_uniq_at = 0;
  if (lane < n) {
    my_extra = extra_of(p, lane);
    my_keys_end = p.pk[(lane + 1ull) * B] + my_extra;
    my_lens_at = my_keys_end + (p.pb[(lane + 1ull) * B] - p.pb[lane * B]) + fc;
    my_uniq_at = my_lens_at + (p.pb[(lane + 1ull) * B] - p.pb[lane * B]);
  }
  for (unsigned long long g = warp; g < B; g += nwarps) {
    const unsigned f = feature_of(s_base, fc, g);
    const LookupFeature* F = p.features + f;
    const unsigned long long b = g - s_base[f];
    unsigned long long o2 = 0;
    if (lane < 2) o2 = F->offsets[b + lane];
    const unsigned long long s = __shfl_sync(~0u, o2, 0), e = __shfl_sync(~0u, o2, 1);
    // (validated by route_count: s <= e <= key_count)
    const bool has_pad = F->has_padding != 0;
    const unsigned long long pad_key = F->padding_key;
    unsigned c = 0, kept = 0, k_at = 0;
    if (lane < n) c = p.cnt[lane * B + g];
    // the bag's valid length: its keys, or its non-padding keys (all routed)
    const unsigned long long valid = has_pad ? __reduce_add_sync(~0u, c) : e - s;
    if (lane < n) {
      k_at = p.pk[lane * B + g];
      kept = p.pb[lane * B + g];
      if (c) {
        const unsigned long long fk = p.pk[lane * B + s_base[f]];
        const unsigned long long fb = p.pb[lane * B + s_base[f]];
        const unsigned long long j = kept - fb;                 // kept index inside (shard, feature)
        const unsigned long long rel = fb - p.pb[lane * B];     // kept bags of earlier features
        p.payload[my_keys_end + rel + f + j + 1] = (unsigned long long)k_at + c - fk;
        p.payload[my_lens_at + rel + j] = valid;
        p.bag_map[kept] = (unsigned)b;
      }
    }
    unsigned run = k_at;                 // lane o: next key index of shard o in this bag
    for (unsigned long long c0 = s; c0 < e; c0 += 32) {
      const unsigned long long i = c0 + lane;
      unsigned long long key = 0;
      unsigned owner = ~0u, rank = 0;
      if (i < e) {
        key = F->keys[i];
        owner = (has_pad && key == pad_key) ? ~0u : (unsigned)(key % n);
      }
      const unsigned before = run;
      for (unsigned o = 0; o < n; ++o) {
        const unsigned m = __ballot_sync(~0u, owner == o);
        if (owner == o) rank = __popc(m & lt);
        if (lane == o) run += __popc(m);
      }
      const unsigned o_safe = owner < n ? owner : 0u;
      const unsigned base = __shfl_sync(~0u, before, o_safe);
      const unsigned long long ex = __shfl_sync(~0u, my_extra, o_safe);
      const unsigned long long ua = __shfl_sync(~0u, my_uniq_at, o_safe);
      if (owner < n) {
        const unsigned q = base + rank;    // shard-ordered key index
        p.payload[q + ex] = key;
        p.pos_map[q] = (unsigned)i;
        const unsigned grp = owner * fc + f;
        if (p.dd_used[grp]) {
          // the key's rank among its group's distinct keys, and the key in the
          // group's unique list (every occurrence writes the same word)
          const unsigned r = dd_find(p, (key << 10) | grp);
          p.dd_idx[q] = r;
          p.payload[ua + (p.dd_words[grp] - p.dd_words[owner * fc]) + 2 + r] = key;
        }
      }
    }
  }
}

// ------------------------------------------------------------------ merge
// Group of G lanes per pooled bag: out = ((0 + p_0) + p_1) + ... over the shards
// that hold keys of the bag, then mean.  Sequence rows are copied to their
// positions by the second loop.
template <int G, int VEC, int ITERS>
__global__ void __launch_bounds__(256) route_merge(RouteLaunch p) {
  __shared__ unsigned long long s_base[kMaxFeatures + 1];
  const unsigned fc = p.feature_count;
  for (unsigned i = threadIdx.x; i < fc; i += blockDim.x) s_base[i] = p.features[i].bag_base;
  if (threadIdx.x == 0) s_base[fc] = p.bag_total;
  __syncthreads();
  constexpr int C = VEC * ITERS;
  const unsigned gl = threadIdx.x % G;
  const unsigned long long gid = (blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x) / G;
  const unsigned long long ngroups = (gridDim.x * (unsigned long long)blockDim.x) / G;
  const unsigned n = p.shard_count;
  const unsigned long long B = p.bag_total;
  for (unsigned long long g = gid; g < B; g += ngroups) {
    const unsigned f = feature_of(s_base, fc, g);
    const LookupFeature* F = p.features + f;
    if (F->pooling == 2) continue;
    const unsigned long long b = g - s_base[f];
    const unsigned D = F->dim;
    float acc[C];
#pragma unroll
    for (int k = 0; k < C; ++k) acc[k] = 0.0f;
    unsigned long long routed = 0;          // the bag's keys on all shards
    for (unsigned o = 0; o < n; ++o) {
      const unsigned c = p.cnt[o * B + g];
      routed += c;
      if (!c) continue;
      // a deduplicated group's row is its key's distinct row
      const unsigned long long j = p.dd_used[o * fc + f] ? p.dd_idx[p.pk[o * B + g]]
                                                          : p.pb[o * B + g] - p.pb[o * B + s_base[f]];
      const float* row = p.partials + p.dd_off[o * fc + f] + j * D;
#pragma unroll
      for (int it = 0; it < ITERS; ++it) {
        const unsigned col = (it * G + gl) * VEC;
        if (col >= D) continue;
        float t[VEC];
        load_vec<VEC>(row + col, t);
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc[it * VEC + v] = __fadd_rn(acc[it * VEC + v], t[v]);
      }
    }
    const bool mean = F->pooling == 1;
    // the valid length: the bag's keys, or (padding) its non-padding keys
    const unsigned long long len = F->has_padding ? routed : F->offsets[b + 1] - F->offsets[b];
    const float denom = (float)len;
    float* out = p.outs[f] + b * D;
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
      const unsigned col = (it * G + gl) * VEC;
      if (col >= D) continue;
      float t[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v)
        t[v] = (mean && len) ? __fdiv_rn(acc[it * VEC + v], denom) : acc[it * VEC + v];
      store_vec<VEC>(out + col, t);
    }
  }
  if (!p.has_sequence) return;
  // sequence features: shard-ordered key q -> position pos_map[q], over the keys
  // that were routed (padding keys were not)
  const unsigned long long routed_total = p.pk[(unsigned long long)n * B];
  for (unsigned long long q = gid; q < routed_total; q += ngroups) {
    // shard: largest o with pk[o * B] <= q; then feature inside the shard
    unsigned o = 0;
    {
      unsigned lo = 0, hi = n;
      while (hi - lo > 1) { const unsigned mid = (lo + hi) >> 1; if (p.bounds[2 * mid * (fc + 1)] <= q) lo = mid; else hi = mid; }
      o = lo;
    }
    const unsigned* ob = p.bounds + 2ull * o * (fc + 1);
    unsigned lo = 0, hi = fc;
    while (hi - lo > 1) { const unsigned mid = (lo + hi) >> 1; if (ob[2 * mid] <= q) lo = mid; else hi = mid; }
    // skip empty features that share the start index
    while (lo + 1 < fc && ob[2 * (lo + 1)] <= q) ++lo;
    const unsigned f = lo;
    const LookupFeature* F = p.features + f;
    if (F->pooling != 2) continue;
    const unsigned D = F->dim;
    const unsigned long long j = p.dd_used[o * fc + f] ? p.dd_idx[q] : q - ob[2 * f];
    const float* row = p.partials + p.dd_off[o * fc + f] + j * (unsigned long long)D;
    float* out = p.outs[f] + (unsigned long long)p.pos_map[q] * D;
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
      const unsigned col = (it * G + gl) * VEC;
      if (col >= D) continue;
      float t[VEC];
      load_vec<VEC>(row + col, t);
      store_vec<VEC>(out + col, t);
    }
  }
  // positions of padded sequence features that hold the padding key read zeros
  for (unsigned f = 0; f < fc; ++f) {
    const LookupFeature* F = p.features + f;
    if (F->pooling != 2 || !F->has_padding) continue;
    const unsigned D = F->dim;
    for (unsigned long long i = gid; i < F->key_count; i += ngroups) {
      if (F->keys[i] != F->padding_key) continue;
      float* out = p.outs[f] + i * D;
#pragma unroll
      for (int it = 0; it < ITERS; ++it) {
        const unsigned col = (it * G + gl) * VEC;
        if (col >= D) continue;
        float t[VEC];
#pragma unroll
        for (int v = 0; v < VEC; ++v) t[v] = 0.0f;
        store_vec<VEC>(out + col, t);
      }
    }
  }
}

// ----------------------------------------------------------------- gather
// Gradient rows sent to each shard, shard-major then feature-major: pooled
// features send the kept bags' rows, sequence features the rows of the keys.
template <int G, int VEC, int ITERS>
__global__ void __launch_bounds__(256) route_gather(RouteLaunch p) {
  const unsigned fc = p.feature_count;
  const unsigned blocks = p.shard_count * fc;        // (shard, feature) row blocks
  const unsigned gl = threadIdx.x % G;
  const unsigned long long gid = (blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x) / G;
  const unsigned long long ngroups = (gridDim.x * (unsigned long long)blockDim.x) / G;
  const unsigned long long B = p.bag_total;
  const unsigned long long row_total = *p.row_total_dev;
  for (unsigned long long r = gid; r < row_total; r += ngroups) {
    unsigned lo = 0, hi = blocks;
    while (hi - lo > 1) { const unsigned mid = (lo + hi) >> 1; if (p.row_pre[mid] <= r) lo = mid; else hi = mid; }
    while (lo + 1 < blocks && p.row_pre[lo + 1] <= r) ++lo;
    const unsigned o = lo / fc, f = lo % fc;
    const LookupFeature* F = p.features + f;
    const unsigned D = F->dim;
    const unsigned long long j = r - p.row_pre[lo];
    unsigned long long src;
    if (F->pooling == 2) src = p.pos_map[p.pk[o * B + F->bag_base] + j];
    else src = p.bag_map[p.pb[o * B + F->bag_base] + j];
    const float* row = p.grads[f] + src * D;
    float* dst = p.send + p.part_off[lo] + j * D;
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
      const unsigned col = (it * G + gl) * VEC;
      if (col >= D) continue;
      float t[VEC];
      load_vec<VEC>(row + col, t);
      store_vec<VEC>(dst + col, t);
    }
  }
  if (!p.nonfinite) return;
  // every gradient value must be finite, sent or not (distributed_client.cpp:249);
  // the largest |g| too, which the owners' pushes take as their overflow bound
  // instead of reading the received rows again
  const unsigned long long tid = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x;
  const unsigned long long nthreads = gridDim.x * (unsigned long long)blockDim.x;
  unsigned bad = 0;
  float mx = 0.0f;
  for (unsigned f = 0; f < fc; ++f) {
    const LookupFeature* F = p.features + f;
    const unsigned long long rows = F->pooling == 2 ? F->key_count : F->bag_count;
    const unsigned long long total = rows * F->dim;
    const float* g = p.grads[f];
    for (unsigned long long i = tid; i < total; i += nthreads) {
      const float x = g[i];
      bad |= !isfinite(x);
      mx = fmaxf(mx, fabsf(x));
    }
  }
  bad = __reduce_or_sync(~0u, bad);
  const unsigned mb = __reduce_max_sync(~0u, __float_as_uint(mx));
  if ((threadIdx.x & 31) == 0) {
    if (bad) atomicOr(p.nonfinite, 1u);
    if (mb) atomicMax(p.nonfinite + 1, mb);
  }
}

unsigned grid_for(unsigned long long groups, unsigned per_block) {
  const unsigned long long want = (groups + per_block - 1) / per_block;
  const unsigned long long cap = 148ull * 8 * 4;
  return (unsigned)std::max(1ull, std::min(want, cap));
}

template <int G, int VEC, int ITERS>
cudaError_t launch_merge_shape(const RouteLaunch& p, cudaStream_t s) {
  const unsigned long long items = std::max(p.bag_total, p.has_sequence ? p.key_total : 0ull);
  route_merge<G, VEC, ITERS><<<grid_for(items, 256 / G), 256, 0, s>>>(p);
  return cudaGetLastError();
}
template <int G, int VEC, int ITERS>
cudaError_t launch_gather_shape(const RouteLaunch& p, cudaStream_t s) {
  // rows are at most keys + bags (the exact count is read on the device)
  route_gather<G, VEC, ITERS><<<grid_for(std::max(p.key_total + p.bag_total, 1ull), 256 / G), 256, 0, s>>>(p);
  return cudaGetLastError();
}

#define EPS_ROUTE_SHAPES(FN)                                         \
  if (p.vec == 4) {                                                  \
    switch (p.group) {                                               \
      case 8: return FN<8, 4, 1>(p, stream);                         \
      case 16: return FN<16, 4, 1>(p, stream);                       \
      default:                                                       \
        if (p.iters == 1) return FN<32, 4, 1>(p, stream);            \
        if (p.iters == 2) return FN<32, 4, 2>(p, stream);            \
        return FN<32, 4, 4>(p, stream);                              \
    }                                                                \
  }                                                                  \
  if (p.iters == 1) return FN<32, 1, 1>(p, stream);                  \
  if (p.iters == 2) return FN<32, 1, 2>(p, stream);                  \
  return FN<32, 1, 4>(p, stream);

}  // namespace

unsigned route_tiles(unsigned long long cells) {
  return (unsigned)((cells + kScanTile - 1) / kScanTile);
}

cudaError_t launch_route_count(const RouteLaunch& p, cudaStream_t stream) {
  if (p.bag_total) {
    route_count<<<grid_for(p.bag_total, 8), 256, 0, stream>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  const unsigned tiles = route_tiles(p.cells);
  if (tiles) {
    route_tile_sums<<<tiles, kScanThreads, 0, stream>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  route_tile_scan<<<1, 1024, 0, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (tiles) {
    route_tile_apply<<<tiles, kScanThreads, 0, stream>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  const unsigned nb = p.shard_count * (p.feature_count + 1);
  route_bounds<<<(nb + 255) / 256, 256, 0, stream>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (p.dd_mask && p.bag_total) {
    route_dedup_claim<<<grid_for(p.bag_total, 8), 256, 0, stream>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  route_layout<<<1, 1024, 0, stream>>>(p);
  return cudaGetLastError();
}

unsigned route_count_launches(const RouteLaunch& p) {
  const unsigned tiles = route_tiles(p.cells);
  return (p.bag_total ? 1u : 0u) + (tiles ? 2u : 0u) + 3u + (p.dd_mask && p.bag_total ? 1u : 0u);
}

cudaError_t launch_route_scatter(const RouteLaunch& p, cudaStream_t stream) {
  const unsigned long long zeros_blocks = ((unsigned long long)p.shard_count * p.feature_count + 255) / 256;
  const unsigned grid = std::max<unsigned>(grid_for(p.bag_total, 8), (unsigned)zeros_blocks);
  route_scatter<<<grid, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_route_merge(const RouteLaunch& p, cudaStream_t stream) {
  EPS_ROUTE_SHAPES(launch_merge_shape)
}

cudaError_t launch_route_gather(const RouteLaunch& p, cudaStream_t stream) {
  EPS_ROUTE_SHAPES(launch_gather_shape)
}

}  // namespace eps_b200
