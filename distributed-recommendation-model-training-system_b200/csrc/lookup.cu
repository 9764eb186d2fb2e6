// lookup.cu -- batched embedding pull: row gather with sum / mean / sequence
// pooling over every feature of a lookup in ONE launch.
//
// Reference semantics followed:
//   * shard partial, src/access/batch_access.cpp:67-78: a zeroed contribution to
//     which each of the shard's rows is added in position order (sum/mean), or
//     one row per position (sequence);
//   * client merge and mean, src/client/distributed_client.cpp:173-188,227-232:
//     the zeroed output receives the shard partial in shard order and mean bags
//     are divided once by (float)valid_length (skipped for length 0).
// The per-bag sum is evaluated in exactly that order, so pooled outputs are
// bit-identical to the reference's.
//
// Work decomposition: a group of G lanes (G = D/4 for D = 32/64/128, so a row
// is read with one 128-bit load per lane) owns one bag at a time; a warp holds
// 32/G bags.  The group fetches G keys with one coalesced load (the next chunk's
// keys are requested before the current chunk's rows), broadcasts the slots by
// shuffle and issues up to DEPTH row loads back to back before the dependent
// adds.  Rows past the end of a chunk are added as -0.0f, the additive identity
// of round-to-nearest addition, so the add loop carries no predicates.
// When the lookup will be pushed (non-read-only), `emit_kernel` writes the
// occurrence list consumed by the coalescing sort before the gather runs:
// composite key (table rank, slot) and gradient source (feature, row), plus the
// mean scale 1.0f/len of every gradient row (src/access/batch_access.cpp:107-108).
#include <cooperative_groups.h>
#include <cooperative_groups/reduce.h>

#include "kernels.cuh"

namespace cg = cooperative_groups;

namespace eps_b200 {
namespace {

// The gather is bound by each bag's chain of dependent loads (offsets, keys,
// rows), so more bags in flight (4 blocks of 256 per SM) pays more than more
// rows in flight per bag (4 per group): cfg2 109 -> 90 us.
#ifndef EPS_LOOKUP_DEPTH_REGS
#define EPS_LOOKUP_DEPTH_REGS 16     // registers per lane for rows in flight
#endif
#ifndef EPS_LOOKUP_MIN_BLOCKS
#define EPS_LOOKUP_MIN_BLOCKS 4
#endif

template <int G, int VEC, int ITERS, typename KeyT>
__global__ void __launch_bounds__(256, EPS_LOOKUP_MIN_BLOCKS) lookup_kernel(LookupLaunch p) {
  __shared__ unsigned long long s_bag_base[kMaxFeatures + 1];
  const unsigned fc = p.feature_count;
  for (unsigned i = threadIdx.x; i < fc; i += blockDim.x) s_bag_base[i] = p.features[i].bag_base;
  if (threadIdx.x == 0) s_bag_base[fc] = p.bag_total;
  __syncthreads();

  const auto grp = cg::tiled_partition<G>(cg::this_thread_block());
  const unsigned gl = grp.thread_rank();
  const unsigned long long gid = (blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x) / G;
  const unsigned long long ngroups = (gridDim.x * (unsigned long long)blockDim.x) / G;
  constexpr int C = VEC * ITERS;
  constexpr int DEPTH = G < EPS_LOOKUP_DEPTH_REGS / C ? G : EPS_LOOKUP_DEPTH_REGS / C;
  unsigned int err = 0;

  for (unsigned long long g = gid; g < p.bag_total; g += ngroups) {
    // feature owning bag g: largest f with bag_base[f] <= g
    unsigned lo = 0, hi = fc;
    while (hi - lo > 1) { const unsigned mid = (lo + hi) >> 1; if (s_bag_base[mid] <= g) lo = mid; else hi = mid; }
    const LookupFeature* F = p.features + lo;
    const unsigned long long b = g - s_bag_base[lo];
    const unsigned long long key_count = F->key_count;
    // offsets[b] and offsets[b + 1] by lanes 0 and 1
    unsigned long long o = 0;
    if (gl < 2) o = F->offsets[b + gl];
    unsigned long long s = grp.shfl(o, 0), e = grp.shfl(o, 1);
    if (b == 0 && s != 0) err |= kLookupBadOffsets;
    if (b + 1 == F->bag_count && e != key_count) err |= kLookupBadOffsets;
    if (s > e || e > key_count) { err |= kLookupBadOffsets; s = e = 0; }
    const unsigned long long* const keys = F->keys;
    const float* const state = F->state;
    float* const out = F->out;
    const unsigned D = F->dim;
    const unsigned long long rows = F->rows;
    const unsigned long long row_stride = 3ull * D;
    const bool sequence = F->pooling == 2;

    float acc[C];
#pragma unroll
    for (int k = 0; k < C; ++k) acc[k] = 0.0f;

    // padding keys (PrepareAdapterInput, src/access/prepare_queue.cpp:69-77) are
    // dropped: no row, no gradient; mean bags divide by the kept count and
    // sequence positions holding padding read as zeros
    const bool has_pad = F->has_padding != 0;
    const unsigned long long pad_key = F->padding_key;
    unsigned long long kept = 0;
    unsigned long long key = (s + gl < e) ? keys[s + gl] : 0ull;
    for (unsigned long long c0 = s; c0 < e; c0 += G) {
      const unsigned long long i = c0 + gl;
      unsigned slot = ~0u;              // slots fit 32 bits: rows < 2^32 - 2 per shard
      if (i < e && has_pad && key == pad_key) {
        slot = kPadSlot;
      } else if (i < e) {
        unsigned long long sl, sh;
        if (p.shard_count == 1) { sl = key; sh = 0; }
        else { sl = key / p.shard_count; sh = key - sl * p.shard_count; }
        if (sh == p.shard_id && sl < rows) slot = (unsigned)sl;
        else err |= kLookupBadKey;
      }
      // next chunk's keys in flight while this chunk's rows load
      if (i + G < e) key = keys[i + G];
      const int cnt = (int)min((unsigned long long)G, e - c0);
      if (has_pad) kept += __popc(grp.ballot(i < e && slot != kPadSlot));
#pragma unroll 1
      for (int j0 = 0; j0 < cnt; j0 += DEPTH) {
        float r[DEPTH][C];
        bool use[DEPTH], padrow[DEPTH];
#pragma unroll
        for (int u = 0; u < DEPTH; ++u) {
          const unsigned su = grp.shfl(slot, (j0 + u) & (G - 1));
          padrow[u] = (j0 + u < cnt) && su == kPadSlot;
          use[u] = (j0 + u < cnt) && su < kPadSlot;
          const float* row = state + (unsigned long long)su * row_stride;
#pragma unroll
          for (int it = 0; it < ITERS; ++it) {
            const unsigned col = (it * G + gl) * VEC;
            float t[VEC];
            if (use[u] && col < D) load_vec<VEC>(row + col, t);
            else {
#pragma unroll
              for (int v = 0; v < VEC; ++v) t[v] = -0.0f;
            }
#pragma unroll
            for (int v = 0; v < VEC; ++v) r[u][it * VEC + v] = t[v];
          }
        }
        if (sequence) {
          // one output row per position: 0 + w (batch_access.cpp:74-76)
#pragma unroll
          for (int u = 0; u < DEPTH; ++u) {
            if (!use[u] && !padrow[u]) continue;
            const unsigned long long pos = c0 + j0 + u;
#pragma unroll
            for (int it = 0; it < ITERS; ++it) {
              const unsigned col = (it * G + gl) * VEC;
              if (col >= D) continue;
              float t[VEC];
#pragma unroll
              for (int v = 0; v < VEC; ++v) t[v] = padrow[u] ? 0.0f : __fadd_rn(0.0f, r[u][it * VEC + v]);
              store_vec<VEC>(out + pos * D + col, t);
            }
          }
        } else {
          // position order; -0.0f padding leaves acc unchanged
#pragma unroll
          for (int u = 0; u < DEPTH; ++u)
#pragma unroll
            for (int k = 0; k < C; ++k) acc[k] = __fadd_rn(acc[k], r[u][k]);
        }
      }
    }
    if (!sequence) {
      unsigned long long len = has_pad ? kept : e - s;
      if (F->lengths) {
        const unsigned long long given = F->lengths[b];
        if (given < len) err |= kLookupShortLength;
        len = given;
      }
      const bool mean = F->pooling == 1;
      const float denom = (float)len;   // u64 -> float, round to nearest
#pragma unroll
      for (int it = 0; it < ITERS; ++it) {
        const unsigned col = (it * G + gl) * VEC;
        if (col >= D) continue;
        float t[VEC];
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          float x = acc[it * VEC + v];
          if (p.client) {
            x = __fadd_rn(0.0f, x);
            if (mean && len) x = __fdiv_rn(x, denom);
          }
          t[v] = x;
        }
        store_vec<VEC>(out + b * D + col, t);
      }
    }
  }
  err = cg::reduce(grp, err, cg::bit_or<unsigned>());
  if (err && gl == 0) atomicOr(p.error, err);
}

// Occurrence list of a lookup that will be pushed, ahead of (and independent
// of) the gather, so that the coalescing sort can run concurrently with the
// gather: one warp per bag writes every occurrence's composite key (table
// rank, slot) and gradient source (feature, bag or position) and the gradient
// row scales (1.0f / valid length for mean, src/access/batch_access.cpp:107-108).
// Validation matches the gather kernel's.
template <typename KeyT>
__global__ void __launch_bounds__(256) emit_kernel(LookupLaunch p) {
  __shared__ unsigned long long s_bag_base[kMaxFeatures + 1];
  const unsigned fc = p.feature_count;
  for (unsigned i = threadIdx.x; i < fc; i += blockDim.x) s_bag_base[i] = p.features[i].bag_base;
  if (threadIdx.x == 0) s_bag_base[fc] = p.bag_total;
  __syncthreads();
  const unsigned lane = threadIdx.x & 31;
  const unsigned long long warp = (blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x) >> 5;
  const unsigned long long nwarps = (gridDim.x * (unsigned long long)blockDim.x) >> 5;
  unsigned err = 0;
  for (unsigned long long g = warp; g < p.bag_total; g += nwarps) {
    unsigned lo = 0, hi = fc;
    while (hi - lo > 1) { const unsigned mid = (lo + hi) >> 1; if (s_bag_base[mid] <= g) lo = mid; else hi = mid; }
    const LookupFeature* F = p.features + lo;
    const unsigned long long b = g - s_bag_base[lo];
    const unsigned long long key_count = F->key_count;
    unsigned long long o = 0;
    if (lane < 2) o = F->offsets[b + lane];
    unsigned long long s = __shfl_sync(~0u, o, 0), e = __shfl_sync(~0u, o, 1);
    if (b == 0 && s != 0) err |= kLookupBadOffsets;
    if (b + 1 == F->bag_count && e != key_count) err |= kLookupBadOffsets;
    if (s > e || e > key_count) { err |= kLookupBadOffsets; s = e = 0; }
    const bool sequence = F->pooling == 2;
    const bool has_pad = F->has_padding != 0;
    const unsigned long long pad_key = F->padding_key;
    const unsigned long long rows = F->rows, occ_base = F->occ_base;
    const unsigned src_hi = F->feature_index << kRowBits;
    const KeyT rank_bits = KeyT(F->table_rank) << p.slot_bits;
    unsigned long long kept = 0;
    for (unsigned long long c0 = s; c0 < e; c0 += 32) {
      const unsigned long long i = c0 + lane;
      bool pad = false;
      if (i < e) {
        const unsigned long long key = F->keys[i];
        KeyT ck = KeyT(0);
        if (has_pad && key == pad_key) {
          pad = true;
          ck = KeyT(p.pad_key);        // sorts after every row key; the push skips it
        } else {
          unsigned long long sl, sh;
          if (p.shard_count == 1) { sl = key; sh = 0; }
          else { sl = key / p.shard_count; sh = key - sl * p.shard_count; }
          if (sh == p.shard_id && sl < rows) ck = rank_bits | KeyT(sl);
          else err |= kLookupBadKey;
        }
        static_cast<KeyT*>(p.occ_key)[occ_base + i] = ck;
        p.occ_src[occ_base + i] = src_hi | (unsigned)(sequence ? i : b);
        if (sequence) p.row_scale[F->scale_base + i] = 1.0f;
      }
      kept += __popc(__ballot_sync(~0u, i < e && !pad));
    }
    if (!sequence && lane == 0) {
      unsigned long long len = has_pad ? kept : e - s;
      if (F->lengths) {
        const unsigned long long given = F->lengths[b];
        if (given < len) err |= kLookupShortLength;
        len = given;
      }
      const bool mean = F->pooling == 1;
      p.row_scale[F->scale_base + b] = (mean && len) ? __fdiv_rn(1.0f, (float)len) : 1.0f;
    }
  }
  err = __reduce_or_sync(~0u, err);
  if (err && lane == 0) atomicOr(p.error, err);
}

template <int G, int VEC, int ITERS>
cudaError_t launch_key(const LookupLaunch& p, cudaStream_t s) {
  const unsigned long long groups_per_block = 256 / G;
  const unsigned long long want = (p.bag_total + groups_per_block - 1) / groups_per_block;
  const unsigned long long cap = 148ull * EPS_LOOKUP_MIN_BLOCKS * 4;   // 4 waves
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  if (p.key64) lookup_kernel<G, VEC, ITERS, unsigned long long><<<grid, 256, 0, s>>>(p);
  else lookup_kernel<G, VEC, ITERS, unsigned int><<<grid, 256, 0, s>>>(p);
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_emit(const LookupLaunch& p, cudaStream_t stream) {
  if (p.bag_total == 0) return cudaSuccess;
  const unsigned long long want = (p.bag_total + 7) / 8;
  const unsigned grid = (unsigned)(want < 148ull * 8 * 2 ? want : 148ull * 8 * 2);
  if (p.key64) emit_kernel<unsigned long long><<<grid, 256, 0, stream>>>(p);
  else emit_kernel<unsigned int><<<grid, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_lookup(const LookupLaunch& p, cudaStream_t stream) {
  if (p.bag_total == 0) return cudaSuccess;
  if (p.vec == 4) {
    switch (p.group) {
      case 8: return launch_key<8, 4, 1>(p, stream);
      case 16: return launch_key<16, 4, 1>(p, stream);
      default:
        if (p.iters == 1) return launch_key<32, 4, 1>(p, stream);
        if (p.iters == 2) return launch_key<32, 4, 2>(p, stream);
        return launch_key<32, 4, 4>(p, stream);
    }
  }
  if (p.iters == 1) return launch_key<32, 1, 1>(p, stream);
  if (p.iters == 2) return launch_key<32, 1, 2>(p, stream);
  return launch_key<32, 1, 4>(p, stream);
}

}  // namespace eps_b200
