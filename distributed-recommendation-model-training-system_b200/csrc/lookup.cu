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
// 32/G bags.  The group fetches G keys with one coalesced load, broadcasts them
// by shuffle and keeps up to 8 row loads in flight ahead of the dependent adds.
// When the lookup will be pushed (non-read-only), the same pass writes the
// occurrence list consumed by the coalescing sort: composite key (table rank,
// slot) and gradient source (feature, row), plus the mean scale 1.0f/len of
// every gradient row (src/access/batch_access.cpp:107-108).
#include <cooperative_groups.h>
#include <cooperative_groups/reduce.h>

#include "kernels.cuh"

namespace cg = cooperative_groups;

namespace eps_b200 {
namespace {

template <int G, int VEC, int ITERS, typename KeyT>
__global__ void __launch_bounds__(256, (VEC * ITERS <= 4) ? 3 : 2) lookup_kernel(LookupLaunch p) {
  __shared__ unsigned long long s_item_base[kMaxFeatures + 1];
  const unsigned fc = p.feature_count;
  for (unsigned i = threadIdx.x; i < fc; i += blockDim.x) s_item_base[i] = p.features[i].item_base;
  if (threadIdx.x == 0) s_item_base[fc] = p.item_total;
  __syncthreads();

  const auto grp = cg::tiled_partition<G>(cg::this_thread_block());
  const unsigned gl = grp.thread_rank();
  const unsigned long long gid = (blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x) / G;
  const unsigned long long ngroups = (gridDim.x * (unsigned long long)blockDim.x) / G;
  constexpr int C = VEC * ITERS;
  constexpr int DEPTH = C <= 4 ? 8 : (C <= 8 ? 4 : 2);
  unsigned int err = 0;

  for (unsigned long long item = gid; item < p.item_total; item += ngroups) {
    // feature owning the item: largest f with item_base[f] <= item
    unsigned lo = 0, hi = fc;
    while (hi - lo > 1) { const unsigned mid = (lo + hi) >> 1; if (s_item_base[mid] <= item) lo = mid; else hi = mid; }
    const LookupFeature* F = p.features + lo;
    const unsigned long long bag_count = F->bag_count;
    const unsigned long long b0 = (item - s_item_base[lo]) * p.bags_per_item;
    const unsigned nb = (unsigned)min((unsigned long long)p.bags_per_item, bag_count - b0);
    const unsigned long long key_count = F->key_count;
    // offsets of bags b0 .. b0+nb in one load: lane j holds offsets[b0 + j]
    unsigned long long ob = 0, lb = 0;
    if (gl <= nb) ob = F->offsets[b0 + gl];
    if (F->lengths && gl < nb) lb = F->lengths[b0 + gl];
    {
      const unsigned long long nxt = grp.shfl_down(ob, 1);
      bool bad = gl < nb && nxt < ob;                              // decreasing
      bad |= gl == nb && ob > key_count;                           // beyond the keys
      bad |= gl == 0 && b0 == 0 && ob != 0;                        // must start at 0
      bad |= gl == nb && b0 + nb == bag_count && ob != key_count;  // must end at N
      if (grp.any(bad)) {
        err |= kLookupBadOffsets;
        // treat every bag as empty (the shuffle runs on every lane of the group)
        const unsigned long long first = grp.shfl(ob, 0);
        ob = (gl <= nb) ? min(first, key_count) : 0;
      }
    }
    const float* state = F->state;
    const unsigned D = F->dim;
    const unsigned long long row_stride = 3ull * D;
    const bool sequence = F->pooling == 2;
    const bool mean = F->pooling == 1;
    float* const out = F->out;
    const unsigned long long k_begin = grp.shfl(ob, 0);
    const unsigned long long k_end = grp.shfl(ob, nb);

    float acc[C];
#pragma unroll
    for (int k = 0; k < C; ++k) acc[k] = 0.0f;
    unsigned j = 0;                                    // bag being accumulated (relative)
    unsigned long long bag_end = grp.shfl(ob, 1);

    // writes the pooled row of relative bag j (sum or mean) and its scale
    auto finish_bag = [&](unsigned jb) {
      const unsigned long long b = b0 + jb;
      const unsigned long long s = grp.shfl(ob, jb), e = grp.shfl(ob, jb + 1);
      unsigned long long len = e - s;
      if (F->lengths) {
        const unsigned long long given = grp.shfl(lb, jb);
        if (given < len) err |= kLookupShortLength;
        len = given;
      }
      if (!sequence) {
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
        if (p.emit && gl == 0)
          p.row_scale[F->scale_base + b] = (mean && len) ? __fdiv_rn(1.0f, denom) : 1.0f;
      }
#pragma unroll
      for (int k = 0; k < C; ++k) acc[k] = 0.0f;
    };
    // bags that end before the first key (empty bags)
    while (j < nb && bag_end <= k_begin) { finish_bag(j); ++j; bag_end = grp.shfl(ob, min(j + 1, nb)); }

    for (unsigned long long c0 = k_begin; c0 < k_end; c0 += G) {
      const unsigned long long i = c0 + gl;
      unsigned slot = ~0u;                     // slots fit 32 bits: rows < 2^32 per shard
      // bag of key i among this item's bags: largest q with offsets[b0 + q] <= i
      // (fixed-step binary search, executed by every lane of the group)
      unsigned long long bag = b0;
      if (p.emit && !sequence) {
        unsigned qlo = 0, qhi = nb;
#pragma unroll
        for (int step = 0; step < 5; ++step) {
          const unsigned mid = (qlo + qhi + 1) >> 1;
          const unsigned long long om = grp.shfl(ob, min(mid, nb));
          if (qhi > qlo && om <= i) qlo = mid; else if (qhi > qlo) qhi = mid - 1;
        }
        bag = b0 + qlo;
      }
      if (i < k_end) {
        const unsigned long long key = F->keys[i];
        unsigned long long sl, sh;
        if (p.shard_count == 1) { sl = key; sh = 0; }
        else { sl = key / p.shard_count; sh = key - sl * p.shard_count; }
        if (sh == p.shard_id && sl < F->rows) slot = (unsigned)sl;
        else err |= kLookupBadKey;
        if (p.emit) {
          const unsigned long long o = F->occ_base + i;
          const KeyT ck = (slot == ~0u) ? KeyT(0)
              : (KeyT(F->table_rank) << p.slot_bits) | KeyT(slot);
          static_cast<KeyT*>(p.occ_key)[o] = ck;
          p.occ_src[o] = (F->feature_index << kRowBits) | (unsigned)(sequence ? i : bag);
          if (sequence) p.row_scale[F->scale_base + i] = 1.0f;
        }
      }
      const int cnt = (int)min((unsigned long long)G, k_end - c0);
      for (int j0 = 0; j0 < cnt; j0 += DEPTH) {
        float r[DEPTH][C];
        unsigned sl[DEPTH];
#pragma unroll
        for (int u = 0; u < DEPTH; ++u) {
          sl[u] = grp.shfl(slot, (j0 + u) & (G - 1));
          const bool use = (j0 + u < cnt) && sl[u] != ~0u;
#pragma unroll
          for (int it = 0; it < ITERS; ++it) {
            const unsigned col = (it * G + gl) * VEC;
            float t[VEC];
            if (use && col < D) load_vec<VEC>(state + (unsigned long long)sl[u] * row_stride + col, t);
            else {
#pragma unroll
              for (int v = 0; v < VEC; ++v) t[v] = 0.0f;
            }
#pragma unroll
            for (int v = 0; v < VEC; ++v) r[u][it * VEC + v] = t[v];
          }
        }
#pragma unroll
        for (int u = 0; u < DEPTH; ++u) {
          if (j0 + u >= cnt) break;
          const unsigned long long ki = c0 + j0 + u;
          if (sl[u] != ~0u) {
            if (sequence) {
              // one output row per position: 0 + w (batch_access.cpp:74-76)
#pragma unroll
              for (int it = 0; it < ITERS; ++it) {
                const unsigned col = (it * G + gl) * VEC;
                if (col >= D) continue;
                float t[VEC];
#pragma unroll
                for (int v = 0; v < VEC; ++v) t[v] = __fadd_rn(0.0f, r[u][it * VEC + v]);
                store_vec<VEC>(out + ki * D + col, t);
              }
            } else {
#pragma unroll
              for (int k = 0; k < C; ++k) acc[k] = __fadd_rn(acc[k], r[u][k]);
            }
          }
          // bags ending at this key (and empty bags right after it)
          while (j < nb && bag_end <= ki + 1) { finish_bag(j); ++j; bag_end = grp.shfl(ob, min(j + 1, nb)); }
        }
      }
    }
    while (j < nb) { finish_bag(j); ++j; }
  }
  err = cg::reduce(grp, err, cg::bit_or<unsigned>());
  if (err && gl == 0) atomicOr(p.error, err);
}

template <int G, int VEC, int ITERS>
cudaError_t launch_key(const LookupLaunch& p, cudaStream_t s) {
  const unsigned long long groups_per_block = 256 / G;
  const unsigned long long want = (p.item_total + groups_per_block - 1) / groups_per_block;
  const unsigned long long cap = 148ull * ((VEC * ITERS <= 4) ? 3 : 2) * 8;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  if (p.key64) lookup_kernel<G, VEC, ITERS, unsigned long long><<<grid, 256, 0, s>>>(p);
  else lookup_kernel<G, VEC, ITERS, unsigned int><<<grid, 256, 0, s>>>(p);
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_lookup(const LookupLaunch& p, cudaStream_t stream) {
  if (p.item_total == 0) return cudaSuccess;
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
