// lookup.cu -- batched embedding pull: row gather with sum / mean / sequence
// pooling over every feature of a lookup in ONE launch.
//
// Reference semantics followed:
//   * shard partial, src/access/batch_access.cpp:67-78: a zeroed contribution to
//     which each of the shard's rows is added in position order (sum/mean), or
//     one row per position (sequence);
//   * client merge and mean, src/client/distributed_client.cpp:173-188,227-232:
//     the zeroed output receives the shard partial(s) in shard order and mean
//     bags are divided once by (float)valid_length (skipped for length 0).
// The per-bag sum is evaluated in exactly that order, so pooled outputs are
// bit-identical to the reference's.
//
// Work decomposition: one warp per bag; lanes split the embedding dimension in
// VEC-wide (up to 128-bit) coalesced chunks; keys of a bag are fetched 32 at a
// time with one coalesced load and broadcast by shuffles; row loads are issued
// four at a time ahead of the dependent adds.  When the lookup will be pushed
// (non-read-only), the same pass writes the occurrence list consumed by the
// coalescing sort: composite key (table rank, slot) and gradient source
// (feature, row), plus the mean scale 1.0f/len of every gradient row
// (src/access/batch_access.cpp:107-108).
#include "kernels.cuh"

namespace eps_b200 {
namespace {

template <int VEC, int ITERS, typename KeyT>
__global__ void __launch_bounds__(256) lookup_kernel(LookupLaunch p) {
  __shared__ unsigned long long s_bag_base[kMaxFeatures + 1];
  const unsigned fc = p.feature_count;
  for (unsigned i = threadIdx.x; i < fc; i += blockDim.x) s_bag_base[i] = p.features[i].bag_base;
  if (threadIdx.x == 0) s_bag_base[fc] = p.bag_total;
  __syncthreads();

  const unsigned lane = lane_id();
  const unsigned long long warp = (blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x) >> 5;
  const unsigned long long nwarps = (gridDim.x * (unsigned long long)blockDim.x) >> 5;
  constexpr int C = VEC * ITERS;
  int cached = -1;
  LookupFeature F;
  unsigned int err = 0;

  for (unsigned long long g = warp; g < p.bag_total; g += nwarps) {
    // feature owning bag g: largest f with bag_base[f] <= g
    unsigned lo = 0, hi = fc;
    while (hi - lo > 1) { const unsigned mid = (lo + hi) >> 1; if (s_bag_base[mid] <= g) lo = mid; else hi = mid; }
    if ((int)lo != cached) { F = p.features[lo]; cached = (int)lo; }
    const unsigned long long b = g - F.bag_base;
    const unsigned D = F.dim;
    unsigned long long s = F.offsets[b], e = F.offsets[b + 1];
    if (b == 0 && s != 0) err |= kLookupBadOffsets;
    if (b + 1 == F.bag_count && e != F.key_count) err |= kLookupBadOffsets;
    if (s > e || e > F.key_count) { err |= kLookupBadOffsets; s = e = 0; }
    unsigned long long len = e - s;
    if (F.lengths) {
      const unsigned long long given = F.lengths[b];
      if (given < len) err |= kLookupShortLength;
      len = given;
    }
    const float* state = F.state;
    const unsigned long long row_stride = 3ull * D;
    const bool sequence = F.pooling == 2;

    float acc[C];
#pragma unroll
    for (int k = 0; k < C; ++k) acc[k] = 0.0f;

    for (unsigned long long c0 = s; c0 < e; c0 += 32) {
      const unsigned long long i = c0 + lane;
      const bool valid = i < e;
      unsigned long long slot = ~0ull;
      if (valid) {
        const unsigned long long key = F.keys[i];
        unsigned long long sl, sh;
        if (p.shard_count == 1) { sl = key; sh = 0; }
        else { sl = key / p.shard_count; sh = key - sl * p.shard_count; }
        if (sh == p.shard_id && sl < F.rows) slot = sl;
        else err |= kLookupBadKey;
        if (p.emit) {
          const unsigned long long o = F.occ_base + i;
          const KeyT ck = (slot == ~0ull) ? KeyT(0)
              : (KeyT(F.table_rank) << p.slot_bits) | KeyT(slot);
          static_cast<KeyT*>(p.occ_key)[o] = ck;
          p.occ_src[o] = (F.feature_index << kRowBits) |
                         (unsigned)(sequence ? i : b);
          if (sequence) p.row_scale[F.scale_base + i] = 1.0f;
        }
      }
      const int cnt = (int)min(32ull, e - c0);
      for (int j0 = 0; j0 < cnt; j0 += 4) {
        float r[4][C];
        unsigned long long sl[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          sl[u] = __shfl_sync(0xffffffffu, slot, (j0 + u) & 31);
          const bool use = (j0 + u < cnt) && sl[u] != ~0ull;
#pragma unroll
          for (int it = 0; it < ITERS; ++it) {
            const unsigned col = (it * 32 + lane) * VEC;
            float t[VEC];
            if (use && col < D) load_vec<VEC>(state + sl[u] * row_stride + col, t);
            else {
#pragma unroll
              for (int v = 0; v < VEC; ++v) t[v] = 0.0f;
            }
#pragma unroll
            for (int v = 0; v < VEC; ++v) r[u][it * VEC + v] = t[v];
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const bool use = (j0 + u < cnt) && sl[u] != ~0ull;
          if (!use) continue;
          if (sequence) {
            // one output row per position: 0 + w (batch_access.cpp:74-76)
            const unsigned long long pos = c0 + j0 + u;
#pragma unroll
            for (int it = 0; it < ITERS; ++it) {
              const unsigned col = (it * 32 + lane) * VEC;
              if (col >= D) continue;
              float t[VEC];
#pragma unroll
              for (int v = 0; v < VEC; ++v) t[v] = __fadd_rn(0.0f, r[u][it * VEC + v]);
              store_vec<VEC>(F.out + pos * D + col, t);
            }
          } else {
#pragma unroll
            for (int k = 0; k < C; ++k) acc[k] = __fadd_rn(acc[k], r[u][k]);
          }
        }
      }
    }
    if (!sequence) {
      const bool mean = F.pooling == 1;
      const float denom = (float)len;   // u64 -> float, round to nearest
#pragma unroll
      for (int it = 0; it < ITERS; ++it) {
        const unsigned col = (it * 32 + lane) * VEC;
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
        store_vec<VEC>(F.out + b * D + col, t);
      }
      if (p.emit && lane == 0)
        p.row_scale[F.scale_base + b] = (mean && len) ? __fdiv_rn(1.0f, denom) : 1.0f;
    }
  }
  // one atomic per warp at most
  err = __reduce_or_sync(0xffffffffu, err);
  if (err && lane == 0) atomicOr(p.error, err);
}

template <int VEC, int ITERS>
cudaError_t launch_key(const LookupLaunch& p, cudaStream_t s, unsigned grid) {
  if (p.key64) lookup_kernel<VEC, ITERS, unsigned long long><<<grid, 256, 0, s>>>(p);
  else lookup_kernel<VEC, ITERS, unsigned int><<<grid, 256, 0, s>>>(p);
  return cudaGetLastError();
}

template <int VEC>
cudaError_t launch_iters(const LookupLaunch& p, cudaStream_t s, unsigned grid) {
  switch (p.iters) {
    case 1: return launch_key<VEC, 1>(p, s, grid);
    case 2: return launch_key<VEC, 2>(p, s, grid);
    default: return launch_key<VEC, 4>(p, s, grid);
  }
}
}  // namespace

cudaError_t launch_lookup(const LookupLaunch& p, cudaStream_t stream) {
  if (p.bag_total == 0) return cudaSuccess;
  const unsigned long long want = (p.bag_total + 7) / 8;
  const unsigned grid = (unsigned)(want < 148ull * 16 ? want : 148ull * 16);
  switch (p.vec) {
    case 4: return launch_iters<4>(p, stream, grid);
    case 2: return launch_iters<2>(p, stream, grid);
    default: return launch_iters<1>(p, stream, grid);
  }
}

}  // namespace eps_b200
