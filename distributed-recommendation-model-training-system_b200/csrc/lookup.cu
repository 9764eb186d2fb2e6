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
// is read with one 128-bit load per lane) owns one work unit at a time -- one
// long bag, G consecutive short bags (walked as one run of keys, rows loaded
// back to back across bag boundaries) or 256 positions of a sequence feature;
// a warp holds 32/G groups.  The group fetches G keys with one coalesced load
// (the next chunk's keys are requested before the current chunk's rows),
// broadcasts the slots by shuffle and issues up to DEPTH row loads back to back
// before the dependent adds.  Rows past the end of a chunk are added as -0.0f, the additive identity
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
#ifndef EPS_LOOKUP_GRID_PER_SM
#define EPS_LOOKUP_GRID_PER_SM (EPS_LOOKUP_MIN_BLOCKS * 4)   // blocks per SM in the grid (4 waves)
#endif

template <int G, int VEC, int ITERS, typename KeyT>
__global__ void __launch_bounds__(256, EPS_LOOKUP_MIN_BLOCKS) lookup_kernel(LookupLaunch p) {
  __shared__ unsigned long long s_unit_base[kMaxFeatures + 1];
  const unsigned fc = p.feature_count;
  for (unsigned i = threadIdx.x; i < fc; i += blockDim.x) s_unit_base[i] = p.features[i].unit_base;
  if (threadIdx.x == 0) s_unit_base[fc] = p.unit_total;
  __syncthreads();

  const auto grp = cg::tiled_partition<G>(cg::this_thread_block());
  const unsigned gl = grp.thread_rank();
  const unsigned long long gid = (blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x) / G;
  const unsigned long long ngroups = (gridDim.x * (unsigned long long)blockDim.x) / G;
  constexpr int C = VEC * ITERS;
  constexpr int DEPTH = G < EPS_LOOKUP_DEPTH_REGS / C ? G : EPS_LOOKUP_DEPTH_REGS / C;
  static_assert(G >= (int)kUnitBags, "a lane per bag of a unit");
  unsigned int err = 0;

  for (unsigned long long u = gid; u < p.unit_total; u += ngroups) {
    // feature owning unit u: largest f with unit_base[f] <= u
    unsigned lo = 0, hi = fc;
    while (hi - lo > 1) { const unsigned mid = (lo + hi) >> 1; if (s_unit_base[mid] <= u) lo = mid; else hi = mid; }
    const LookupFeature* F = p.features + lo;
    const unsigned long long lu = u - s_unit_base[lo];
    const unsigned long long key_count = F->key_count, B = F->bag_count;
    const unsigned long long* const keys = F->keys;
    const float* const state = F->state;
    float* const out = F->out;
    const unsigned D = F->dim;
    const unsigned long long rows = F->rows;
    const unsigned long long row_stride = 3ull * D;
    const bool sequence = F->pooling == 2;
    // padding keys (PrepareAdapterInput, src/access/prepare_queue.cpp:69-77) are
    // dropped: no row, no gradient; mean bags divide by the kept count and
    // sequence positions holding padding read as zeros
    const bool has_pad = F->has_padding != 0;
    const unsigned long long pad_key = F->padding_key;

    // the unit's bags (pooled: unit_bags bags; sequence: one run of up to
    // kUnitPositions positions), lane k holding bag k's first occurrence and end
    // (32-bit: a feature holds fewer than 2^31 keys)
    unsigned long long b0 = 0;
    unsigned s_mine = 0, e_mine = 0, nb = 0;
    if (sequence) {
      b0 = lu * kUnitPositions;
      nb = b0 < key_count ? 1u : 0u;
      s_mine = (unsigned)b0;
      e_mine = nb ? (unsigned)min(key_count, b0 + kUnitPositions) : (unsigned)b0;
      // this unit's span of offsets (a sequence feature's bags do not shape its outputs)
#pragma unroll 1
      for (unsigned q = gl; q < kUnitPositions; q += G) {
        const unsigned long long i = b0 + q;
        if (B > 0 && i <= B) {
          const unsigned long long o = F->offsets[i];
          if (i == 0 && o != 0) err |= kLookupBadOffsets;
          if (i == B && o != key_count) err |= kLookupBadOffsets;
          if (o > key_count || (i > 0 && F->offsets[i - 1] > o)) err |= kLookupBadOffsets;
        }
      }
    } else {
      b0 = lu * F->unit_bags;
      nb = (unsigned)min((unsigned long long)F->unit_bags, B - b0);
      if (gl < nb) {
        const unsigned long long b = b0 + gl;
        unsigned long long s = F->offsets[b], e = F->offsets[b + 1];
        if (b == 0 && s != 0) err |= kLookupBadOffsets;
        if (b + 1 == B && e != key_count) err |= kLookupBadOffsets;
        if (s > e || e > key_count) { err |= kLookupBadOffsets; s = e = 0; }
        s_mine = (unsigned)s;
        e_mine = (unsigned)e;
      }
    }
    if (!sequence && F->unit_bags > 1) {
      // short bags: the unit's keys [S, E) walked as one run in position order,
      // DEPTH rows in flight across bag boundaries.  Bag `cur`'s sum is stored
      // when the run reaches its end: the adds per bag stay in position order,
      // so the sums equal the per-bag loop's.  Everything here is uniform over
      // the group (positions, bag ends and slots come by shuffle).
      const unsigned S = grp.shfl(s_mine, 0);
      const unsigned E = grp.shfl(e_mine, (nb - 1) & (G - 1));
      unsigned cur = 0, kept = 0;
      unsigned e_cur = grp.shfl(e_mine, 0);
      float acc[C];
#pragma unroll
      for (int q = 0; q < C; ++q) acc[q] = 0.0f;
      auto close_bag = [&]() {
        const unsigned long long b = b0 + cur;
        const unsigned s_cur = grp.shfl(s_mine, cur & (G - 1));
        unsigned long long len = has_pad ? kept : (unsigned long long)(e_cur - s_cur);
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
#pragma unroll
        for (int q = 0; q < C; ++q) acc[q] = 0.0f;
        kept = 0;
        ++cur;
        e_cur = grp.shfl(e_mine, cur & (G - 1));
      };
      unsigned long long key = (S + gl < E) ? keys[S + gl] : 0ull;
#pragma unroll 1
      for (unsigned c0 = S; c0 < E; c0 += G) {
        const unsigned i = c0 + gl;
        unsigned slot = ~0u;
        if (i < E && has_pad && key == pad_key) {
          slot = kPadSlot;
        } else if (i < E && F->slots) {
          const unsigned hs = F->slots[i];
          if (hs < kPadSlot) slot = hs;
          else err |= kLookupBadKey;
        } else if (i < E) {
          unsigned long long sl, sh;
          if (p.shard_count == 1) { sl = key; sh = 0; }
          else { sl = key / p.shard_count; sh = key - sl * p.shard_count; }
          if (sh == p.shard_id && sl < rows) slot = (unsigned)sl;
          else err |= kLookupBadKey;
        }
        if (i + G < E) key = keys[i + G];   // the next chunk's keys in flight
        const int cnt = (int)min((unsigned)G, E - c0);
#pragma unroll 1
        for (int j0 = 0; j0 < cnt; j0 += DEPTH) {
          float r[DEPTH][C];
          bool use[DEPTH];
#pragma unroll
          for (int uu = 0; uu < DEPTH; ++uu) {
            const unsigned su = grp.shfl(slot, (j0 + uu) & (G - 1));
            use[uu] = (j0 + uu < cnt) && su < kPadSlot;
            const float* row = state + (unsigned long long)su * row_stride;
#pragma unroll
            for (int it = 0; it < ITERS; ++it) {
              const unsigned col = (it * G + gl) * VEC;
              float t[VEC];
              if (use[uu] && col < D) load_vec<VEC>(row + col, t);
              else {
#pragma unroll
                for (int v = 0; v < VEC; ++v) t[v] = -0.0f;
              }
#pragma unroll
              for (int v = 0; v < VEC; ++v) r[uu][it * VEC + v] = t[v];
            }
          }
#pragma unroll
          for (int uu = 0; uu < DEPTH; ++uu) {
            if (j0 + uu >= cnt) break;
            const unsigned pos = c0 + (unsigned)(j0 + uu);
            while (cur < nb && pos >= e_cur) close_bag();
            if (cur < nb) {
#pragma unroll
              for (int q = 0; q < C; ++q) acc[q] = __fadd_rn(acc[q], r[uu][q]);
              kept += use[uu] ? 1u : 0u;
            }
          }
        }
      }
      while (cur < nb) close_bag();      // bags ending at E, empty bags included
      continue;
    }
    unsigned s = grp.shfl(s_mine, 0), e = grp.shfl(e_mine, 0);
    unsigned long long key = (s + gl < e) ? keys[s + gl] : 0ull;
#pragma unroll 1
    for (unsigned k = 0; k < nb; ++k) {
      // bag k's range [s, e); its first chunk's keys were requested before
      float acc[C];
#pragma unroll
      for (int q = 0; q < C; ++q) acc[q] = 0.0f;
      unsigned kept = 0;
      if (s == e && k + 1 < nb) {
        const unsigned ns = grp.shfl(s_mine, (k + 1) & (G - 1));
        const unsigned ne = grp.shfl(e_mine, (k + 1) & (G - 1));
        key = (ns + gl < ne) ? keys[ns + gl] : 0ull;
      }
#pragma unroll 1
      for (unsigned c0 = s; c0 < e; c0 += G) {
        const unsigned i = c0 + gl;
        unsigned slot = ~0u;              // slots fit 32 bits: rows < 2^32 - 2 per shard
        if (i < e && has_pad && key == pad_key) {
          slot = kPadSlot;
        } else if (i < e && F->slots) {
          const unsigned hs = F->slots[i];      // a hashed table's resolved slot
          if (hs < kPadSlot) slot = hs;
          else err |= kLookupBadKey;
        } else if (i < e) {
          unsigned long long sl, sh;
          if (p.shard_count == 1) { sl = key; sh = 0; }
          else { sl = key / p.shard_count; sh = key - sl * p.shard_count; }
          if (sh == p.shard_id && sl < rows) slot = (unsigned)sl;
          else err |= kLookupBadKey;
        }
        // the next chunk's keys -- of this bag, or of the next one -- in flight
        // while this chunk's rows load
        if (c0 + G < e) {
          if (i + G < e) key = keys[i + G];
        } else if (k + 1 < nb) {
          const unsigned ns = grp.shfl(s_mine, (k + 1) & (G - 1));
          const unsigned ne = grp.shfl(e_mine, (k + 1) & (G - 1));
          key = (ns + gl < ne) ? keys[ns + gl] : 0ull;
        }
        const int cnt = (int)min((unsigned)G, e - c0);
        if (has_pad) kept += __popc(grp.ballot(i < e && slot != kPadSlot));
#pragma unroll 1
        for (int j0 = 0; j0 < cnt; j0 += DEPTH) {
          float r[DEPTH][C];
          bool use[DEPTH], padrow[DEPTH];
#pragma unroll
          for (int uu = 0; uu < DEPTH; ++uu) {
            const unsigned su = grp.shfl(slot, (j0 + uu) & (G - 1));
            padrow[uu] = (j0 + uu < cnt) && su == kPadSlot;
            use[uu] = (j0 + uu < cnt) && su < kPadSlot;
            const float* row = state + (unsigned long long)su * row_stride;
#pragma unroll
            for (int it = 0; it < ITERS; ++it) {
              const unsigned col = (it * G + gl) * VEC;
              float t[VEC];
              if (use[uu] && col < D) load_vec<VEC>(row + col, t);
              else {
#pragma unroll
                for (int v = 0; v < VEC; ++v) t[v] = -0.0f;
              }
#pragma unroll
              for (int v = 0; v < VEC; ++v) r[uu][it * VEC + v] = t[v];
            }
          }
          if (sequence) {
            // one output row per position: 0 + w (batch_access.cpp:74-76)
#pragma unroll
            for (int uu = 0; uu < DEPTH; ++uu) {
              if (!use[uu] && !padrow[uu]) continue;
              const unsigned long long pos = (unsigned long long)(c0 + j0 + uu);
#pragma unroll
              for (int it = 0; it < ITERS; ++it) {
                const unsigned col = (it * G + gl) * VEC;
                if (col >= D) continue;
                float t[VEC];
#pragma unroll
                for (int v = 0; v < VEC; ++v) t[v] = padrow[uu] ? 0.0f : __fadd_rn(0.0f, r[uu][it * VEC + v]);
                store_vec<VEC>(out + pos * D + col, t);
              }
            }
          } else {
            // position order; -0.0f padding leaves acc unchanged
#pragma unroll
            for (int uu = 0; uu < DEPTH; ++uu)
#pragma unroll
              for (int q = 0; q < C; ++q) acc[q] = __fadd_rn(acc[q], r[uu][q]);
          }
        }
      }
      if (!sequence) {
        const unsigned long long b = b0 + k;
        unsigned long long len = has_pad ? kept : (unsigned long long)(e - s);
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
      s = grp.shfl(s_mine, (k + 1) & (G - 1));
      e = grp.shfl(e_mine, (k + 1) & (G - 1));
    }
  }
  err = cg::reduce(grp, err, cg::bit_or<unsigned>());
  if (err && gl == 0) atomicOr(p.error, err);
}

// Occurrence list of a lookup that will be pushed, ahead of (and independent
// of) the gather, so that the coalescing sort can run concurrently with the
// gather: every occurrence's composite key (table rank, slot) and gradient
// source (feature, bag or position), and the gradient row scales (1.0f / valid
// length for mean, src/access/batch_access.cpp:107-108).  Validation matches the
// gather kernel's.
//
// One warp per emit unit (LookupFeature::emit_units), 32 occurrences per step:
// a pooled unit is kUnitBags consecutive bags of a long-bag feature, or
// kEmitShortBags of a short-bag one -- their offsets are read once, and lane j of
// a step finds its bag among them -- and a sequence unit is
// kUnitPositions consecutive positions plus the same span of offsets, which it
// validates (a sequence feature's bags do not shape its outputs).  So neither a
// very long bag nor many one-key bags serialise on one warp.
constexpr int kEmitSteps = 4;   // 32-entry steps whose keys load together

template <typename KeyT>
__global__ void __launch_bounds__(256, 4) emit_kernel(LookupLaunch p) {
  __shared__ unsigned long long s_unit_base[kMaxFeatures + 1];
  __shared__ unsigned s_kept[8][kEmitShortBags];
  __shared__ unsigned s_hist[8][256];   // the sort's digit histograms, block part
  const unsigned fc = p.feature_count;
  const unsigned passes = p.digit_hist ? p.digit_passes : 0u;
  for (unsigned i = threadIdx.x; i < fc; i += blockDim.x) s_unit_base[i] = p.features[i].emit_base;
  for (unsigned i = threadIdx.x; i < passes * 256u; i += blockDim.x) (&s_hist[0][0])[i] = 0;
  if (threadIdx.x == 0) s_unit_base[fc] = p.emit_total;
  __syncthreads();
  // the sort's digits of a key this lane wrote (shared-memory atomics; warp
  // aggregation by __match_any_sync, or a vote for digits shared by the whole
  // step, measured slower on every config)
  auto count_digits = [&](KeyT ck, bool valid) {
    if (valid)
      for (unsigned q = 0; q < passes; ++q) atomicAdd(&s_hist[q][(unsigned)(ck >> (8 * q)) & 255u], 1u);
  };


  const unsigned lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const unsigned long long warp = (blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x) >> 5;
  const unsigned long long nwarps = (gridDim.x * (unsigned long long)blockDim.x) >> 5;
  unsigned err = 0;
  for (unsigned long long u = warp; u < p.emit_total; u += nwarps) {
    unsigned lo = 0, hi = fc;
    while (hi - lo > 1) { const unsigned mid = (lo + hi) >> 1; if (s_unit_base[mid] <= u) lo = mid; else hi = mid; }
    const LookupFeature* F = p.features + lo;
    const unsigned long long lu = u - s_unit_base[lo];
    const unsigned long long key_count = F->key_count, B = F->bag_count;
    const bool has_pad = F->has_padding != 0;
    const unsigned long long pad_key = F->padding_key;
    const unsigned long long rows = F->rows, occ_base = F->occ_base;
    const unsigned src_hi = F->feature_index << kRowBits;
    const KeyT rank_bits = KeyT(F->table_rank) << p.slot_bits;
    // composite key of occurrence `idx` (its key `key`); pad / bad reported
    // through the flags; a hashed table's slot was resolved before
    auto composite = [&](unsigned long long key, unsigned long long idx, bool* pad) -> KeyT {
      *pad = false;
      if (has_pad && key == pad_key) { *pad = true; return KeyT(p.pad_key); }
      if (F->slots) {
        const unsigned hs = F->slots[idx];
        if (hs < kPadSlot) return rank_bits | KeyT(hs);
        err |= kLookupBadKey;
        return KeyT(0);
      }
      unsigned long long sl, sh;
      if (p.shard_count == 1) { sl = key; sh = 0; }
      else { sl = key / p.shard_count; sh = key - sl * p.shard_count; }
      if (sh == p.shard_id && sl < rows) return rank_bits | KeyT(sl);
      err |= kLookupBadKey;
      return KeyT(0);
    };
    if (F->pooling == 2) {
      // positions [lu * kUnitPositions, ...) and the offsets with the same indices;
      // every slice's keys are requested before the first store (a store might
      // alias the keys, so the compiler would not move a later load above it)
      const unsigned long long base = lu * kUnitPositions;
      unsigned long long kq[kUnitSlices];
#pragma unroll
      for (unsigned q = 0; q < kUnitSlices; ++q) {
        const unsigned long long i = base + q * 32 + lane;
        kq[q] = i < key_count ? F->keys[i] : 0ull;
      }
#pragma unroll
      for (unsigned q = 0; q < kUnitSlices; ++q) {
        const unsigned long long i = base + q * 32 + lane;
        KeyT ck = KeyT(0);
        if (i < key_count) {
          bool pad;
          ck = composite(kq[q], i, &pad);
          static_cast<KeyT*>(p.occ_key)[occ_base + i] = ck;
          p.occ_src[occ_base + i] = src_hi | (unsigned)i;
          p.row_scale[F->scale_base + i] = 1.0f;
        }
        count_digits(ck, i < key_count);
        if (B > 0 && i <= B) {
          const unsigned long long o = F->offsets[i];
          if (i == 0 && o != 0) err |= kLookupBadOffsets;
          if (i == B && o != key_count) err |= kLookupBadOffsets;
          if (o > key_count || (i > 0 && F->offsets[i - 1] > o)) err |= kLookupBadOffsets;
        }
      }
      continue;
    }
    // pooled: bags b0 .. b0 + nb - 1 (ub <= 32 bags per unit, lane k holding bag k)
    const unsigned ub = emit_unit_bags(key_count, B);
    const unsigned long long b0 = lu * ub;
    const unsigned nb = (unsigned)min((unsigned long long)ub, B - b0);
    unsigned long long s = 0, e = 0;
    unsigned n = 0;
    if (lane < nb) {
      const unsigned long long b = b0 + lane;
      s = F->offsets[b];
      e = F->offsets[b + 1];
      if (b == 0 && s != 0) err |= kLookupBadOffsets;
      if (b + 1 == B && e != key_count) err |= kLookupBadOffsets;
      if (s > e || e > key_count) { err |= kLookupBadOffsets; s = e = 0; }
      n = (unsigned)(e - s);
    }
    unsigned incl = n;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const unsigned y = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= (unsigned)d) incl += y;
    }
    const unsigned total = __shfl_sync(0xffffffffu, incl, 31);
    const unsigned excl = incl - n;       // bag's first entry in the unit's run
    s_kept[w][lane] = 0;
    __syncwarp();
    // kEmitSteps steps of 32 entries at a time: their keys are requested
    // before the first store (see the sequence branch)
#pragma unroll 1
    for (unsigned c0 = 0; c0 < total; c0 += 32 * kEmitSteps) {
      unsigned long long kq[kEmitSteps];
      unsigned occ[kEmitSteps], kb[kEmitSteps];   // a feature holds fewer than 2^31 keys
#pragma unroll
      for (int q = 0; q < kEmitSteps; ++q) {
        const unsigned i = c0 + q * 32 + lane;
        // bag of entry i: the last bag whose first entry is <= i (binary lifting
        // over the lanes' non-decreasing first entries; bag 0's is 0)
        unsigned k = 0;
        for (unsigned step = ub >> 1; step; step >>= 1) {
          const unsigned ek = __shfl_sync(0xffffffffu, excl, k + step);
          if (k + step < nb && ek <= i) k += step;
        }
        const unsigned long long sk = __shfl_sync(0xffffffffu, s, k);
        const unsigned ek = __shfl_sync(0xffffffffu, excl, k);
        kb[q] = k;
        occ[q] = (unsigned)(sk + (i - ek));
        kq[q] = i < total ? F->keys[occ[q]] : 0ull;
      }
#pragma unroll
      for (int q = 0; q < kEmitSteps; ++q) {
        const bool valid = c0 + q * 32 + lane < total;
        KeyT ck = KeyT(0);
        if (valid) {
          bool pad;
          ck = composite(kq[q], occ[q], &pad);
          static_cast<KeyT*>(p.occ_key)[occ_base + occ[q]] = ck;
          p.occ_src[occ_base + occ[q]] = src_hi | (unsigned)(b0 + kb[q]);
          if (has_pad && !pad) atomicAdd(&s_kept[w][kb[q]], 1u);
        }
        count_digits(ck, valid);
      }
    }
    __syncwarp();
    if (lane < nb) {
      unsigned long long len = has_pad ? s_kept[w][lane] : n;
      if (F->lengths) {
        const unsigned long long given = F->lengths[b0 + lane];
        if (given < len) err |= kLookupShortLength;
        len = given;
      }
      const bool mean = F->pooling == 1;
      p.row_scale[F->scale_base + b0 + lane] = (mean && len) ? __fdiv_rn(1.0f, (float)len) : 1.0f;
    }
    __syncwarp();
  }
  err = __reduce_or_sync(~0u, err);
  if (err && lane == 0) atomicOr(p.error, err);
  if (passes) {
    __syncthreads();
    for (unsigned i = threadIdx.x; i < passes * 256u; i += blockDim.x) {
      const unsigned c = (&s_hist[0][0])[i];
      if (c) atomicAdd(p.digit_hist + i, c);
    }
  }
}

template <int G, int VEC, int ITERS>
cudaError_t launch_key(const LookupLaunch& p, cudaStream_t s) {
  const unsigned long long groups_per_block = 256 / G;
  const unsigned long long want = (p.unit_total + groups_per_block - 1) / groups_per_block;
  const unsigned long long cap = 148ull * EPS_LOOKUP_GRID_PER_SM;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  if (p.key64) lookup_kernel<G, VEC, ITERS, unsigned long long><<<grid, 256, 0, s>>>(p);
  else lookup_kernel<G, VEC, ITERS, unsigned int><<<grid, 256, 0, s>>>(p);
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_emit(const LookupLaunch& p, cudaStream_t stream) {
  if (p.emit_total == 0) return cudaSuccess;
  const unsigned long long want = (p.emit_total + 7) / 8;
  const unsigned grid = (unsigned)(want < 148ull * 8 * 2 ? want : 148ull * 8 * 2);
  if (p.key64) emit_kernel<unsigned long long><<<grid, 256, 0, stream>>>(p);
  else emit_kernel<unsigned int><<<grid, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_lookup(const LookupLaunch& p, cudaStream_t stream) {
  if (p.unit_total == 0) return cudaSuccess;
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
