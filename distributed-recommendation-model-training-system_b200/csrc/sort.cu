// sort.cu -- stable least-significant-digit radix sort of (composite key, source)
// pairs: the id-coalescing step of a Push.
//
// The reference coalesces duplicate ids with a hash map that keeps the first
// occurrence order of unique rows and the occurrence order inside each row
// (src/access/batch_access.cpp:99-121).  A STABLE sort by key keeps exactly
// that per-row occurrence order, so every coalesced row receives the same
// ordered list of (gradient row, scale) references as in the reference.  The
// order of the unique rows themselves is not observable in the resulting state.
//
// Single-pass-per-digit ("onesweep") design, 8-bit digits:
//   1. one histogram kernel computes the global digit counts of EVERY pass in a
//      single read of the keys (digit counts do not depend on the order);
//   2. per pass, one kernel: each CTA takes the next tile in launch order from an
//      atomic counter, ranks its 4096 items stably (warp-private running counts
//      with __match_any_sync), publishes its per-digit counts, obtains the
//      exclusive prefix of all earlier tiles by decoupled look-back over their
//      published (flag, count) words, and scatters.
// A tile only waits for tiles taken earlier, whose CTAs are already running and
// publish their counts before they wait themselves, so every wait ends; each
// wait is nevertheless bounded, and a wait that runs out records an error that
// rejects the dependent push instead of hanging.
#include "kernels.cuh"

#ifndef EPS_HIST_BLOCKS_PER_SM
#define EPS_HIST_BLOCKS_PER_SM 4      // histogram blocks per SM: each flushes its counts
                                      // with global atomics (cfg2: 8 -> 4 blocks, 15.3 -> 10.7 us)
#endif

namespace eps_b200 {
namespace {
constexpr int kThreads = 256;
constexpr int kItems = 16;
constexpr int kSortTile = kThreads * kItems;       // 4096 items per tile
constexpr int kWarps = kThreads / 32;
constexpr int kWarpSpan = kSortTile / kWarps;      // 512 items per warp
constexpr unsigned long long kFlagAggregate = 1ull << 32;
constexpr unsigned long long kFlagPrefix = 2ull << 32;
constexpr unsigned kSpinLimit = 1u << 22;

// Global digit histograms of all passes: hist[pass][256] (a lookup's emit kernel
// counts them as it writes the keys; this kernel serves the other sorts).
template <typename KeyT>
__global__ void __launch_bounds__(kThreads) digit_histograms(const KeyT* keys, unsigned long long n,
                                                             unsigned passes, unsigned* hist) {
  __shared__ unsigned s_hist[8][256];
  for (unsigned i = threadIdx.x; i < 8 * 256; i += kThreads) (&s_hist[0][0])[i] = 0;
  __syncthreads();
  for (unsigned long long i = blockIdx.x * (unsigned long long)kThreads + threadIdx.x; i < n;
       i += (unsigned long long)gridDim.x * kThreads) {
    const KeyT k = keys[i];
    for (unsigned p = 0; p < passes; ++p) atomicAdd(&s_hist[p][(unsigned)(k >> (8 * p)) & 255u], 1u);
  }
  __syncthreads();
  for (unsigned i = threadIdx.x; i < passes * 256; i += kThreads) {
    const unsigned c = (&s_hist[0][0])[i];
    if (c) atomicAdd(hist + i, c);
  }
}

// Order-preserving compaction of segment heads of the sorted keys:
// seg_start[u] = position of the u-th run of equal keys, seg_start[U] = n,
// *seg_total = U, over tiles of 4096 positions (16 consecutive per thread).
// Segment heads without a look-back chain, for up to kDirectTiles tiles: the
// first launch counts each tile's run heads, the second gives every tile the
// sum of its predecessors' counts (read directly, at most kDirectTiles values)
// and writes its heads' positions.  The look-back kernel below serves larger
// inputs: with every tile of a one-wave grid running at once, its prefix
// frontier crosses the tiles only a few at a time.
constexpr unsigned kDirectTiles = 4096;

template <typename KeyT>
__device__ __forceinline__ unsigned tile_head_flags(const KeyT* keys, unsigned long long n,
                                                    unsigned long long base) {
  unsigned flags = 0;
  if (base < n) {
    KeyT prev = base > 0 ? keys[base - 1] : KeyT(0);
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      const unsigned long long i = base + j;
      if (i < n) {
        const KeyT k = keys[i];
        if (i == 0 || k != prev) flags |= 1u << j;
        prev = k;
      }
    }
  }
  return flags;
}

template <typename KeyT>
__global__ void __launch_bounds__(kThreads) segment_counts(const KeyT* keys, unsigned long long n,
                                                           unsigned* tile_cnt) {
  __shared__ unsigned s_warp[kWarps];
  const unsigned w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned long long base = (unsigned long long)blockIdx.x * kSortTile + threadIdx.x * kItems;
  const unsigned c = __reduce_add_sync(0xffffffffu, (unsigned)__popc(tile_head_flags(keys, n, base)));
  if (lane == 0) s_warp[w] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned t = 0;
#pragma unroll
    for (int q = 0; q < kWarps; ++q) t += s_warp[q];
    tile_cnt[blockIdx.x] = t;
  }
}

template <typename KeyT>
__global__ void __launch_bounds__(kThreads) segment_write(const KeyT* keys, unsigned long long n,
                                                          const unsigned* tile_cnt,
                                                          unsigned* seg_start, unsigned* seg_total) {
  __shared__ unsigned s_warp[kWarps], s_pre[kWarps];
  const unsigned w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned tile = blockIdx.x;
  // heads of the earlier tiles
  unsigned part = 0;
  for (unsigned t = threadIdx.x; t < tile; t += kThreads) part += tile_cnt[t];
  part = __reduce_add_sync(0xffffffffu, part);
  const unsigned long long base = (unsigned long long)tile * kSortTile + threadIdx.x * kItems;
  unsigned flags = tile_head_flags(keys, n, base);
  const unsigned cnt = __popc(flags);
  unsigned x = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= (unsigned)o) x += y;
  }
  if (lane == 31) s_warp[w] = x;
  if (lane == 0) s_pre[w] = part;
  __syncthreads();
  unsigned before = 0, total = 0, prefix = 0;
#pragma unroll
  for (int q = 0; q < kWarps; ++q) {
    if ((unsigned)q < w) before += s_warp[q];
    total += s_warp[q];
    prefix += s_pre[q];
  }
  unsigned r = prefix + before + x - cnt;
  while (flags) {
    const int j = __ffs(flags) - 1;
    flags &= flags - 1;
    seg_start[r++] = (unsigned)(base + j);
  }
  const unsigned long long tiles = (n + kSortTile - 1) / kSortTile;
  if (tile == tiles - 1 && threadIdx.x == 0) {
    seg_start[prefix + total] = (unsigned)n;
    *seg_total = prefix + total;
  }
}

// The look-back variant: tiles taken in launch order; a warp-wide look-back
// reads 32 predecessors per step.
template <typename KeyT>
__global__ void __launch_bounds__(kThreads) segment_heads(const KeyT* keys, unsigned long long n,
                                                          unsigned* seg_start, unsigned* seg_total,
                                                          unsigned long long* status,
                                                          unsigned* tile_counter, unsigned* error) {
  __shared__ unsigned s_tile, s_warp[kWarps], s_prefix;
  const unsigned w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) s_tile = atomicAdd(tile_counter, 1u);
  __syncthreads();
  const unsigned tile = s_tile;
  const unsigned long long base = (unsigned long long)tile * kSortTile + threadIdx.x * kItems;
  unsigned flags = 0;
  if (base < n) {
    KeyT prev = base > 0 ? keys[base - 1] : KeyT(0);
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      const unsigned long long i = base + j;
      if (i < n) {
        const KeyT k = keys[i];
        if (i == 0 || k != prev) flags |= 1u << j;
        prev = k;
      }
    }
  }
  const unsigned cnt = __popc(flags);
  unsigned x = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= (unsigned)o) x += y;
  }
  if (lane == 31) s_warp[w] = x;
  __syncthreads();
  unsigned before = 0, total = 0;
#pragma unroll
  for (int q = 0; q < kWarps; ++q) { if ((unsigned)q < w) before += s_warp[q]; total += s_warp[q]; }
  const unsigned excl = before + x - cnt;
  unsigned long long* mine = status + tile;
  if (w == 0) {
    unsigned prefix = 0;
    if (tile == 0) {
      if (lane == 0) __stcg(mine, kFlagPrefix | total);
    } else {
      if (lane == 0) __stcg(mine, kFlagAggregate | total);
      long long t = (long long)tile - 1;
      unsigned spins = 0;
      bool failed = false;
      while (t >= 0) {
        const long long tt = t - lane;
        const unsigned long long s = tt >= 0 ? __ldcg(status + tt) : kFlagPrefix;
        const unsigned flag = (unsigned)(s >> 32);
        const unsigned pref = __ballot_sync(0xffffffffu, flag == 2);
        const unsigned waiting = __ballot_sync(0xffffffffu, flag == 0);
        const int pl = pref ? __ffs(pref) - 1 : 32;
        const unsigned upto = pl >= 31 ? 0xffffffffu : ((2u << pl) - 1u);
        if (waiting & upto) {
          if (++spins > kSpinLimit) { failed = true; break; }
          __nanosleep(64);
          continue;
        }
        prefix += __reduce_add_sync(0xffffffffu, (unsigned)lane <= (unsigned)pl ? (unsigned)s : 0u);
        if (pl < 32) break;
        t -= 32;
      }
      if (failed && lane == 0) atomicOr(error, kLookupSortFailed);
      if (lane == 0) __stcg(mine, kFlagPrefix | (prefix + total));
    }
    if (lane == 0) s_prefix = prefix;
  }
  __syncthreads();
  unsigned r = s_prefix + excl;
  while (flags) {
    const int j = __ffs(flags) - 1;
    flags &= flags - 1;
    seg_start[r++] = (unsigned)(base + j);
  }
  const unsigned long long tiles = (n + kSortTile - 1) / kSortTile;
  if (tile == tiles - 1 && threadIdx.x == 0) {
    const unsigned U = s_prefix + total;
    seg_start[U] = (unsigned)n;
    *seg_total = U;
  }
}

template <typename KeyT>
struct OnesweepSmem {
  unsigned cnt[kWarps][256];     // warp-private digit counts, then warp offsets
  unsigned dig_off[256];         // tile-local exclusive prefix of the digit counts
  unsigned gbase[256];           // global position of tile position 0 of each digit
  unsigned warp_sum[kWarps];
  unsigned tile;
  KeyT keys[kSortTile];          // the tile in tile-sorted order
  unsigned vals[kSortTile];
};

// One digit pass: each CTA takes the next tile in launch order from an atomic
// counter, ranks its items stably (per warp: __match_any_sync groups the lanes
// with the same digit, a warp-private running count per digit orders the warp's
// rounds), publishes its per-digit counts, scatters the tile into shared memory
// in tile-sorted order while the exclusive prefix of the earlier tiles is
// obtained by decoupled look-back over their published (flag, count) words, and
// finally writes the tile out in tile-sorted order, so that consecutive threads
// write consecutive positions of each digit's run.
template <typename KeyT>
__global__ void __launch_bounds__(kThreads) onesweep_pass(const KeyT* kin, const unsigned* vin,
                                                          KeyT* kout, unsigned* vout,
                                                          unsigned long long n, unsigned shift,
                                                          const unsigned* hist,
                                                          unsigned long long* status,
                                                          unsigned* tile_counter,
                                                          unsigned* error) {
  extern __shared__ __align__(16) unsigned char os_raw[];
  OnesweepSmem<KeyT>& S = *reinterpret_cast<OnesweepSmem<KeyT>*>(os_raw);
  const unsigned w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (unsigned i = threadIdx.x; i < kWarps * 256; i += kThreads) (&S.cnt[0][0])[i] = 0;
  if (threadIdx.x == 0) S.tile = atomicAdd(tile_counter, 1u);
  __syncthreads();
  const unsigned tile = S.tile;
  const unsigned long long tbase = (unsigned long long)tile * kSortTile;
  const unsigned tcount = (unsigned)min((unsigned long long)kSortTile, n - tbase);
  const unsigned long long base = tbase + w * kWarpSpan;
  const unsigned lt = (1u << lane) - 1u;
  KeyT k[kItems];
  unsigned v[kItems], rank[kItems];
#pragma unroll
  for (int r = 0; r < kItems; ++r) {
    const unsigned long long idx = base + r * 32 + lane;
    const bool valid = idx < n;
    k[r] = valid ? kin[idx] : KeyT(0);
    v[r] = valid ? vin[idx] : 0u;
  }
  // stable rank of every item among the warp's earlier items with its digit
#pragma unroll
  for (int r = 0; r < kItems; ++r) {
    const bool valid = base + r * 32 + lane < n;
    const unsigned d = valid ? ((unsigned)(k[r] >> shift) & 255u) : 256u + lane;
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    unsigned prior = 0;
    if (valid) prior = S.cnt[w][d];
    __syncwarp();
    if (valid) {
      rank[r] = prior + __popc(peers & lt);
      if ((peers & lt) == 0) S.cnt[w][d] = prior + __popc(peers);
    }
    __syncwarp();
  }
  __syncthreads();
  // per digit (thread d): warp offsets, tile total, published aggregate
  const unsigned d = threadIdx.x;          // kThreads == 256 digits
  unsigned total = 0;
#pragma unroll
  for (int x = 0; x < kWarps; ++x) { const unsigned c = S.cnt[x][d]; S.cnt[x][d] = total; total += c; }
  unsigned long long* mine = status + (unsigned long long)tile * 256 + d;
  __stcg(mine, (tile == 0 ? kFlagPrefix : kFlagAggregate) | total);
  // tile-local and global exclusive digit prefixes (block scans over 256 digits)
  const unsigned hcount = hist[d];
  unsigned xt = total, xh = hcount;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned yt = __shfl_up_sync(0xffffffffu, xt, o);
    const unsigned yh = __shfl_up_sync(0xffffffffu, xh, o);
    if (lane >= (unsigned)o) { xt += yt; xh += yh; }
  }
  __shared__ unsigned s_wh[kWarps];
  if (lane == 31) { S.warp_sum[w] = xt; s_wh[w] = xh; }
  __syncthreads();
  unsigned bt = 0, bh = 0;
  for (unsigned q = 0; q < w; ++q) { bt += S.warp_sum[q]; bh += s_wh[q]; }
  const unsigned dig_off = bt + xt - total;
  const unsigned digit_base = bh + xh - hcount;
  S.dig_off[d] = dig_off;
  __syncthreads();
  // scatter the tile into shared memory in tile-sorted order
#pragma unroll
  for (int r = 0; r < kItems; ++r) {
    if (base + r * 32 + lane < n) {
      const unsigned dd = (unsigned)(k[r] >> shift) & 255u;
      const unsigned pos = S.dig_off[dd] + S.cnt[w][dd] + rank[r];
      S.keys[pos] = k[r];
      S.vals[pos] = v[r];
    }
  }
  // decoupled look-back over earlier tiles of this digit (8 predecessors per
  // step loaded together; every wait bounded)
  unsigned prefix = 0;
  if (tile > 0) {
    constexpr int W = 8;
    long long t = (long long)tile - 1;
    unsigned spins = 0;
    bool failed = false;
    while (t >= 0) {
      unsigned long long sw[W];
#pragma unroll
      for (int j = 0; j < W; ++j)
        sw[j] = (t - j >= 0) ? __ldcg(status + (unsigned long long)(t - j) * 256 + d) : (kFlagPrefix);
      int used = 0;
      bool done = false, not_ready = false;
#pragma unroll
      for (int j = 0; j < W; ++j) {
        if (done || not_ready) continue;
        const unsigned flag = (unsigned)(sw[j] >> 32);
        if (flag == 0) { not_ready = true; continue; }
        prefix += (unsigned)sw[j];
        ++used;
        if (flag == 2) done = true;
      }
      if (done) break;
      t -= used;
      if (not_ready) {
        if (++spins > kSpinLimit) { failed = true; break; }
        __nanosleep(64);
      }
    }
    if (failed) atomicOr(error, kLookupSortFailed);
    __stcg(mine, kFlagPrefix | (prefix + total));
  }
  S.gbase[d] = digit_base + prefix - dig_off;
  __syncthreads();
  // write out in tile-sorted order: runs of one digit land on consecutive
  // positions (the bound is a guard only: counts and ranks always agree)
  for (unsigned i = threadIdx.x; i < tcount; i += kThreads) {
    const KeyT kk = S.keys[i];
    const unsigned pos = S.gbase[(unsigned)(kk >> shift) & 255u] + i;
    if (pos < n) {
      kout[pos] = kk;
      vout[pos] = S.vals[i];
    }
  }
}

template <typename KeyT>
cudaError_t run_sort(const SortLaunch& p, cudaStream_t s, int* swapped) {
  KeyT* k0 = static_cast<KeyT*>(p.keys);
  KeyT* k1 = static_cast<KeyT*>(p.keys_alt);
  unsigned* v0 = p.vals;
  unsigned* v1 = p.vals_alt;
  *swapped = 0;
  if (p.n <= 1) return cudaSuccess;
  const unsigned passes = (p.bits + 7) / 8;
  // scratch: hist[passes][256] | counters[passes] | status[passes][tiles][256]
  unsigned* hist = p.scratch;
  unsigned* counters = hist + passes * 256;
  unsigned long long* status = reinterpret_cast<unsigned long long*>(
      reinterpret_cast<char*>(p.scratch) + sort_scratch_header(passes));
  // the caller hands over zeroed scratch (sort_scratch_bytes)
  if (!p.hist_ready) {
    const unsigned long long hist_grid = min(148ull * EPS_HIST_BLOCKS_PER_SM, (p.n + kThreads - 1) / kThreads);
    digit_histograms<KeyT><<<(unsigned)hist_grid, kThreads, 0, s>>>(k0, p.n, passes, hist);
  }
  const size_t smem = sizeof(OnesweepSmem<KeyT>);
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (!attr_set[dev & 63]) {
    e = cudaFuncSetAttribute(onesweep_pass<KeyT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr_set[dev & 63] = true;
  }
  for (unsigned pass = 0; pass < passes; ++pass) {
    onesweep_pass<KeyT><<<p.tiles, kThreads, smem, s>>>(
        k0, v0, k1, v1, p.n, pass * 8, hist + pass * 256,
        status + (unsigned long long)pass * p.tiles * 256, counters + pass, p.error);
    KeyT* tk = k0; k0 = k1; k1 = tk;
    unsigned* tv = v0; v0 = v1; v1 = tv;
    *swapped ^= 1;
  }
  return cudaGetLastError();
}

template <typename KeyT>
cudaError_t run_heads(const SegmentLaunch& p, cudaStream_t s) {
  if (p.n == 0) {
    return cudaMemsetAsync(p.seg_total, 0, sizeof(unsigned), s);
  }
  const unsigned tiles = (unsigned)((p.n + kSortTile - 1) / kSortTile);
  // the caller hands over zeroed scratch (segment_scratch_bytes)
  unsigned* counter = p.scratch;
  unsigned long long* status = reinterpret_cast<unsigned long long*>(
      reinterpret_cast<char*>(p.scratch) + 256);
  if (tiles <= kDirectTiles) {
    unsigned* tile_cnt = reinterpret_cast<unsigned*>(status);   // tiles x 8 bytes available
    segment_counts<KeyT><<<tiles, kThreads, 0, s>>>(static_cast<const KeyT*>(p.keys), p.n, tile_cnt);
    segment_write<KeyT><<<tiles, kThreads, 0, s>>>(static_cast<const KeyT*>(p.keys), p.n, tile_cnt,
                                                   p.seg_start, p.seg_total);
    return cudaGetLastError();
  }
  segment_heads<KeyT><<<tiles, kThreads, 0, s>>>(static_cast<const KeyT*>(p.keys), p.n,
                                                 p.seg_start, p.seg_total, status, counter,
                                                 p.error);
  return cudaGetLastError();
}
}  // namespace

// ------------------------------------------------------------------ row plan
// One thread per coalesced row u (a block takes 256 consecutive rows): rows[u]
// gets the row's key and, for a row with one occurrence, its gradient source
// and row scale.  A row with 2..long_run occurrences gets one piece covering
// all of them (reserved with one atomic per block), reduced in order by the
// piece kernel; a longer row reserves ceil(len / kPiece) contiguous pieces
// (its warp writes them) and a LongRecord.  Padding rows (table rank >=
// table_count) are skipped.
template <typename KeyT>
__global__ void __launch_bounds__(256) row_plan(PlanLaunch p) {
  __shared__ unsigned s_cnt[8];
  __shared__ unsigned s_base;
  const unsigned U = *(volatile const unsigned*)p.seg_total;
  const unsigned lane = threadIdx.x & 31u, w = threadIdx.x >> 5;
  const unsigned below = (1u << lane) - 1u;
  const KeyT* keys = static_cast<const KeyT*>(p.keys);
  for (unsigned long long base = blockIdx.x * 256ull; base < U; base += gridDim.x * 256ull) {
    const unsigned long long u = base + threadIdx.x;
    unsigned kind = 0;                    // 1 single, 2 multi, 3 long
    unsigned s0 = 0, len = 0;
    unsigned long long key = 0;
    RowRec r{0ull, 0u, kRowSkip};
    if (u < U) {
      s0 = p.seg_start[u];
      len = p.seg_start[u + 1] - s0;
      const KeyT K = keys[s0];
      const unsigned src = p.srcs[s0];
      key = (unsigned long long)K;
      r.key = key;
      // a source outside the lookup's features or rows can only come from an
      // invalid lookup (whose push is rejected): such rows are skipped
      const unsigned f = src >> kRowBits, gr = src & ((1u << kRowBits) - 1u);
      bool src_ok = f < p.feature_count;
      if (src_ok) {
        const LookupFeature& F = p.features[f];
        src_ok = gr < (F.pooling == 2 ? F.key_count : F.bag_count);
      }
      if ((unsigned)(K >> p.slot_bits) < p.table_count && src_ok) {
        if (len > p.long_run) {
          kind = 3;
        } else if (len == 1) {
          kind = 1;
          r.a = src;
          r.b = __float_as_uint(p.row_scale[p.features[f].scale_base + gr]);
        } else {
          kind = 2;
          r.b = kRowMulti | len;
        }
      }
    }
    const unsigned mm = __ballot_sync(0xffffffffu, kind == 2);
    if (lane == 0) s_cnt[w] = __popc(mm);
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned tot = 0;
      for (int q = 0; q < 8; ++q) tot += s_cnt[q];
      s_base = tot ? atomicAdd(&p.plan->piece_count, tot) : 0u;
    }
    __syncthreads();
    if (kind == 2) {
      unsigned piece = s_base + __popc(mm & below);
      for (unsigned q = 0; q < w; ++q) piece += s_cnt[q];
      r.a = piece;
      p.pieces[piece] = make_uint2(s0, len);
    }
    if (u < U) p.rows[u] = r;
    for (unsigned todo = __ballot_sync(0xffffffffu, kind == 3); todo; todo &= todo - 1u) {
      const int L = __ffs(todo) - 1;
      const unsigned ls0 = __shfl_sync(0xffffffffu, s0, L);
      const unsigned llen = __shfl_sync(0xffffffffu, len, L);
      const unsigned long long lkey = __shfl_sync(0xffffffffu, key, L);
      const unsigned np = (llen + kPiece - 1) / kPiece;
      unsigned pbase = 0;
      if (lane == 0) {
        pbase = atomicAdd(&p.plan->piece_count, np);
        const unsigned rec = atomicAdd(&p.plan->long_count, 1u);
        p.longs[rec] = LongRecord{lkey, pbase, np};
      }
      pbase = __shfl_sync(0xffffffffu, pbase, 0);
      for (unsigned q = lane; q < np; q += 32)
        p.pieces[pbase + q] = make_uint2(ls0 + q * kPiece, min((unsigned)kPiece, llen - q * kPiece));
    }
    __syncthreads();                      // s_cnt / s_base are reused
  }
}

template <typename KeyT>
cudaError_t run_plan(const PlanLaunch& p, cudaStream_t s) {
  const unsigned long long want = (p.n + 255) / 256;
  row_plan<KeyT><<<(unsigned)max(1ull, min(want, 148ull * 8)), 256, 0, s>>>(p);
  return cudaGetLastError();
}

size_t segment_scratch_bytes(unsigned long long n) {
  return 256 + (size_t)((n + kSortTile - 1) / kSortTile) * sizeof(unsigned long long);
}

unsigned segment_launch_count(unsigned long long n) {
  if (n == 0) return 0;
  return (n + kSortTile - 1) / kSortTile <= kDirectTiles ? 2u : 1u;
}

cudaError_t launch_segments(const SegmentLaunch& p, cudaStream_t stream) {
  return p.key64 ? run_heads<unsigned long long>(p, stream) : run_heads<unsigned int>(p, stream);
}

cudaError_t launch_row_plan(const PlanLaunch& p, cudaStream_t stream) {
  if (!p.n) return cudaSuccess;
  return p.key64 ? run_plan<unsigned long long>(p, stream) : run_plan<unsigned int>(p, stream);
}

unsigned int sort_tiles(unsigned long long n) {
  return (unsigned)((n + kSortTile - 1) / kSortTile);
}

size_t sort_scratch_header(unsigned passes) {
  return ((size_t)passes * 257 * sizeof(unsigned) + 255) & ~size_t(255);
}

size_t sort_scratch_bytes(unsigned long long n, unsigned bits) {
  const unsigned passes = (bits + 7) / 8;
  return sort_scratch_header(passes) +
         (size_t)passes * sort_tiles(n) * 256 * sizeof(unsigned long long);
}

unsigned int sort_launch_count(const SortLaunch& p) {
  return p.n <= 1 ? 0u : (p.hist_ready ? 0u : 1u) + (p.bits + 7) / 8;
}

cudaError_t launch_sort(const SortLaunch& p, cudaStream_t stream, int* swapped) {
  return p.key64 ? run_sort<unsigned long long>(p, stream, swapped)
                 : run_sort<unsigned int>(p, stream, swapped);
}

}  // namespace eps_b200
