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
// Each 8-bit pass is reduce-then-scan: (1) per-tile digit histograms,
// (2) one exclusive scan over the digit-major [digit][tile] table, (3) a stable
// scatter in which every warp ranks its items with __match_any_sync, keeps
// per-warp running digit counts in shared memory and combines warps in order.
#include "kernels.cuh"

namespace eps_b200 {
namespace {
constexpr int kThreads = 256;
constexpr int kItems = 16;
constexpr int kSortTile = kThreads * kItems;       // 4096 items per tile
constexpr int kWarps = kThreads / 32;
constexpr int kWarpSpan = kSortTile / kWarps;      // 512 items per warp

template <typename KeyT>
__global__ void __launch_bounds__(kThreads) upsweep(const KeyT* keys, unsigned long long n,
                                                    unsigned shift, unsigned* hist,
                                                    unsigned tiles) {
  __shared__ unsigned s_hist[kWarps][256];
  const unsigned w = threadIdx.x >> 5;
  for (unsigned i = threadIdx.x; i < kWarps * 256; i += kThreads) (&s_hist[0][0])[i] = 0;
  __syncthreads();
  const unsigned long long base = (unsigned long long)blockIdx.x * kSortTile;
#pragma unroll 4
  for (int k = 0; k < kItems; ++k) {
    const unsigned long long idx = base + (unsigned long long)k * kThreads + threadIdx.x;
    if (idx < n) atomicAdd(&s_hist[w][(unsigned)(keys[idx] >> shift) & 255u], 1u);
  }
  __syncthreads();
  for (unsigned d = threadIdx.x; d < 256; d += kThreads) {
    unsigned sum = 0;
#pragma unroll
    for (int x = 0; x < kWarps; ++x) sum += s_hist[x][d];
    hist[(unsigned long long)d * tiles + blockIdx.x] = sum;
  }
}

// Exclusive scan of `total` counters in place, one block of 1024 threads.
__global__ void __launch_bounds__(1024) scan_counts(unsigned* data, unsigned total) {
  __shared__ unsigned s_warp[32];
  const unsigned t = threadIdx.x, lane = t & 31, w = t >> 5;
  const unsigned chunk = (total + 1023) / 1024;
  const unsigned begin = min(total, t * chunk), end = min(total, begin + chunk);
  unsigned sum = 0;
  for (unsigned i = begin; i < end; ++i) sum += data[i];
  // block exclusive scan of per-thread sums
  unsigned x = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= (unsigned)o) x += y;
  }
  if (lane == 31) s_warp[w] = x;
  __syncthreads();
  if (w == 0) {
    unsigned z = s_warp[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned y = __shfl_up_sync(0xffffffffu, z, o);
      if (lane >= (unsigned)o) z += y;
    }
    s_warp[lane] = z;
  }
  __syncthreads();
  unsigned run = x - sum + (w ? s_warp[w - 1] : 0u);
  for (unsigned i = begin; i < end; ++i) { const unsigned c = data[i]; data[i] = run; run += c; }
}

template <typename KeyT>
__global__ void __launch_bounds__(kThreads) downsweep(const KeyT* kin, const unsigned* vin,
                                                      KeyT* kout, unsigned* vout,
                                                      unsigned long long n, unsigned shift,
                                                      const unsigned* hist, unsigned tiles) {
  __shared__ unsigned s_cnt[kWarps][256];
  __shared__ unsigned s_glob[256];
  const unsigned w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (unsigned i = threadIdx.x; i < kWarps * 256; i += kThreads) (&s_cnt[0][0])[i] = 0;
  for (unsigned d = threadIdx.x; d < 256; d += kThreads)
    s_glob[d] = hist[(unsigned long long)d * tiles + blockIdx.x];
  __syncthreads();
  const unsigned long long base = (unsigned long long)blockIdx.x * kSortTile + w * kWarpSpan;
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
#pragma unroll
  for (int r = 0; r < kItems; ++r) {
    const unsigned long long idx = base + r * 32 + lane;
    const bool valid = idx < n;
    const unsigned d = valid ? ((unsigned)(k[r] >> shift) & 255u) : 256u;
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    unsigned prior = 0;
    if (valid) prior = s_cnt[w][d];
    __syncwarp();
    if (valid) {
      rank[r] = prior + __popc(peers & lt);
      if (lane == (unsigned)(__ffs(peers) - 1)) s_cnt[w][d] = prior + __popc(peers);
    }
    __syncwarp();
  }
  __syncthreads();
  if (threadIdx.x < 256) {
    unsigned run = 0;
#pragma unroll
    for (int x = 0; x < kWarps; ++x) { const unsigned c = s_cnt[x][threadIdx.x]; s_cnt[x][threadIdx.x] = run; run += c; }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < kItems; ++r) {
    const unsigned long long idx = base + r * 32 + lane;
    if (idx < n) {
      const unsigned d = (unsigned)(k[r] >> shift) & 255u;
      const unsigned long long pos = (unsigned long long)s_glob[d] + s_cnt[w][d] + rank[r];
      kout[pos] = k[r];
      vout[pos] = v[r];
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
  for (unsigned pass = 0; pass < passes; ++pass) {
    const unsigned shift = pass * 8;
    upsweep<KeyT><<<p.tiles, kThreads, 0, s>>>(k0, p.n, shift, p.tile_hist, p.tiles);
    scan_counts<<<1, 1024, 0, s>>>(p.tile_hist, 256u * p.tiles);
    downsweep<KeyT><<<p.tiles, kThreads, 0, s>>>(k0, v0, k1, v1, p.n, shift, p.tile_hist,
                                                 p.tiles);
    KeyT* tk = k0; k0 = k1; k1 = tk;
    unsigned* tv = v0; v0 = v1; v1 = tv;
    *swapped ^= 1;
  }
  return cudaGetLastError();
}
}  // namespace

unsigned int sort_tiles(unsigned long long n) {
  return (unsigned)((n + kSortTile - 1) / kSortTile);
}

unsigned int sort_launch_count(const SortLaunch& p) {
  return p.n <= 1 ? 0u : 3u * ((p.bits + 7) / 8);
}

cudaError_t launch_sort(const SortLaunch& p, cudaStream_t stream, int* swapped) {
  return p.key64 ? run_sort<unsigned long long>(p, stream, swapped)
                 : run_sort<unsigned int>(p, stream, swapped);
}

}  // namespace eps_b200
