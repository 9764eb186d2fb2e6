// sync.cu -- the synchronous multi-worker round reduce on the device:
// SynchronousGradientCollector::Reduce (src/training/synchronous_gradients.cpp:91-126).
//
// Every worker submits, per table, sorted unique keys owned by this shard and
// their float gradient rows.  The round's gradient for a key is
//     float( sum over workers in worker order of double(value) * scale_w )
// with scale_w = 1 / denominator (sum: 1, worker_mean: workers, sample_mean:
// the round's total samples, each worker weighted by its sample count), keys
// in ascending order (the reference's std::map).  Accumulation is in double
// from 0.0 with explicit round-to-nearest multiply and add (no contraction),
// so the result is bit-identical to the reference's loop.
//
// Device steps: the workers' (key, row) pairs are concatenated worker-major,
// stably sorted by key (the coalescing radix sort), the runs of equal keys are
// compacted, and one group per run accumulates its rows -- which the stable sort
// leaves in worker order.
#include "kernels.cuh"

namespace eps_b200 {
namespace {

// Concatenates the workers' keys (validated: strictly increasing, owned by the
// shard, inside the key space) and their rows' global indices.
__global__ void sync_pack(SyncLaunch p) {
  const unsigned long long n = p.total_rows;
  for (unsigned long long g = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; g < n;
       g += (unsigned long long)gridDim.x * blockDim.x) {
    unsigned lo = 0, hi = p.worker_count;
    while (hi - lo > 1) { const unsigned mid = (lo + hi) >> 1; if (p.row_base[mid] <= g) lo = mid; else hi = mid; }
    while (lo + 1 < p.worker_count && p.row_base[lo + 1] <= g) ++lo;
    const SyncWorker& W = p.workers[lo];
    const unsigned long long r = g - p.row_base[lo];
    const unsigned long long key = W.keys[r];
    unsigned bad = 0;
    if (r > 0 && W.keys[r - 1] >= key) bad |= 1u;                        // sorted unique
    if (key >= p.key_space || key % p.shard_count != p.shard_id) bad |= 2u;  // owned
    for (unsigned d = 0; d < p.dim; ++d)
      if (!isfinite(W.values[r * p.dim + d])) bad |= 4u;
    if (bad) atomicOr(p.error, bad);
    p.keys[g] = key;
    p.rows[g] = (unsigned)g;
  }
}

// One group of 32 lanes per run of equal keys; lanes over the dimension.
__global__ void sync_accumulate(SyncLaunch p) {
  const unsigned U = *(volatile const unsigned*)p.seg_total;
  const unsigned lane = threadIdx.x & 31;
  const unsigned long long warp = (blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x) >> 5;
  const unsigned long long nwarps = (gridDim.x * (unsigned long long)blockDim.x) >> 5;
  unsigned overflow = 0;
  for (unsigned long long u = warp; u < U; u += nwarps) {
    const unsigned s0 = p.seg_start[u], s1 = p.seg_start[u + 1];
    const unsigned long long key = p.sorted_keys[s0];
    if (lane == 0) p.keys_out[u] = key;
    for (unsigned d0 = 0; d0 < p.dim; d0 += 32) {
      const unsigned d = d0 + lane;
      double acc = 0.0;
      for (unsigned j = s0; j < s1; ++j) {
        const unsigned long long g = p.sorted_rows[j];
        unsigned lo = 0, hi = p.worker_count;
        while (hi - lo > 1) { const unsigned mid = (lo + hi) >> 1; if (p.row_base[mid] <= g) lo = mid; else hi = mid; }
        while (lo + 1 < p.worker_count && p.row_base[lo + 1] <= g) ++lo;
        if (d < p.dim) {
          const float v = p.workers[lo].values[(g - p.row_base[lo]) * p.dim + d];
          // synchronous_gradients.cpp:116-117: += double(value) * scale
          acc = __dadd_rn(acc, __dmul_rn((double)v, p.scale[lo]));
        }
      }
      if (d < p.dim) {
        const float f = __double2float_rn(acc);
        if (!isfinite(f)) overflow = 1;
        p.values_out[u * p.dim + d] = f;
      }
    }
  }
  overflow = __reduce_or_sync(~0u, overflow);
  if (overflow && lane == 0) atomicOr(p.error, 16u);
}

}  // namespace

cudaError_t launch_sync_pack(const SyncLaunch& p, cudaStream_t s) {
  if (!p.total_rows) return cudaSuccess;
  const unsigned long long want = (p.total_rows + 255) / 256;
  sync_pack<<<(unsigned)(want < 148ull * 8 ? want : 148ull * 8), 256, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_sync_accumulate(const SyncLaunch& p, cudaStream_t s) {
  if (!p.total_rows) return cudaSuccess;
  const unsigned long long want = (p.total_rows + 7) / 8;
  sync_accumulate<<<(unsigned)(want < 148ull * 8 ? want : 148ull * 8), 256, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace eps_b200
