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
