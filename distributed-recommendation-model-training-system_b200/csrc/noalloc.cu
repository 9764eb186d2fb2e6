// noalloc.cu -- fixed device scratch for the allocation-free lookup entry point
// (eps_b200_lookup_noalloc).  This has no counterpart in the reference.
//
// Why it exists: some callers cannot allocate device memory while they serve a
// request.  Examples are an inference server or framework that owns every byte
// of GPU memory through its own pool and forbids allocations on its request
// path, and latency-critical serving loops that must never wait on the
// allocator.  The regular lookup places its per-call feature descriptors in a
// freshly allocated block; the allocation-free variant places them here
// instead.
//
// The block below is one file-scope array per GPU, created when the library's
// device code is loaded on that GPU and held until the process exits.  It
// holds the descriptors of at most kNoAllocFeatures features (168 bytes each,
// 42 KiB in all).  Every allocation-free lookup on a GPU reuses it and
// overwrites what the previous call left there.  The calls of one store are
// ordered on the GPU (each waits for the store's previous call), so only calls
// of different stores on one GPU, or of other users of this library in the
// same process, can overlap and race on it.
//
// The descriptors reach the array through the parameters of a small kernel
// (up to 24 per launch): the launch copies its parameters when it is enqueued,
// so no host memory is read after the entry point returns.
#include <mutex>

#include "kernels.cuh"

namespace eps_b200 {

static __device__ __align__(256) LookupFeature g_noalloc_features[kNoAllocFeatures];

namespace {
constexpr unsigned kNoAllocChunk = 24;
struct NoAllocChunk {
  unsigned first, count;
  LookupFeature f[kNoAllocChunk];
};
static_assert(sizeof(LookupFeature) == 168, "descriptor size stated in eps_b200.h");
static_assert(sizeof(NoAllocChunk) <= 4096, "descriptor chunk must fit the kernel parameter space");

__global__ void noalloc_store_descriptors(NoAllocChunk c) {
  for (unsigned i = threadIdx.x; i < c.count; i += blockDim.x) g_noalloc_features[c.first + i] = c.f[i];
}
}  // namespace

cudaError_t noalloc_store_features(const LookupFeature* desc, unsigned count, cudaStream_t stream,
                                   unsigned* launches) {
  *launches = 0;
  if (count > kNoAllocFeatures) return cudaErrorInvalidValue;
  for (unsigned first = 0; first < count; first += kNoAllocChunk) {
    NoAllocChunk c{};
    c.first = first;
    c.count = count - first < kNoAllocChunk ? count - first : kNoAllocChunk;
    for (unsigned i = 0; i < c.count; ++i) c.f[i] = desc[first + i];
    noalloc_store_descriptors<<<1, kNoAllocChunk, 0, stream>>>(c);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ++*launches;
  }
  return cudaSuccess;
}

// Host code may not use g_noalloc_features as an address: on the host the name
// refers to a host-side stand-in, not to device memory.  The device address is
// asked for once per GPU, with that GPU current, and cached for the life of the
// process (the address belongs to the device's primary context, which the
// library assumes lives as long as the process).
cudaError_t noalloc_feature_table(int device, LookupFeature** out) {
  static std::mutex mutex;
  static LookupFeature* addresses[kNoAllocMaxDevices] = {};
  if (device < 0 || device >= kNoAllocMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mutex);
  if (!addresses[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_features);
    if (e != cudaSuccess) return e;
    addresses[device] = static_cast<LookupFeature*>(p);
  }
  *out = addresses[device];
  return cudaSuccess;
}

}  // namespace eps_b200
