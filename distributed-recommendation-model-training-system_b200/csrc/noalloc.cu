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
// holds the descriptors of at most kNoAllocFeatures features (about 26 KiB).
// Every allocation-free lookup on a GPU reuses it and overwrites what the
// previous call left there; two such lookups that overlap on the same GPU
// (different streams, or different stores on one GPU) race on it.
#include <mutex>

#include "kernels.cuh"

namespace eps_b200 {

static __device__ __align__(256) LookupFeature g_noalloc_features[kNoAllocFeatures];

// Host code may not use g_noalloc_features as an address: on the host the name
// refers to a host-side stand-in, not to device memory.  The device address is
// asked for once per GPU, with that GPU current, and cached.
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
