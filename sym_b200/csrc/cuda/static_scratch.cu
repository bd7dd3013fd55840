// Statically allocated device scratch for callers that cannot allocate.
//
// Some callers of this library cannot call cudaMalloc: code running under a
// caching allocator that owns the device heap, graph-building code that must
// not allocate between captures, embedded or sandboxed hosts whose memory
// budget is fixed at load time. sb_execute_h2d_static (include/sym_b200.h)
// serves them with the scratch below instead of a context's HBM ring: a
// file-scope __device__ array of SBC_STATIC_SCRATCH_BYTES that the CUDA
// driver reserves on every GPU when the module loads, held until exit.
//
// In host code the name g_static_scratch is a host-side stand-in, not a
// device address: a kernel given it would fault (or, where the GPU can reach
// host memory, silently use the wrong memory). The device address is
// resolved here, once per device, with cudaGetSymbolAddress while that device
// is current, and handed to the kernels through their descriptors.
#include "static_scratch.h"

#include <cuda_runtime.h>

#include <map>
#include <mutex>

namespace {
__device__ __align__(256) unsigned char g_static_scratch[SBC_STATIC_SCRATCH_BYTES];

std::mutex g_mutex;
std::map<int, void *> g_addresses; // device ordinal -> resolved address
} // namespace

extern "C" int sbc_static_scratch(void **device_ptr, size_t *bytes) {
  int device = -1;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess)
    return e;
  std::lock_guard<std::mutex> g(g_mutex);
  auto it = g_addresses.find(device);
  if (it == g_addresses.end()) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess)
      return e;
    it = g_addresses.emplace(device, p).first;
  }
  *device_ptr = it->second;
  *bytes = SBC_STATIC_SCRATCH_BYTES;
  return cudaSuccess;
}
