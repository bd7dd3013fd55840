// sym_b200 -- the CUDA runtime half of the thin C-ABI layer (include/sb_cuda.h):
// devices, pinned/device memory, async copies, streams and events. Each
// function is one checked CUDA runtime call; status codes are cudaError_t
// values. Counterpart of the reference's CudaBackend
// (libreloc/cuda/CudaBackend.cu:55-282).
#include "sb_cuda.h"

#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstring>

namespace {
cudaStream_t S(void *s) { return static_cast<cudaStream_t>(s); }
cudaEvent_t E(void *e) { return static_cast<cudaEvent_t>(e); }

// Test-only failure injection (sbc_test_fault_mode): the wrapped call reports
// cudaErrorUnknown without being issued. Off unless a test arms it.
std::atomic<int> g_fault_mode{0};
std::atomic<int> g_fault_copies{0};
bool inject_event_record() {
  const int m = g_fault_mode.load(std::memory_order_relaxed);
  return m == 1 || m == 2;
}
bool inject_stream_sync() {
  const int m = g_fault_mode.load(std::memory_order_relaxed);
  return m == 2 || m == 4 || m == 6;
}
bool inject_event_sync() {
  const int m = g_fault_mode.load(std::memory_order_relaxed);
  return m == 5 || m == 6;
}
bool inject_h2d_copy() {
  const int m = g_fault_mode.load(std::memory_order_relaxed);
  return (m == 3 || m == 4) && g_fault_copies.fetch_add(1) + 1 == 3;
}
} // namespace

extern "C" {

int sbc_device_count(int *count) { return cudaGetDeviceCount(count); }
int sbc_set_device(int device) { return cudaSetDevice(device); }
int sbc_get_device(int *device) { return cudaGetDevice(device); }

int sbc_device_info(int device, int *major, int *minor, int *sms, size_t *hbm_bytes) {
  cudaDeviceProp p;
  cudaError_t e = cudaGetDeviceProperties(&p, device);
  if (e != cudaSuccess)
    return e;
  *major = p.major;
  *minor = p.minor;
  *sms = p.multiProcessorCount;
  *hbm_bytes = p.totalGlobalMem;
  return 0;
}

int sbc_malloc_device(void **ptr, size_t bytes) { return cudaMalloc(ptr, bytes); }
int sbc_free_device(void *ptr) { return cudaFree(ptr); }

int sbc_malloc_host(void **ptr, size_t bytes, int mapped) {
  return cudaHostAlloc(ptr, bytes, mapped ? (cudaHostAllocMapped | cudaHostAllocPortable) : cudaHostAllocPortable);
}
int sbc_free_host(void *ptr) { return cudaFreeHost(ptr); }

int sbc_host_register(void *ptr, size_t bytes, int mapped) {
  return cudaHostRegister(ptr, bytes, mapped ? (cudaHostRegisterMapped | cudaHostRegisterPortable)
                                             : cudaHostRegisterPortable);
}
int sbc_host_unregister(void *ptr) { return cudaHostUnregister(ptr); }

int sbc_host_device_pointer(void *host, void **device) {
  const cudaError_t e = cudaHostGetDevicePointer(device, host, 0);
  if (e != cudaSuccess)
    cudaGetLastError(); // an expected probe failure must not poison later launch checks
  return e;
}

namespace {
PFN_cuMemGetAddressRange_v3020 address_range() {
  static PFN_cuMemGetAddressRange_v3020 fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
    cudaGetLastError();
    return static_cast<PFN_cuMemGetAddressRange_v3020>(nullptr);
  }();
  return fn;
}
} // namespace

int sbc_ipc_get_handle(void *device_ptr, unsigned char handle[64], size_t *offset) {
  // An IPC handle names a whole allocation; a pointer inside a larger
  // allocation (a caching allocator's segment) is its base plus an offset.
  PFN_cuMemGetAddressRange_v3020 range = address_range();
  if (!range)
    return cudaErrorNotSupported;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(device_ptr)) != CUDA_SUCCESS)
    return cudaErrorInvalidDevicePointer;
  *offset = static_cast<size_t>(reinterpret_cast<CUdeviceptr>(device_ptr) - base);
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return e;
  }
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle, &h, sizeof(h));
  return 0;
}

int sbc_ipc_open_handle(const unsigned char handle[64], void **device_ptr) {
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(device_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess)
    cudaGetLastError();
  return e;
}

int sbc_ipc_close_handle(void *device_ptr) { return cudaIpcCloseMemHandle(device_ptr); }

int sbc_pointer_info(const void *ptr, int *kind, int *device) {
  cudaPointerAttributes a;
  cudaError_t e = cudaPointerGetAttributes(&a, ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return e;
  }
  switch (a.type) {
  case cudaMemoryTypeHost: *kind = 1; break;
  case cudaMemoryTypeDevice: *kind = 2; break;
  case cudaMemoryTypeManaged: *kind = 3; break;
  default: *kind = 0; break;
  }
  *device = (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) ? a.device : -1;
  return 0;
}

int sbc_memcpy_h2d_async(void *dst, const void *src, size_t bytes, void *stream) {
  if (inject_h2d_copy())
    return cudaErrorUnknown;
  return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, S(stream));
}
int sbc_memcpy_d2h_async(void *dst, const void *src, size_t bytes, void *stream) {
  return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, S(stream));
}
int sbc_memcpy_d2d_async(void *dst, const void *src, size_t bytes, void *stream) {
  return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, S(stream));
}
int sbc_memcpy_h2d_2d_async(void *dst, size_t dpitch, const void *src, size_t spitch, size_t width, size_t rows,
                            void *stream) {
  return cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, rows, cudaMemcpyHostToDevice, S(stream));
}

int sbc_stream_create(void **stream) {
  cudaStream_t s = nullptr;
  cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  *stream = s;
  return e;
}
int sbc_stream_destroy(void *stream) { return cudaStreamDestroy(S(stream)); }
int sbc_stream_synchronize(void *stream) {
  if (inject_stream_sync())
    return cudaErrorUnknown;
  return cudaStreamSynchronize(S(stream));
}

int sbc_event_create(void **event, int timing) {
  cudaEvent_t ev = nullptr;
  cudaError_t e = cudaEventCreateWithFlags(&ev, timing ? cudaEventDefault : cudaEventDisableTiming);
  *event = ev;
  return e;
}
int sbc_event_destroy(void *event) { return cudaEventDestroy(E(event)); }
int sbc_event_record(void *event, void *stream) {
  if (inject_event_record())
    return cudaErrorUnknown;
  return cudaEventRecord(E(event), S(stream));
}
int sbc_event_query(void *event) {
  cudaError_t e = cudaEventQuery(E(event));
  if (e == cudaErrorNotReady) {
    return 1;
  }
  return e;
}
int sbc_event_synchronize(void *event) {
  if (inject_event_sync())
    return cudaErrorUnknown;
  return cudaEventSynchronize(E(event));
}
int sbc_stream_wait_event(void *stream, void *event) { return cudaStreamWaitEvent(S(stream), E(event), 0); }
int sbc_event_elapsed_ms(void *start, void *stop, float *ms) { return cudaEventElapsedTime(ms, E(start), E(stop)); }

int sbc_test_fault_mode(int mode) {
  if (mode < 0 || mode > 6)
    return SBC_EINVAL;
  g_fault_copies.store(0);
  g_fault_mode.store(mode);
  return 0;
}

const char *sbc_error_string(int status) {
  if (status == SBC_EINVAL)
    return "descriptor violates the launcher's preconditions";
  if (status == SBC_EUNSUPPORTED)
    return "layout is not of this kernel family";
  return cudaGetErrorString(static_cast<cudaError_t>(status));
}

} // extern "C"
