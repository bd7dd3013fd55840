// One device's execution context over the thin C-ABI layer; see
// include/reloc/CudaBackend.h.
#include "reloc/CudaBackend.h"

#include "sb_cuda.h"

namespace reloc {

bool CudaBackend::fail(const std::string &what, int status) {
  if (!failed_) {
    failed_ = true;
    error_ = what + ": " + sbc_error_string(status);
  }
  return false;
}

bool CudaBackend::activate() {
  const int rc = sbc_set_device(device_);
  return rc == 0 || fail("cudaSetDevice", rc);
}

std::unique_ptr<CudaBackend> CudaBackend::create(int device, std::string &error) {
  std::unique_ptr<CudaBackend> b(new CudaBackend());
  b->device_ = device;
  int rc = sbc_set_device(device);
  if (rc) {
    error = std::string("cudaSetDevice: ") + sbc_error_string(rc);
    return nullptr;
  }
  void *host = nullptr;
  if ((rc = sbc_stream_create(&b->copy_)) || (rc = sbc_stream_create(&b->compute_)) ||
      (rc = sbc_event_create(&b->done_, 0)) || (rc = sbc_event_create(&b->fence_, 0)) ||
      (rc = sbc_event_create(&b->start_, 1)) || (rc = sbc_event_create(&b->stop_, 1)) ||
      (rc = sbc_event_create(&b->stagingReady_, 0)) || (rc = sbc_event_create(&b->stagingFree_, 0)) ||
      (rc = sbc_malloc_device(reinterpret_cast<void **>(&b->status_), 16)) || (rc = sbc_malloc_host(&host, 16, 0))) {
    error = std::string("context creation: ") + sbc_error_string(rc);
    return nullptr;
  }
  b->statusHost_ = static_cast<int32_t *>(host);
  return b;
}

CudaBackend::~CudaBackend() {
  if (device_ < 0)
    return;
  sbc_set_device(device_);
  quiesce();
  for (void *p : ring_)
    sbc_free_device(p);
  for (void *e : ready_)
    sbc_event_destroy(e);
  for (void *e : free_)
    sbc_event_destroy(e);
  if (staging_)
    sbc_free_device(staging_);
  if (params_)
    sbc_free_device(params_);
  if (status_)
    sbc_free_device(status_);
  if (statusHost_)
    sbc_free_host(statusHost_);
  for (void *e : {done_, fence_, start_, stop_, stagingReady_, stagingFree_})
    if (e)
      sbc_event_destroy(e);
  if (copy_)
    sbc_stream_destroy(copy_);
  if (compute_)
    sbc_stream_destroy(compute_);
}

bool CudaBackend::waitStream(const void *external) {
  int rc;
  if ((rc = sbc_event_record(fence_, const_cast<void *>(external))))
    return fail("cudaEventRecord(caller stream)", rc);
  ++eventRecords;
  if ((rc = sbc_stream_wait_event(copy_, fence_)) || (rc = sbc_stream_wait_event(compute_, fence_)))
    return fail("cudaStreamWaitEvent", rc);
  eventWaits += 2;
  ++callerWaits;
  return true;
}

bool CudaBackend::signalStream(const void *external, bool hasExternal) {
  int rc;
  if ((rc = sbc_event_record(fence_, copy_)) || (rc = sbc_stream_wait_event(compute_, fence_)) ||
      (rc = sbc_event_record(done_, compute_)))
    return fail("cudaEventRecord", rc);
  eventRecords += 2;
  // A null handle is the legacy default stream, a real caller stream.
  if (hasExternal && (rc = sbc_stream_wait_event(const_cast<void *>(external), done_)))
    return fail("cudaStreamWaitEvent(caller stream)", rc);
  return true;
}

QueueCompletion CudaBackend::quiesce() {
  bool ok = true;
  for (void *s : {copy_, compute_})
    if (s) {
      const int rc = sbc_stream_synchronize(s);
      if (rc) {
        fail("cudaStreamSynchronize", rc);
        ok = false;
      }
    }
  return ok ? QueueCompletion::Complete : QueueCompletion::Unknown;
}

bool CudaBackend::ensureRing(int slots, size_t bytes) {
  if (static_cast<int>(ring_.size()) >= slots && slotBytes_ >= bytes)
    return true;
  // Growing: the old slots may still be read by queued kernels.
  quiesce();
  for (void *p : ring_)
    sbc_free_device(p);
  ring_.clear();
  const size_t want = bytes > slotBytes_ ? bytes : slotBytes_;
  const int n = slots > static_cast<int>(ready_.size()) ? slots : static_cast<int>(ready_.size());
  for (int i = 0; i < n; ++i) {
    void *p = nullptr;
    int rc = sbc_malloc_device(&p, want);
    if (rc)
      return fail("cudaMalloc(ring slot)", rc);
    ring_.push_back(p);
    if (static_cast<int>(ready_.size()) <= i) {
      void *a = nullptr, *b = nullptr;
      if ((rc = sbc_event_create(&a, 0)) || (rc = sbc_event_create(&b, 0)))
        return fail("cudaEventCreate", rc);
      ready_.push_back(a);
      free_.push_back(b);
    }
  }
  slotBytes_ = want;
  return true;
}

void *CudaBackend::staging(size_t bytes) {
  if (bytes <= stagingBytes_)
    return staging_;
  quiesce();
  if (staging_)
    sbc_free_device(staging_);
  staging_ = nullptr;
  stagingBytes_ = 0;
  const int rc = sbc_malloc_device(&staging_, bytes);
  if (rc) {
    fail("cudaMalloc(staging)", rc);
    return nullptr;
  }
  stagingBytes_ = bytes;
  return staging_;
}

void *CudaBackend::params(size_t bytes) {
  if (bytes == 0)
    bytes = 16;
  if (bytes <= paramBytes_)
    return params_;
  quiesce();
  if (params_)
    sbc_free_device(params_);
  params_ = nullptr;
  paramBytes_ = 0;
  const int rc = sbc_malloc_device(&params_, bytes);
  if (rc) {
    fail("cudaMalloc(parameters)", rc);
    return nullptr;
  }
  paramBytes_ = bytes;
  return params_;
}

size_t CudaBackend::deviceBytes() const { return ring_.size() * slotBytes_ + stagingBytes_ + paramBytes_ + 16; }

} // namespace reloc
