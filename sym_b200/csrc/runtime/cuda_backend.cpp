// One device's execution context over the thin C-ABI layer; see
// include/reloc/CudaBackend.h.
#include "reloc/CudaBackend.h"

#include "sb_cuda.h"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <thread>

namespace reloc {

/// Worker threads that split one host memcpy with the calling thread. A
/// bounce copy hands out one piece every few hundred microseconds, so both
/// sides poll for up to kSpinUs before sleeping on a condition variable
/// (waking a sleeping thread can cost more than a piece's copy).
struct CudaBackend::HostCopyPool {
  static constexpr int64_t kSpinUs = 200;

  explicit HostCopyPool(int workers) {
    for (int k = 1; k <= workers; ++k)
      threads.emplace_back([this, k] { run(k); });
  }
  ~HostCopyPool() {
    {
      std::lock_guard<std::mutex> g(m);
      stop.store(true);
    }
    wake.notify_all();
    for (auto &t : threads)
      t.join();
  }
  /// Copy [src, src + bytes) to dst with every thread; returns when done.
  void copy(void *dst, const void *src, size_t bytes) {
    const size_t parts = threads.size() + 1;
    if (threads.empty() || bytes < (size_t(1) << 20)) {
      std::memcpy(dst, src, bytes);
      return;
    }
    dst_ = static_cast<uint8_t *>(dst);
    src_ = static_cast<const uint8_t *>(src);
    bytes_ = bytes;
    part_ = ((bytes + parts - 1) / parts + 63) & ~size_t(63);
    pending.store(static_cast<int>(threads.size()), std::memory_order_relaxed);
    {
      std::lock_guard<std::mutex> g(m);
      generation.fetch_add(1, std::memory_order_release); // publishes the job fields
    }
    wake.notify_all();
    std::memcpy(dst, src, std::min(part_, bytes));
    if (!spinUntil([this] { return pending.load(std::memory_order_acquire) == 0; })) {
      std::unique_lock<std::mutex> g(m);
      finished.wait(g, [this] { return pending.load(std::memory_order_acquire) == 0; });
    }
  }

private:
  template <class Pred> static bool spinUntil(Pred ready) {
    const auto t0 = std::chrono::steady_clock::now();
    for (uint32_t i = 1;; ++i) {
      if (ready())
        return true;
      if ((i & 63u) == 0 &&
          std::chrono::steady_clock::now() - t0 > std::chrono::microseconds(kSpinUs))
        return false;
    }
  }
  void run(int k) {
    uint64_t seen = 0;
    for (;;) {
      auto fresh = [&] { return stop.load(std::memory_order_relaxed) ||
                                generation.load(std::memory_order_acquire) != seen; };
      if (!spinUntil(fresh)) {
        std::unique_lock<std::mutex> g(m);
        wake.wait(g, fresh);
      }
      if (stop.load())
        return;
      seen = generation.load(std::memory_order_acquire);
      const size_t lo = std::min(bytes_, part_ * static_cast<size_t>(k));
      const size_t hi = std::min(bytes_, lo + part_);
      if (hi > lo)
        std::memcpy(dst_ + lo, src_ + lo, hi - lo);
      if (pending.fetch_sub(1, std::memory_order_acq_rel) == 1) {
        std::lock_guard<std::mutex> g(m);
        finished.notify_one();
      }
    }
  }
  std::vector<std::thread> threads;
  std::mutex m;
  std::condition_variable wake, finished;
  std::atomic<uint64_t> generation{0};
  std::atomic<int> pending{0};
  std::atomic<bool> stop{false};
  uint8_t *dst_ = nullptr;
  const uint8_t *src_ = nullptr;
  size_t bytes_ = 0, part_ = 0;
};

namespace {
/// Host threads that help with a pageable copy (SYM_B200_HOST_COPY_THREADS,
/// default a quarter of the hardware threads, 1 to 4, plus the caller).
int hostCopyWorkers() {
  if (const char *v = std::getenv("SYM_B200_HOST_COPY_THREADS"))
    return std::max(0, std::atoi(v) - 1);
  const int hw = static_cast<int>(std::thread::hardware_concurrency());
  return std::clamp(hw / 4, 1, 4);
}
} // namespace

bool CudaBackend::bounceH2D(void *dst, const void *src, size_t bytes) {
  constexpr size_t kPiece = size_t(8) << 20;
  if (!bounce_[0]) {
    for (int k = 0; k < kBounceBuffers; ++k) {
      int rc;
      if ((rc = sbc_malloc_host(&bounce_[k], kPiece, 0)))
        return fail("cudaHostAlloc(bounce)", rc);
      if ((rc = sbc_event_create(&bounceFree_[k], 0)))
        return fail("cudaEventCreate", rc);
    }
  }
  if (!pool_)
    pool_.reset(new HostCopyPool(hostCopyWorkers()));
  const auto *s = static_cast<const uint8_t *>(src);
  auto *d = static_cast<uint8_t *>(dst);
  for (size_t off = 0, piece = 0; off < bytes; ++piece) {
    const size_t n = std::min(kPiece, bytes - off);
    const int k = static_cast<int>(piece % kBounceBuffers);
    int rc;
    if (bounceUsed_[k] && (rc = sbc_event_synchronize(bounceFree_[k]))) // its last DMA has read it
      return fail("bounce buffer wait", rc);
    pool_->copy(bounce_[k], s + off, n);
    if ((rc = sbc_memcpy_h2d_async(d + off, bounce_[k], n, copy_)) || (rc = sbc_event_record(bounceFree_[k], copy_)))
      return fail("bounce upload", rc);
    bounceUsed_[k] = true;
    ++copyCalls;
    ++eventRecords;
    off += n;
  }
  bouncedBytes += bytes;
  return true;
}

bool CudaBackend::fail(const std::string &what, int status) {
  if (!failed_) {
    failed_ = true;
    error_ = what + ": " + sbc_error_string(status);
  }
  return false;
}

bool CudaBackend::failWith(const std::string &message) {
  if (!failed_) {
    failed_ = true;
    error_ = message;
  }
  return false;
}

FaultWord::~FaultWord() {
  if (host)
    sbc_free_host(host);
}

int32_t FaultWord::take() {
  auto *w = reinterpret_cast<volatile int32_t *>(host);
  const int32_t v = *w;
  if (v)
    *w = 0;
  return v;
}

bool CudaBackend::healthy() {
  if (fault_ && fault_->take())
    failWith("a kernel's bounded wait for a TMA copy ran out; the output is incomplete");
  return !failed_;
}

// ---- CopyBackend ------------------------------------------------------------

void *CudaBackend::allocStaging(size_t bytes) {
  void *p = nullptr;
  const int rc = sbc_malloc_host(&p, bytes ? bytes : 1, 0);
  if (rc) {
    fail("cudaHostAlloc(staging)", rc);
    return nullptr;
  }
  stagingBlocks_.push_back(p);
  return p;
}

void CudaBackend::freeStaging(void *p) {
  auto it = std::find(stagingBlocks_.begin(), stagingBlocks_.end(), p);
  if (it == stagingBlocks_.end())
    return;
  stagingBlocks_.erase(it);
  const int rc = sbc_free_host(p);
  if (rc)
    fail("cudaFreeHost(staging)", rc);
}

void CudaBackend::copyAsync(int queue, void *dst, const void *src, size_t bytes, CopyDir dir) {
  if (failed_)
    return;
  void *s = queue == 1 ? compute_ : copy_;
  const int rc = dir == CopyDir::HostToDevice ? sbc_memcpy_h2d_async(dst, src, bytes, s)
                                              : sbc_memcpy_d2h_async(dst, src, bytes, s);
  if (rc)
    fail("cudaMemcpyAsync", rc);
  else
    ++copyCalls;
}

EventHandle CudaBackend::recordEvent(int queue) {
  if (failed_)
    return 0;
  void *e = nullptr;
  int rc = sbc_event_create(&e, 0);
  if (rc) {
    fail("cudaEventCreate", rc);
    return 0;
  }
  if ((rc = sbc_event_record(e, queue == 1 ? compute_ : copy_))) {
    sbc_event_destroy(e);
    fail("cudaEventRecord", rc);
    return 0;
  }
  ++eventRecords;
  events_.push_back(e);
  return static_cast<EventHandle>(events_.size());
}

void CudaBackend::waitEvent(EventHandle ev) {
  if (ev == 0 || ev > events_.size() || !events_[ev - 1])
    return;
  void *&e = events_[ev - 1];
  const int rc = sbc_event_synchronize(e);
  if (rc) {
    fail("cudaEventSynchronize", rc);
    return;
  }
  sbc_event_destroy(e);
  e = nullptr;
}

bool CudaBackend::queryEvent(EventHandle ev) {
  if (ev == 0 || ev > events_.size() || !events_[ev - 1])
    return true;
  const int rc = sbc_event_query(events_[ev - 1]);
  if (rc == 1)
    return false;
  if (rc)
    fail("cudaEventQuery", rc);
  return true;
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
  // The fault word: mapped pinned memory the kernels write and the host reads
  // without a CUDA call.
  auto fw = std::make_shared<FaultWord>();
  void *word = nullptr, *dev = nullptr;
  if ((rc = sbc_malloc_host(&word, 64, 1))) {
    error = std::string("context creation (fault word): ") + sbc_error_string(rc);
    return nullptr;
  }
  fw->host = static_cast<int32_t *>(word);
  *fw->host = 0;
  if ((rc = sbc_host_device_pointer(word, &dev))) {
    error = std::string("context creation (fault word mapping): ") + sbc_error_string(rc);
    return nullptr;
  }
  fw->device = static_cast<int32_t *>(dev);
  b->fault_ = std::move(fw);
  return b;
}

CudaBackend::~CudaBackend() {
  if (device_ < 0)
    return;
  int current = -1; // restored below: retiring a context leaves the caller's device alone
  sbc_get_device(&current);
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
  for (int k = 0; k < kBounceBuffers; ++k) {
    if (bounce_[k])
      sbc_free_host(bounce_[k]);
    if (bounceFree_[k])
      sbc_event_destroy(bounceFree_[k]);
  }
  for (void *e : {done_, fence_, start_, stop_, stagingReady_, stagingFree_})
    if (e)
      sbc_event_destroy(e);
  for (void *e : events_)
    if (e)
      sbc_event_destroy(e);
  for (void *p : stagingBlocks_)
    sbc_free_host(p);
  if (copy_)
    sbc_stream_destroy(copy_);
  if (compute_)
    sbc_stream_destroy(compute_);
  if (current >= 0 && current != device_)
    sbc_set_device(current);
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

bool CudaBackend::signalStream(const void *external, bool hasExternal, bool copyUsed) {
  int rc;
  // Join the copy stream into the compute stream only when this execution
  // queued copies there; `done` then covers both.
  if (copyUsed && ((rc = sbc_event_record(fence_, copy_)) || (rc = sbc_stream_wait_event(compute_, fence_))))
    return fail("cudaEventRecord", rc);
  if ((rc = sbc_event_record(done_, compute_)))
    return fail("cudaEventRecord", rc);
  eventRecords += copyUsed ? 2 : 1;
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
  peakDeviceBytes = std::max(peakDeviceBytes, deviceBytes());
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
  peakDeviceBytes = std::max(peakDeviceBytes, deviceBytes());
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
  peakDeviceBytes = std::max(peakDeviceBytes, deviceBytes());
  return params_;
}

size_t CudaBackend::deviceBytes() const { return ring_.size() * slotBytes_ + stagingBytes_ + paramBytes_ + 16; }

size_t CudaBackend::ringSlotBudget(int slots, bool retained) const {
  size_t limit = liveLimit ? liveLimit : SIZE_MAX;
  if (retained && retainedLimit < limit)
    limit = retainedLimit;
  if (limit == SIZE_MAX)
    return SIZE_MAX;
  const size_t other = stagingBytes_ + paramBytes_ + 16;
  return limit > other ? (limit - other) / static_cast<size_t>(slots > 0 ? slots : 1) : 0;
}

bool CudaBackend::trim(size_t keep) {
  if (deviceBytes() <= keep)
    return false;
  quiesce();
  for (void *p : ring_)
    sbc_free_device(p);
  ring_.clear();
  slotBytes_ = 0;
  if (deviceBytes() > keep && staging_) {
    sbc_free_device(staging_);
    staging_ = nullptr;
    stagingBytes_ = 0;
  }
  ++trims;
  return true;
}

} // namespace reloc
