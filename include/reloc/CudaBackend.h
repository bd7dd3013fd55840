// sym_b200 -- one device's execution context: two non-blocking streams (copy
// engine and compute), the HBM ring, a parameter buffer, events, and the
// sticky error state of the reference's CopyBackend contract
// (libreloc/include/reloc/Backend.h:34-89: failed()/error(), quiesce(),
// waitStream()). All CUDA work goes through the thin C-ABI layer
// (include/sb_cuda.h); this header pulls in no CUDA headers.
#ifndef SYM_B200_RELOC_CUDABACKEND_H
#define SYM_B200_RELOC_CUDABACKEND_H

#include "reloc/Backend.h"

#include <cstddef>
#include <climits>
#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

namespace reloc {

/// A context's fault word: one word of mapped pinned host memory that the
/// kernels with bounded waits set to 2 when a wait runs out (sbc_relocate::
/// fault). The host reads it with a plain load, no CUDA call, once the work
/// that may have set it completed. Shared with pending completions, which
/// read it after their event.
struct FaultWord {
  int32_t *host = nullptr;
  int32_t *device = nullptr; // the same word's device address
  FaultWord() = default;
  FaultWord(const FaultWord &) = delete;
  FaultWord &operator=(const FaultWord &) = delete;
  ~FaultWord();
  /// The word's value, then cleared (0: no wait ran out).
  int32_t take();
};

/// One device's streams, HBM ring and parameter buffers behind the
/// reference's CopyBackend interface (reference Backend.h:34-89). Queue 0 is
/// the copy-engine stream, queue 1 the compute stream.
class CudaBackend : public CopyBackend {
public:
  /// Create a context on `device` (made current for the calling thread).
  static std::unique_ptr<CudaBackend> create(int device, std::string &error);
  ~CudaBackend() override;
  CudaBackend(const CudaBackend &) = delete;
  CudaBackend &operator=(const CudaBackend &) = delete;

  // ---- CopyBackend
  void *allocStaging(size_t bytes) override;
  void freeStaging(void *p) override;
  int numQueues() const override { return 2; }
  void copyAsync(int queue, void *dst, const void *src, size_t bytes, CopyDir dir) override;
  EventHandle recordEvent(int queue) override;
  void waitEvent(EventHandle ev) override;
  bool queryEvent(EventHandle ev) override;
  int device() const override { return device_; }
  bool failed() const override { return failed_; }
  const std::string &error() const override { return error_; }
  /// Record a failure (first one wins). Returns false for call chaining.
  bool fail(const std::string &what, int status);
  /// Record a failure with a message of its own (first one wins).
  bool failWith(const std::string &message);
  /// Reads (and clears) the fault word: a wait that ran out in work that has
  /// completed makes the context failed. Returns !failed().
  bool healthy();
  /// Device address of the fault word, for the descriptors of this context.
  int32_t *faultWord() const { return fault_->device; }
  const std::shared_ptr<FaultWord> &faultShared() const { return fault_; }
  /// Make this backend's device current on the calling thread.
  bool activate();

  void *copyStream() const { return copy_; }
  void *computeStream() const { return compute_; }

  /// Order both private streams after the work already on `external`.
  bool waitStream(const void *external) override;
  /// Record completion of everything enqueued so far on the private streams;
  /// with `hasExternal`, order `external` (a null handle = the legacy default
  /// stream) after it.
  bool signalStream(const void *external, bool hasExternal, bool copyUsed = true);
  /// Block until all enqueued work completed (every queue is attempted
  /// despite earlier failures); Unknown when a queue cannot be drained.
  QueueCompletion quiesce() override;

  /// HBM ring of `slots` buffers of `slotBytes` (grown, never shrunk).
  bool ensureRing(int slots, size_t slotBytes);
  void *slot(int i) const { return ring_[static_cast<size_t>(i)]; }
  void *slotReady(int i) const { return ready_[static_cast<size_t>(i)]; }
  void *slotFree(int i) const { return free_[static_cast<size_t>(i)]; }
  int slots() const { return static_cast<int>(ring_.size()); }
  size_t slotBytes() const { return slotBytes_; }

  /// Device scratch for staged sources (whole-source route), grown on demand.
  void *staging(size_t bytes);
  /// Device parameter buffer (grown on demand).
  void *params(size_t bytes);
  /// A device status word (channel range errors) and its pinned readback.
  int32_t *statusWord() const { return status_; }
  int32_t *statusHost() const { return statusHost_; }

  void *stagingReady() const { return stagingReady_; }
  void *stagingFree() const { return stagingFree_; }
  void *doneEvent() const { return done_; }
  void *startEvent() const { return start_; }
  void *stopEvent() const { return stop_; }

  size_t deviceBytes() const;
  /// Scratch budget of this context (the owner's limits divided among its
  /// contexts): `liveLimit` caps the device scratch an execution may hold
  /// (0 = unlimited); scratch beyond `retainedLimit` is released when a
  /// blocking execution's lease ends.
  size_t liveLimit = 0;
  size_t retainedLimit = SIZE_MAX;
  /// Bytes a ring slot may take for `slots` slots under the live limit (and,
  /// when `retained`, also the retained limit), after the other scratch.
  size_t ringSlotBudget(int slots, bool retained) const;
  /// Release ring and staging scratch until at most `keep` bytes remain
  /// (waits for queued work first). Returns whether anything was released.
  bool trim(size_t keep);
  size_t peakDeviceBytes = 0;
  uint64_t trims = 0;
  size_t ringBytes() const { return ring_.size() * slotBytes_; }
  size_t stagingCapacity() const { return stagingBytes_; }
  uint64_t copyCalls = 0;
  uint64_t eventRecords = 0;
  uint64_t eventWaits = 0;
  uint64_t callerWaits = 0;
  uint64_t kernelLaunches = 0;
  /// Set while a group runs: its members share one status word, cleared once
  /// before the first member instead of once per execution.
  bool keepStatus = false;

  /// Measured route choice per plan class: key -> seconds per byte of each
  /// route, from its latest timed execution. A route counts as measured after
  /// two samples (the first may include one-time ring allocation).
  struct RouteStats {
    double dmaSecondsPerByte = -1, zeroCopySecondsPerByte = -1;
    uint32_t dmaSamples = 0, zeroCopySamples = 0;
    bool known() const { return dmaSamples >= 2 && zeroCopySamples >= 2; }
    uint32_t executions = 0; // auto-route executions since both were measured
    bool probe = false;      // this timed execution re-measures the slower route
  };
  std::map<std::string, RouteStats> routeStats;
  std::mutex mutex; // one request at a time per context

  /// Copy `bytes` of pageable (unregistered) host memory at `src` to device
  /// memory `dst`, queued on the copy stream, through pinned bounce buffers:
  /// host threads fill one buffer while the copy engine drains the previous
  /// one. Returns when the last piece is queued (the host source may change
  /// afterwards). The driver's own pageable path copies on one thread.
  bool bounceH2D(void *dst, const void *src, size_t bytes);
  uint64_t bouncedBytes = 0;

private:
  struct HostCopyPool;
  static constexpr int kBounceBuffers = 3;
  CudaBackend() = default;
  std::unique_ptr<HostCopyPool> pool_;
  void *bounce_[kBounceBuffers] = {};
  void *bounceFree_[kBounceBuffers] = {};
  bool bounceUsed_[kBounceBuffers] = {};
  int device_ = -1;
  bool failed_ = false;
  std::string error_;
  void *copy_ = nullptr, *compute_ = nullptr;
  void *done_ = nullptr, *start_ = nullptr, *stop_ = nullptr, *fence_ = nullptr;
  void *stagingReady_ = nullptr, *stagingFree_ = nullptr;
  std::vector<void *> ring_, ready_, free_;
  size_t slotBytes_ = 0;
  void *staging_ = nullptr;
  size_t stagingBytes_ = 0;
  void *params_ = nullptr;
  size_t paramBytes_ = 0;
  int32_t *status_ = nullptr;
  int32_t *statusHost_ = nullptr;
  std::shared_ptr<FaultWord> fault_;
  // CopyBackend events handed out by recordEvent (handle = index + 1) and
  // staging blocks handed out by allocStaging.
  std::vector<void *> events_;
  std::vector<void *> stagingBlocks_;
};

} // namespace reloc

#endif
