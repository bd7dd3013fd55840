// sym_b200 -- typed contexts: a bounded, thread-safe pool of per-device
// execution contexts (streams, HBM ring, parameter buffers).
//
// Interface of the reference's dispatch::Resources
// (libreloc/include/reloc/DispatchResources.h:9-103; execute :74-86): leases
// by device, FIFO admission per device, sticky quarantine after a failure
// whose completion is unknown, stats(), clear(), close(). A context here is a
// CudaBackend; there are no host worker pools because no plan runs on the CPU.
#ifndef SYM_B200_RELOC_DISPATCHRESOURCES_H
#define SYM_B200_RELOC_DISPATCHRESOURCES_H

#include "reloc/CudaBackend.h"
#include "reloc/Dispatch.h"

#include <cstddef>
#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <optional>
#include <variant>

namespace reloc {
namespace dispatch {

/// The pending completion of a submitted group (reference
/// DispatchResources.h:9-25). It owns one event recorded after the group's
/// last member. Dropping a handle without wait() still waits (drains).
class Completion {
public:
  struct State;
  explicit Completion(std::shared_ptr<State> state);
  ~Completion();
  Completion(const Completion &) = delete;
  Completion &operator=(const Completion &) = delete;
  /// Host wait; then the device fault word is checked. Idempotent.
  TransferOutcome wait();
  /// true once complete (and finalized as by wait()), false while pending.
  std::variant<bool, TransferError> query();
  /// GPU-side dependency: `consumer` (a cudaStream_t) waits for the group
  /// without blocking the host.
  std::optional<TransferError> waitStream(const void *consumer);

private:
  std::shared_ptr<State> state_;
};

struct ResourceStats {
  uint64_t requests = 0, hits = 0, contexts = 0;
  uint64_t deviceAllocations = 0, frees = 0;
  size_t retainedBytes = 0, deviceBytes = 0;
  uint64_t copyCalls = 0, eventRecords = 0, eventWaits = 0, callerWaits = 0, kernelLaunches = 0;
  bool closed = false, quarantined = false;
  size_t retainedLimit = 0, liveLimit = 0;
  unsigned contextLimit = 0;
  size_t peakLiveBytes = 0; // sum over contexts of each one's peak scratch
  uint64_t releases = 0;    // scratch releases at lease end (over the retained quota)
  uint64_t evictions = 0;   // contexts retired to admit one for another device
  uint64_t retirements = 0; // contexts retired after a failed execution (completion proven)
};

class Resources {
public:
  explicit Resources(size_t maxRetainedBytes = size_t(64) << 20, size_t maxLiveBytes = 0, unsigned maxContexts = 1);
  ~Resources();
  Resources(const Resources &) = delete;
  Resources &operator=(const Resources &) = delete;

  /// Lease the context of `device` and run the request on it.
  TransferOutcome execute(DispatchRequest &request, int device, int streams, const TransferOptions &options,
                          std::shared_ptr<void> owners);
  /// Run a group on the context of its device and complete it (blocking
  /// unless options.asyncCompletion, then the caller stream carries it).
  TransferOutcome execute(GroupRequest &group, const TransferOptions &options, std::shared_ptr<void> owners);
  /// Enqueue a group and return its completion without waiting (reference
  /// DispatchResources.h:85-86). Plans with device-checked channel maps still
  /// complete before returning (their status word is read back).
  std::variant<std::shared_ptr<Completion>, TransferError> submit(GroupRequest &group, const TransferOptions &options,
                                                                  std::shared_ptr<void> owners);
  /// Run `fn` with the leased context of `device` (window/device executions).
  /// With `releaseAfter` (blocking work), scratch beyond the context's
  /// retained quota is released before the lease ends. Each context holds
  /// an equal share of the owner's retained and live limits; a nonzero live
  /// limit caps the scratch one execution may hold (insufficient_capacity
  /// when a plan cannot run within it), zero leaves it unlimited.
  TransferOutcome withContext(int device, const std::function<std::optional<TransferError>(CudaBackend &)> &fn,
                              bool releaseAfter = true);

  /// Bound the wait for a context another call holds (reference
  /// typed_acquire_timeout_ms): after `ms` milliseconds (0: at once) the call
  /// fails with acquire_timeout; a negative value waits without limit.
  void setAcquireTimeout(int64_t ms) { acquireTimeoutMs_ = ms; }

  ResourceStats stats() const;
  std::optional<TransferError> clear();
  std::optional<TransferError> close();

  /// Keep `anything` (a context, buffer owners) alive until the process
  /// exits: work that may still touch it has no proven completion.
  static void quarantine(std::shared_ptr<void> anything);

private:
  struct Slot {
    std::unique_ptr<CudaBackend> backend;
    std::timed_mutex lease;
    uint64_t lastUse = 0;
  };
  int64_t acquireTimeoutMs_ = -1; // < 0: wait for a leased context without limit
  /// The context of `device`; at the context limit the least recently used
  /// context is retired (its scratch is freed once its current lease ends).
  std::optional<TransferError> acquire(int device, std::shared_ptr<Slot> &slot);
  mutable std::mutex mutex_;
  std::map<int, std::shared_ptr<Slot>> slots_;
  uint64_t clock_ = 0, evictions_ = 0;
  size_t maxRetained_, maxLive_;
  unsigned maxContexts_;
  bool closed_ = false, quarantined_ = false;
  uint64_t requests_ = 0, hits_ = 0, created_ = 0, retired_ = 0;
};

} // namespace dispatch
} // namespace reloc

#endif
