// Typed contexts; see include/reloc/DispatchResources.h.
#include "reloc/DispatchResources.h"

#include "sb_cuda.h"

#include <algorithm>
#include <chrono>

namespace reloc {
namespace dispatch {
namespace {
TransferError terr(const char *code, std::string msg) { return TransferError{code, std::move(msg)}; }
} // namespace

Resources::Resources(size_t maxRetainedBytes, size_t maxLiveBytes, unsigned maxContexts)
    : maxRetained_(maxRetainedBytes), maxLive_(maxLiveBytes), maxContexts_(maxContexts ? maxContexts : 1) {}

Resources::~Resources() { close(); }

std::optional<TransferError> Resources::acquire(int device, std::shared_ptr<Slot> &slot) {
  std::shared_ptr<Slot> retired; // destroyed (drained, freed) outside the lock
  std::lock_guard<std::mutex> g(mutex_);
  if (closed_)
    return terr("resources_closed", "typed resources are closed");
  if (quarantined_)
    return terr("completion_unknown", "typed resources are quarantined after an unknown completion");
  ++requests_;
  auto it = slots_.find(device);
  if (it != slots_.end()) {
    ++hits_;
    it->second->lastUse = ++clock_;
    slot = it->second;
    return std::nullopt;
  }
  if (slots_.size() >= maxContexts_) {
    auto victim = slots_.begin();
    for (auto v = slots_.begin(); v != slots_.end(); ++v)
      if (v->second->lastUse < victim->second->lastUse)
        victim = v;
    retired = std::move(victim->second); // a lease in progress keeps it alive until it ends
    slots_.erase(victim);
    ++evictions_;
  }
  std::string err;
  auto b = CudaBackend::create(device, err);
  if (!b)
    return terr("backend_failure", err);
  // The owner's scratch limits divided into fixed per-context quotas (the
  // first contexts take the remainder).
  const size_t k = slots_.size();
  auto quota = [&](size_t limit) { return limit / maxContexts_ + (k < limit % maxContexts_ ? 1 : 0); };
  b->retainedLimit = quota(maxRetained_);
  b->liveLimit = maxLive_ ? std::max<size_t>(quota(maxLive_), 1) : 0;
  auto s = std::make_shared<Slot>();
  s->backend = std::move(b);
  s->lastUse = ++clock_;
  slot = s;
  slots_[device] = std::move(s);
  ++created_;
  return std::nullopt;
}

TransferOutcome Resources::withContext(int device,
                                       const std::function<std::optional<TransferError>(CudaBackend &)> &fn,
                                       bool releaseAfter) {
  TransferOutcome out;
  // The work runs with the context's device current; the caller's current
  // device is put back afterwards (callers may target a GPU that is not
  // their current one).
  int callerDevice = -1;
  sbc_get_device(&callerDevice);
  struct Restore {
    int device;
    ~Restore() {
      int now = -1;
      if (device >= 0 && sbc_get_device(&now) == 0 && now != device)
        sbc_set_device(device);
    }
  } restore{callerDevice};
  std::shared_ptr<Slot> slot;
  if (auto e = acquire(device, slot)) {
    out.error = e;
    return out;
  }
  std::unique_lock<std::timed_mutex> lease(slot->lease, std::defer_lock); // one call at a time per context
  if (acquireTimeoutMs_ < 0) {
    lease.lock();
  } else if (!lease.try_lock_for(std::chrono::milliseconds(acquireTimeoutMs_))) {
    out.error = terr("acquire_timeout", "typed context admission timed out");
    return out;
  }
  out.error = fn(*slot->backend);
  out.completion = TransferCompletion::Complete;
  // Idle scratch beyond the retained quota is released at the end of a
  // blocking lease (its work has completed, so nothing waits on it).
  if (releaseAfter && !slot->backend->failed())
    slot->backend->trim(slot->backend->retainedLimit);
  if (out.error && slot->backend->failed()) {
    // A failed CUDA call leaves completion unknown: retire the context.
    if (slot->backend->quiesce() != QueueCompletion::Complete) {
      out.completion = TransferCompletion::Unknown;
      std::lock_guard<std::mutex> g(mutex_);
      quarantined_ = true;
    }
  }
  return out;
}

TransferOutcome Resources::execute(DispatchRequest &request, int device, int /*streams*/,
                                   const TransferOptions &options, std::shared_ptr<void> owners) {
  TransferOutcome out = withContext(
      device, [&](CudaBackend &b) { return executeDispatch(request, b, options); }, !options.asyncCompletion);
  if (out.completion == TransferCompletion::Unknown) {
    std::lock_guard<std::mutex> g(mutex_);
    quarantinedOwners_.push_back(std::move(owners)); // keep buffers alive for good
  }
  if (!out.error && options.asyncCompletion)
    out.completion = TransferCompletion::Pending;
  return out;
}

// ---- groups and completions ---------------------------------------------------

struct Completion::State {
  std::mutex m;
  void *event = nullptr;
  int device = -1;
  bool finished = false;
  uint64_t waitsBefore = 0; // sbc_wait_launch_count() before the work was enqueued
  TransferOutcome outcome;
  std::shared_ptr<void> owners; // buffers kept alive until completion
  ~State() {
    if (event) {
      if (!finished)
        sbc_event_synchronize(event); // drain before releasing anything
      sbc_event_destroy(event);
    }
  }
  /// Finalize after the event completed: the device's fault word.
  void finalizeLocked() {
    finished = true;
    if (sbc_wait_launch_count() == waitsBefore) { // no kernel that writes the fault word ran
      outcome.completion = TransferCompletion::Complete;
      owners.reset();
      return;
    }
    int fault = 0;
    int dev = -1;
    sbc_get_device(&dev);
    if (dev != device)
      sbc_set_device(device);
    const int rc = sbc_device_fault(&fault);
    if (dev != device && dev >= 0)
      sbc_set_device(dev);
    if (rc) {
      outcome.error = terr("backend_failure", std::string("fault word: ") + sbc_error_string(rc));
      outcome.completion = TransferCompletion::Unknown;
    } else if (fault) {
      outcome.error = terr("backend_failure", "a kernel's bounded wait for a TMA copy ran out; the output is incomplete");
      outcome.completion = TransferCompletion::Complete;
    } else {
      outcome.completion = TransferCompletion::Complete;
    }
    owners.reset();
  }
};

Completion::Completion(std::shared_ptr<State> state) : state_(std::move(state)) {}

Completion::~Completion() {
  if (state_) {
    std::lock_guard<std::mutex> g(state_->m);
    if (!state_->finished && state_->event && sbc_event_synchronize(state_->event) == 0)
      state_->finalizeLocked();
  }
}

TransferOutcome Completion::wait() {
  std::lock_guard<std::mutex> g(state_->m);
  if (!state_->finished) {
    const int rc = sbc_event_synchronize(state_->event);
    if (rc) {
      state_->finished = true;
      state_->outcome.error = terr("backend_failure", std::string("completion: ") + sbc_error_string(rc));
      state_->outcome.completion = TransferCompletion::Unknown; // owners stay referenced for good
      return state_->outcome;
    }
    state_->finalizeLocked();
  }
  return state_->outcome;
}

std::variant<bool, TransferError> Completion::query() {
  std::lock_guard<std::mutex> g(state_->m);
  if (state_->finished) {
    if (state_->outcome.error)
      return *state_->outcome.error;
    return true;
  }
  const int rc = sbc_event_query(state_->event);
  if (rc == 1)
    return false;
  if (rc) {
    state_->finished = true;
    state_->outcome.error = terr("backend_failure", std::string("completion: ") + sbc_error_string(rc));
    state_->outcome.completion = TransferCompletion::Unknown;
    return *state_->outcome.error;
  }
  state_->finalizeLocked();
  if (state_->outcome.error)
    return *state_->outcome.error;
  return true;
}

std::optional<TransferError> Completion::waitStream(const void *consumer) {
  std::lock_guard<std::mutex> g(state_->m);
  if (state_->finished && state_->outcome.error)
    return state_->outcome.error;
  const int rc = sbc_stream_wait_event(const_cast<void *>(consumer), state_->event);
  if (rc)
    return terr("backend_failure", std::string("cudaStreamWaitEvent(consumer): ") + sbc_error_string(rc));
  return std::nullopt;
}

TransferOutcome Resources::execute(GroupRequest &group, const TransferOptions &options, std::shared_ptr<void> owners) {
  if (group.consumed) {
    TransferOutcome out;
    out.error = terr("already_executed", "dispatch groups are single-use");
    return out;
  }
  TransferOutcome out = withContext(
      group.device, [&](CudaBackend &b) { return executeGroup(group, b, options, nullptr); },
      !options.asyncCompletion);
  if (out.completion == TransferCompletion::Unknown) {
    std::lock_guard<std::mutex> g(mutex_);
    quarantinedOwners_.push_back(std::move(owners));
  }
  if (!out.error && options.asyncCompletion)
    out.completion = TransferCompletion::Pending;
  return out;
}

std::variant<std::shared_ptr<Completion>, TransferError>
Resources::submit(GroupRequest &group, const TransferOptions &options, std::shared_ptr<void> owners) {
  if (group.consumed)
    return terr("already_executed", "dispatch groups are single-use");
  auto state = std::make_shared<Completion::State>();
  state->device = group.device;
  TransferOptions o = options;
  o.asyncCompletion = true;
  TransferOutcome out = withContext(group.device, [&](CudaBackend &b) -> std::optional<TransferError> {
    if (!b.activate())
      return terr("backend_failure", b.error());
    const int rc = sbc_event_create(&state->event, 0);
    if (rc) {
      state->event = nullptr;
      return terr("backend_failure", std::string("cudaEventCreate: ") + sbc_error_string(rc));
    }
    state->waitsBefore = sbc_wait_launch_count();
    return executeGroup(group, b, o, state->event);
  }, false);
  if (out.error) {
    if (out.completion == TransferCompletion::Unknown) {
      std::lock_guard<std::mutex> g(mutex_);
      quarantinedOwners_.push_back(std::move(owners));
    }
    return *out.error;
  }
  state->owners = std::move(owners);
  return std::make_shared<Completion>(std::move(state));
}

ResourceStats Resources::stats() const {
  std::lock_guard<std::mutex> g(mutex_);
  ResourceStats s;
  s.requests = requests_;
  s.hits = hits_;
  s.contexts = slots_.size();
  s.deviceAllocations = created_;
  s.closed = closed_;
  s.quarantined = quarantined_;
  s.retainedLimit = maxRetained_;
  s.liveLimit = maxLive_;
  s.contextLimit = maxContexts_;
  for (const auto &kv : slots_) {
    const CudaBackend &b = *kv.second->backend;
    s.deviceBytes += b.deviceBytes();
    s.peakLiveBytes += b.peakDeviceBytes;
    s.releases += b.trims;
    s.copyCalls += b.copyCalls;
    s.eventRecords += b.eventRecords;
    s.eventWaits += b.eventWaits;
    s.callerWaits += b.callerWaits;
    s.kernelLaunches += b.kernelLaunches;
  }
  s.evictions = evictions_;
  s.retainedBytes = s.deviceBytes;
  return s;
}

std::optional<TransferError> Resources::clear() {
  std::lock_guard<std::mutex> g(mutex_);
  if (quarantined_)
    return terr("completion_unknown", "quarantined resources are never released");
  for (auto &kv : slots_)
    std::lock_guard<std::timed_mutex> lease(kv.second->lease);
  slots_.clear();
  return std::nullopt;
}

std::optional<TransferError> Resources::close() {
  {
    std::lock_guard<std::mutex> g(mutex_);
    if (closed_)
      return quarantined_ ? std::optional<TransferError>(terr("completion_unknown", "quarantined")) : std::nullopt;
    closed_ = true;
    if (quarantined_)
      return terr("completion_unknown", "quarantined resources are never released");
  }
  std::lock_guard<std::mutex> g(mutex_);
  slots_.clear();
  return std::nullopt;
}

} // namespace dispatch
} // namespace reloc
