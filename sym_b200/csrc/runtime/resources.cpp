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
    // A failed backend call: completion must be proven before anything the
    // work touched may be reused. Proven: the context is retired (freed once
    // this lease ends) and the next call gets a fresh one. Not proven: the
    // context and the owners stay alive for the life of the process and the
    // owner refuses all further work.
    const bool known = slot->backend->quiesce() == QueueCompletion::Complete;
    std::lock_guard<std::mutex> g(mutex_);
    auto it = slots_.find(device);
    if (it != slots_.end() && it->second == slot)
      slots_.erase(it);
    if (known) {
      ++retired_;
    } else {
      out.completion = TransferCompletion::Unknown;
      out.error = terr("completion_unknown", "typed dispatch and its owners were quarantined (" +
                                                 out.error->message + ")");
      quarantined_ = true;
      quarantine(slot);
    }
  }
  return out;
}

void Resources::quarantine(std::shared_ptr<void> keep) {
  // Never freed: work that may still touch these allocations has no proven
  // end (reference: process-lifetime quarantine of the context and owners).
  static auto *kept = new std::vector<std::shared_ptr<void>>();
  static std::mutex m;
  std::lock_guard<std::mutex> g(m);
  kept->push_back(std::move(keep));
}

TransferOutcome Resources::execute(DispatchRequest &request, int device, int /*streams*/,
                                   const TransferOptions &options, std::shared_ptr<void> owners) {
  TransferOutcome out = withContext(
      device, [&](CudaBackend &b) { return executeDispatch(request, b, options); }, !options.asyncCompletion);
  if (out.completion == TransferCompletion::Unknown)
    quarantine(std::move(owners)); // keep the buffers alive for good
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
  std::shared_ptr<FaultWord> fault; // the context's fault word
  TransferOutcome outcome;
  std::shared_ptr<void> owners; // buffers kept alive until completion
  ~State() {
    if (event) {
      if (!finished)
        sbc_event_synchronize(event); // drain before releasing anything
      sbc_event_destroy(event);
    }
  }
  /// Finalize after the event completed: the context's fault word (plain
  /// host memory, written by any kernel of the group whose wait ran out).
  void finalizeLocked() {
    finished = true;
    outcome.completion = TransferCompletion::Complete;
    if (fault && fault->take())
      outcome.error = terr("backend_failure", "a kernel's bounded wait for a TMA copy ran out; the output is incomplete");
    owners.reset();
  }
  /// The event could not be waited for: completion is unknown, and the
  /// owners are kept for the life of the process.
  void unknownLocked(int rc) {
    finished = true;
    outcome.error = terr("completion_unknown", std::string("completion: ") + sbc_error_string(rc));
    outcome.completion = TransferCompletion::Unknown;
    Resources::quarantine(std::move(owners));
  }
};

Completion::Completion(std::shared_ptr<State> state) : state_(std::move(state)) {}

Completion::~Completion() {
  if (state_) {
    std::lock_guard<std::mutex> g(state_->m);
    if (!state_->finished && state_->event) {
      const int rc = sbc_event_synchronize(state_->event);
      if (rc)
        state_->unknownLocked(rc);
      else
        state_->finalizeLocked();
    }
  }
}

TransferOutcome Completion::wait() {
  std::lock_guard<std::mutex> g(state_->m);
  if (!state_->finished) {
    const int rc = sbc_event_synchronize(state_->event);
    if (rc)
      state_->unknownLocked(rc);
    else
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
  if (rc)
    state_->unknownLocked(rc);
  else
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
  if (out.completion == TransferCompletion::Unknown)
    quarantine(std::move(owners));
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
    state->fault = b.faultShared();
    return executeGroup(group, b, o, state->event);
  }, false);
  if (out.error) {
    if (out.completion == TransferCompletion::Unknown)
      quarantine(std::move(owners));
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
  s.retirements = retired_;
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
