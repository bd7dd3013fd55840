// Typed contexts; see include/reloc/DispatchResources.h.
#include "reloc/DispatchResources.h"

namespace reloc {
namespace dispatch {
namespace {
TransferError terr(const char *code, std::string msg) { return TransferError{code, std::move(msg)}; }
} // namespace

Resources::Resources(size_t maxRetainedBytes, size_t maxLiveBytes, unsigned maxContexts)
    : maxRetained_(maxRetainedBytes), maxLive_(maxLiveBytes), maxContexts_(maxContexts ? maxContexts : 1) {}

Resources::~Resources() { close(); }

std::optional<TransferError> Resources::acquire(int device, Slot *&slot) {
  std::lock_guard<std::mutex> g(mutex_);
  if (closed_)
    return terr("resources_closed", "typed resources are closed");
  if (quarantined_)
    return terr("completion_unknown", "typed resources are quarantined after an unknown completion");
  ++requests_;
  auto it = slots_.find(device);
  if (it != slots_.end()) {
    ++hits_;
    slot = it->second.get();
    return std::nullopt;
  }
  if (slots_.size() >= maxContexts_)
    return terr("invalid_options", "context limit reached (" + std::to_string(maxContexts_) + ")");
  std::string err;
  auto b = CudaBackend::create(device, err);
  if (!b)
    return terr("backend_failure", err);
  auto s = std::make_unique<Slot>();
  s->backend = std::move(b);
  slot = s.get();
  slots_[device] = std::move(s);
  ++created_;
  return std::nullopt;
}

TransferOutcome Resources::withContext(int device,
                                       const std::function<std::optional<TransferError>(CudaBackend &)> &fn) {
  TransferOutcome out;
  Slot *slot = nullptr;
  if (auto e = acquire(device, slot)) {
    out.error = e;
    return out;
  }
  std::lock_guard<std::mutex> lease(slot->lease); // FIFO per context
  out.error = fn(*slot->backend);
  out.completion = TransferCompletion::Complete;
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
  TransferOutcome out = withContext(device, [&](CudaBackend &b) { return executeDispatch(request, b, options); });
  if (out.completion == TransferCompletion::Unknown) {
    std::lock_guard<std::mutex> g(mutex_);
    quarantinedOwners_.push_back(std::move(owners)); // keep buffers alive for good
  }
  if (!out.error && options.asyncCompletion)
    out.completion = TransferCompletion::Pending;
  return out;
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
    s.copyCalls += b.copyCalls;
    s.eventRecords += b.eventRecords;
    s.eventWaits += b.eventWaits;
    s.callerWaits += b.callerWaits;
    s.kernelLaunches += b.kernelLaunches;
  }
  s.retainedBytes = s.deviceBytes;
  return s;
}

std::optional<TransferError> Resources::clear() {
  std::lock_guard<std::mutex> g(mutex_);
  if (quarantined_)
    return terr("completion_unknown", "quarantined resources are never released");
  for (auto &kv : slots_)
    std::lock_guard<std::mutex> lease(kv.second->lease);
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
