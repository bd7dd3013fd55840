// sym_b200 -- buffer views, transfer options and error/outcome types shared by
// the dispatch layer. Field names and error codes follow the reference's
// libreloc/include/reloc/Transfer.h:31-160 so callers keep their option
// plumbing; `route` is this executor's addition (the H2D data path).
#ifndef SYM_B200_RELOC_TRANSFER_H
#define SYM_B200_RELOC_TRANSFER_H

#include "reloc/Backend.h"
#include "reloc/Bind.h"

#include <cstddef>
#include <cstdint>
#include <optional>
#include <string>
#include <variant>
#include <vector>

namespace reloc {

enum class MemoryKind : uint8_t { Host, Cuda };
enum class TransferDirection : uint8_t { HostToDevice, DeviceToHost };

/// A caller's buffer: the allocation plus the logical view inside it.
struct BufferView {
  uintptr_t base = 0;
  size_t capacityBytes = 0;
  size_t offsetBytes = 0;
  std::vector<int64_t> extents;
  std::vector<int64_t> strides;
  uint32_t elementSize = 0;
  MemoryKind kind = MemoryKind::Host;
  int device = -1;
};

/// Stable code + detail. Codes: invalid_view, unsupported_layout,
/// insufficient_capacity, integer_overflow, plan_mismatch, direction_mismatch,
/// already_executed, device_mismatch, backend_failure, typed_unsupported,
/// invalid_options, resources_closed, completion_unknown,
/// implementation_unavailable, backend_mismatch, and the typed program's
/// execution codes (channel_out_of_range, ...).
struct TransferError {
  std::string code;
  std::string message;
};

enum class TransferCompletion { NotLaunched, Complete, Unknown, Pending };

struct TransferOutcome {
  std::optional<TransferError> error;
  TransferCompletion completion = TransferCompletion::NotLaunched;
};

enum class PinningPolicy { Auto, Pinned, Pageable };

/// H2D data path of the B200 rows.
///   Auto      measured choice per plan shape (cached per context)
///   DmaRing   copy-engine DMA of raw source chunks into an HBM ring,
///             overlapped with the transform kernels on a second stream
///   ZeroCopy  the transform kernels read pinned host memory directly
///   Staged    one DMA of the whole source into HBM, then one kernel
enum class Route { Auto, DmaRing, ZeroCopy, Staged };

struct TransferOptions {
  int nBuffers = 4;             // HBM ring slots (DmaRing)
  size_t chunkSizeOverride = 0; // ring slot bytes; 0 = heuristic
  unsigned gatherThreads = 1;   // accepted for API compatibility (no CPU gather)
  bool hasCallerStream = false;
  const void *callerStream = nullptr; // order after this stream; signal it at the end
  bool directDenseUpload = true;
  bool pipelineTypedH2D = true;
  PinningPolicy pinning = PinningPolicy::Pinned;
  std::optional<size_t> minPinnedBytes;
  size_t maxScratchBytes = 0;
  Route route = Route::Auto;
  /// When true the call returns once the work is enqueued and the caller
  /// stream (if any) is ordered after it; completion is the caller's to
  /// establish through that stream. Default: block until complete.
  bool asyncCompletion = false;
};

// ---- layout-only (wire v0) transfers ------------------------------------------
// The reference's validated forward-transfer API (libreloc/include/reloc/
// Transfer.h:100-200), kept with its names, signatures and error codes so C++
// callers compile unchanged. Execution is the B200 executor's: the bound
// layout plan runs as a stage-free fused kernel on a CudaBackend (host-to-
// device through the HBM DMA ring, device-to-host through the result-row
// ring); any other backend gets `backend_mismatch`.

/// A validated request; owns copies of the plan and both views. Single-use.
struct TransferRequest {
  BoundPlan bound;
  BufferView source;
  BufferView destination;
  TransferDirection direction = TransferDirection::HostToDevice;
  size_t sourceSpanBytes = 0;  // bytes the plan may read from the source's element 0
  size_t destinationBytes = 0; // == bound.totalBytes
  bool consumed = false;
};

/// Bytes a view addresses, elementSize * (1 + sum((extent - 1) * stride)),
/// after rejecting null, empty, negative-stride, broadcast (stride 0) and
/// overlapping views and checking the capacity; every step overflow-checked.
std::variant<size_t, TransferError> viewSpanBytes(const BufferView &view, const char *role);

/// The source half of validateTransfer: the view is admissible for the
/// direction and every source read of the plan lies inside it. Returns the
/// source span in bytes.
std::variant<size_t, TransferError> validateTransferSource(const BoundPlan &bound, const BufferView &source,
                                                           TransferDirection direction);

/// Full validation: the source as above, a dense row-major destination of
/// exactly bound.totalBytes that holds every plan write, both capacities.
std::variant<TransferRequest, TransferError> validateTransfer(const BoundPlan &bound, const BufferView &source,
                                                              const BufferView &destination,
                                                              TransferDirection direction);

/// Execute a validated request and block until its work completed (no
/// device-wide synchronization). The request is re-validated (its public
/// fields may have changed) and marked consumed before any work; a consumed
/// request fails with already_executed. `backend` must be a CudaBackend
/// (backend_mismatch otherwise) of the device end's ordinal
/// (device_mismatch otherwise). Errors are returned, never thrown.
std::optional<TransferError> executeTransfer(TransferRequest &request, CopyBackend &backend,
                                             const TransferOptions &options);


} // namespace reloc

#endif
