// sym_b200 -- buffer views, transfer options and error/outcome types shared by
// the dispatch layer. Field names and error codes follow the reference's
// libreloc/include/reloc/Transfer.h:31-160 so callers keep their option
// plumbing; `route` is this executor's addition (the H2D data path).
#ifndef SYM_B200_RELOC_TRANSFER_H
#define SYM_B200_RELOC_TRANSFER_H

#include <cstddef>
#include <cstdint>
#include <optional>
#include <string>
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


} // namespace reloc

#endif
