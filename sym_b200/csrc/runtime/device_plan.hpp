// Lowering of a checked typed program to the fused device kernels, and the
// H2D execution engine (DMA ring, zero copy, staged) built on it.
#ifndef SYM_B200_DEVICE_PLAN_HPP
#define SYM_B200_DEVICE_PLAN_HPP

#include "reloc/CudaBackend.h"
#include "reloc/Dispatch.h"
#include "reloc/TypedExecute.h"

#include "sb_cuda.h"

#include <map>
#include <memory>
#include <mutex>
#include <optional>
#include <string>
#include <variant>
#include <vector>

namespace reloc {
namespace b200 {

enum class Family { Generic = 0, Contiguous = 1, Transpose = 2, Runs = 3 };
const char *familyName(Family f);
/// Launch the family kernel for `d` on `stream`, falling back to the generic
/// kernel when the family's kernel does not take the descriptor.
int launchFamily(Family f, const sbc_relocate &d, void *stream);

/// Device copies of a lowered program's parameter blob, one per device,
/// uploaded on first use and freed with the program. A bound program's
/// parameters are an immutable snapshot, so every execution on a device
/// reuses the same copy (no per-call upload, no host sync).
struct ParamCache {
  std::mutex mutex;
  std::map<int, void *> device;
  ~ParamCache();
};

/// A program in device-ready form. `desc` carries the full padded box and
/// everything but pointers; parameter arrays are packed into `paramBlob`.
struct Lowered {
  std::shared_ptr<ParamCache> params = std::make_shared<ParamCache>();
  sbc_relocate desc{};
  Family family = Family::Generic;
  int64_t padded[SBC_MAX_RANK] = {};
  bool denseCover = false;  // dst strides are dense row-major over the padded box
  int srcOuter = -1;        // axis whose source rows are contiguous blocks
  bool rowsChunkable = false;
  int64_t srcElements = 0;  // dense source elements
  int64_t dstElements = 0;
  bool needsStatus = false; // a channel map is checked on the device
  std::vector<uint8_t> paramBlob;
  std::vector<size_t> paramOffset, zpOffset; // per stage, SIZE_MAX = none
  std::string classKey; // route-measurement class
};

std::variant<Lowered, TransferError> lower(const typed::Program &program);

/// A window of physical (padded) rows of axis 0; {0, padded[0]} = whole.
struct RowWindow {
  int64_t begin = 0, end = -1;
};

struct RunStats {
  std::string route, kernel;
  uint64_t launches = 0, copies = 0;
  size_t chunks = 0, chunkBytes = 0, buffers = 0;
  int64_t payloadBytes = 0;
};

/// Device source: the transform alone (source already in HBM). Enqueued on
/// the backend's compute stream.
std::optional<TransferError> runDevice(const Lowered &l, CudaBackend &b, const void *dsrc, void *ddst,
                                       RowWindow window, RunStats &stats);

/// Host source -> device destination through `route` (Auto resolved by the
/// caller). Enqueued on the backend's streams; the caller orders/blocks.
std::optional<TransferError> runH2D(const Lowered &l, CudaBackend &b, const void *hsrc, void *ddst, Route route,
                                    RowWindow window, const TransferOptions &options, RunStats &stats);

/// Device source -> host destination: the fused kernel writes chunks of
/// result rows into the HBM ring (or, zero copy, straight into mapped pinned
/// host memory) and the copy engine drains each chunk to the host. Enqueued
/// on the backend's streams; the caller orders/blocks.
std::optional<TransferError> runD2H(const Lowered &l, CudaBackend &b, const void *dsrc, void *hdst, Route route,
                                    const TransferOptions &options, RunStats &stats);

/// A window of source rows (the plan's source-outer axis) held in device
/// memory -- this GPU's or a peer's through an IPC mapping: `rows` points at
/// source row `rowBegin`; the kernel writes exactly the result cells rows
/// [rowBegin, rowEnd) produce (plus the pad rows before the first / after
/// the last row) into the full destination `ddst`.
std::optional<TransferError> runSourceRows(const Lowered &l, CudaBackend &b, const void *rows, int64_t rowBegin,
                                           int64_t rowEnd, void *ddst, RunStats &stats);

/// All of a plan's source rows, held as `n` consecutive blocks in device
/// memory (this GPU's or peers'): block j is `shards[j]` with rows
/// [bounds[j], bounds[j + 1]); bounds[0] = 0 and bounds[n] = the row count.
/// One tile launch reads every block when the plan and the blocks fit the
/// TMA tile kernel, else one launch per block.
std::optional<TransferError> runSourceShards(const Lowered &l, CudaBackend &b, const void *const *shards,
                                             const int64_t *bounds, int n, void *ddst, RunStats &stats);

/// Route::Auto for a device-to-host execution: the DMA ring when the result
/// splits into row chunks, else zero copy into pinned memory, else staged.
Route chooseRouteD2H(const Lowered &l, void *hdst, const TransferOptions &options);

/// Host source -> device destination on the caller's `stream` through the
/// statically allocated scratch `scratch` (`scratchBytes`), allocating
/// nothing: parameters and one staging slot live in the scratch, chunks of
/// source rows are copied and transformed in stream order.
std::optional<TransferError> runH2DStatic(const Lowered &l, const void *hsrc, void *ddst, void *stream,
                                          uint8_t *scratch, size_t scratchBytes);

/// Resolve Route::Auto for this plan class on this backend (measurement-
/// driven; see dispatch.cpp).
Route chooseRoute(const Lowered &l, CudaBackend &b, const void *hsrc, const TransferOptions &options);

/// Upload the parameter blob and patch the stage pointers of `desc`.
std::optional<TransferError> uploadParams(const Lowered &l, CudaBackend &b, sbc_relocate &desc);

} // namespace b200
} // namespace reloc

#endif
