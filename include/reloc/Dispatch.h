// sym_b200 -- plan-driven typed dispatch onto the B200 rows.
//
// Same entry points, request/template/report types and policy vocabulary as
// the reference's libreloc/include/reloc/Dispatch.h:100-271
// (queryCapability :100, prepareDispatchTemplate/prepareDispatch :170-175,
// executeDispatch :269). The capability table is new: every supported typed
// plan is eligible for the B200 rows, which do all value work on the GPU and
// fuse it into the host->device transfer:
//   b200_fused_h2d            route chosen per plan (Route::Auto or options)
//   b200_fused_h2d@dma_ring   raw source chunks DMA'd into an HBM ring, then
//                             the fused transform kernel per chunk
//   b200_fused_h2d@zero_copy  the fused kernel reads pinned host memory
//   b200_fused_d2h            device source -> host destination: the fused
//                             kernel writes result-row chunks into the HBM
//                             ring, the copy engine drains them to the host
//                             (@dma_ring), or the kernel writes mapped pinned
//                             host memory directly (@zero_copy)
// The reference's CPU rows (cpu_reference, cpu_stages_cuda_stages@k) and its
// legacy CUDA rows are listed as excluded with a reason: no supported plan
// executes on the CPU here.
#ifndef SYM_B200_RELOC_DISPATCH_H
#define SYM_B200_RELOC_DISPATCH_H

#include "reloc/Transfer.h"
#include "reloc/TypedExecute.h"

#include <cstdint>
#include <memory>
#include <optional>
#include <string>
#include <variant>
#include <vector>

namespace reloc {

class CudaBackend;
namespace b200 {
struct Lowered;
}

namespace dispatch {

enum class Policy { OriginalCpu, Auto };

inline constexpr const char *kB200FusedH2D = "b200_fused_h2d";
inline constexpr const char *kB200FusedD2H = "b200_fused_d2h";
inline constexpr const char *kCpuReference = "cpu_reference";
inline constexpr const char *kCpuStagesCudaStages = "cpu_stages_cuda_stages";
inline constexpr const char *kCudaStagesThenCpu = "cuda_stages_then_cpu";
inline constexpr const char *kCudaDequantRelocate = "cuda_dequant_relocate";
inline constexpr const char *kCudaRelocateF32 = "cuda_relocate_f32";

struct Implementation {
  std::string id;
  std::string variant; // "", "dma_ring" or "zero_copy"
  uint32_t wireBoundary = 0;
  bool wireResultLayout = false;
  int64_t wireBytes = 0;
  int64_t deviceTempBytes = 0;
  std::string method;
  std::string label() const { return variant.empty() ? id : id + "@" + variant; }
};

struct Exclusion {
  std::string id;
  std::string reason;
};

struct Capability {
  std::vector<Implementation> eligible;
  std::vector<Exclusion> excluded;
};

/// Pure: which rows can run `program` in `direction` with a CUDA device end.
Capability queryCapability(const typed::Program &program, TransferDirection direction, bool cuda);

struct Report {
  std::string implementation;
  std::string policy;
  std::string placementReason;
  std::string method;
  uint32_t wireBoundary = 0;
  int64_t sourceBytes = 0;
  int64_t wireBytes = 0;
  int64_t destinationBytes = 0;
  int64_t parameterBytes = 0;
  int64_t payloadBytesTransferred = 0;
  int64_t deviceTempBytes = 0;
  uint32_t artifactVersion = 1;
  bool executed = false;
  std::string hostPipeline = "not_applicable";
  std::string hostKernel = "not_applicable";
  size_t hostChunks = 0, hostChunkBytes = 0, hostBuffers = 0;
  // B200 additions
  std::string route;        // "dma_ring", "zero_copy" or "staged"
  std::string deviceKernel; // "contiguous", "transpose" or "generic"
  uint64_t kernelLaunches = 0;
  uint64_t copyCalls = 0;
};

struct Options {
  Policy policy = Policy::Auto;
  int threads = 8;
  bool cuda = false;
  std::string implementation; // explicit row label
};

struct DispatchRequest {
  typed::Program program;
  BufferView source;
  BufferView destination;
  TransferDirection direction = TransferDirection::HostToDevice;
  Implementation selected;
  Report report;
  bool consumed = false;
  bool executing = false;
  /// The program lowered to device kernels (shared with the template).
  std::shared_ptr<const b200::Lowered> lowered;
};

struct Selection {
  Implementation row;
  std::string policy;
  std::string reason;
};

struct DispatchTemplate {
  typed::Program program;
  Capability capability;
  Selection selection;
  TransferDirection direction = TransferDirection::HostToDevice;
  bool cuda = false;
  std::shared_ptr<const b200::Lowered> lowered;
};

std::variant<Selection, TransferError> selectImplementation(const typed::Program &, TransferDirection,
                                                            const Options &);
std::variant<DispatchTemplate, TransferError> prepareDispatchTemplate(const TypedBoundPlan &, TransferDirection,
                                                                      const Options &);
std::variant<DispatchRequest, TransferError> prepareDispatch(const DispatchTemplate &, const BufferView &source,
                                                             const BufferView &destination);
std::variant<DispatchRequest, TransferError> prepareDispatch(const TypedBoundPlan &plan, const BufferView &source,
                                                             const BufferView &destination,
                                                             TransferDirection direction, const Options &options);

/// The CUDA device a request runs on: the destination's (H2D) or the
/// source's (D2H).
int executionDevice(const DispatchRequest &request);

/// Run the selected row on `backend` (one device's streams, HBM ring and
/// parameter buffers). Blocks until this request's work completed unless
/// options.asyncCompletion. Marks the request consumed before launching.
std::optional<TransferError> executeDispatch(DispatchRequest &request, CudaBackend &backend,
                                             const TransferOptions &options);
/// The reference's signature (Dispatch.h:269): every B200 row needs a
/// CudaBackend; any other CopyBackend gets backend_mismatch before any work
/// (the request stays unconsumed).
std::optional<TransferError> executeDispatch(DispatchRequest &request, CopyBackend &backend,
                                             const TransferOptions &options);

/// A layout-only (wire v0) bound plan as a stage-free dispatch template: the
/// source is the dense 1-D span the plan reads (its element 0 is the view's
/// element 0), the result the dense padded destination. Used by
/// executeTransfer and by the C-ABI's layout transfers.
std::variant<DispatchTemplate, TransferError> prepareTransferTemplate(const BoundPlan &bound,
                                                                      TransferDirection direction);

/// Execute the physical row window [rowBegin, rowEnd) of axis 0 of the
/// padded result (a shard of the result, e.g. one GPU's rows of a sharded
/// weight fetch). `dst` is the window's own storage; channels keep their
/// global coordinates (the reference's executeHostChunk contract,
/// libreloc/include/reloc/TypedExecute.h:160-170). `hostSource` selects the
/// H2D routes; otherwise `src` is already in this device's memory and only
/// the transform runs.
std::optional<TransferError> executeWindow(const DispatchTemplate &tmpl, CudaBackend &backend, const void *src,
                                           bool hostSource, void *dst, int64_t rowBegin, int64_t rowEnd,
                                           const TransferOptions &options, Report &report);

/// The source-row counterpart of executeWindow: `rows` (device memory of
/// this GPU, or a peer GPU's mapped into this process) holds source rows
/// [rowBegin, rowEnd) of the plan's source-outer axis; the transform writes
/// the result cells those rows produce into the full destination `dst`.
/// Disjoint row windows, possibly from different GPUs, assemble the result.
std::optional<TransferError> executeSourceRows(const DispatchTemplate &tmpl, CudaBackend &backend, const void *rows,
                                               int64_t rowBegin, int64_t rowEnd, void *dst,
                                               const TransferOptions &options, Report &report);

/// All source rows as `n` blocks (block j at `shards[j]`, rows
/// [bounds[j], bounds[j + 1])), each in device memory of this GPU or a peer;
/// the whole result is written to `dst`, in one launch where possible.
std::optional<TransferError> executeSourceShards(const DispatchTemplate &tmpl, CudaBackend &backend,
                                                 const void *const *shards, const int64_t *bounds, int n, void *dst,
                                                 const TransferOptions &options, Report &report);

/// Explicit consumer-sized group (reference Dispatch.h:177-214,
/// prepareDispatchGroup :213): fresh views per member, one CUDA device, one
/// caller-stream ordering and one completion for all members. Typed
/// templates and layout plans (through their transfer template) mix freely.
struct GroupEntry {
  const DispatchTemplate *plan = nullptr; // read during preparation only
  BufferView source, destination;
  TransferDirection direction = TransferDirection::HostToDevice;
};
struct GroupReport {
  uint64_t payloadCopyCalls = 0, parameterUploads = 0, parameterReuses = 0;
  uint64_t parameterUploadBytes = 0, hostTransformBytes = 0;
  uint64_t packingBytes = 0; // payloads are never packed together
  uint64_t kernelLaunches = 0, outputBytes = 0;
  uint64_t copyCalls = 0, eventRecords = 0, eventWaits = 0, callerWaits = 0;
  size_t scratchPeakBytes = 0;
};
struct GroupRequest {
  std::vector<DispatchRequest> items;
  std::vector<Report> reports;
  GroupReport report;
  int device = -1;
  bool consumed = false, executing = false, failed = false;
};
/// Validate the whole group before anything is allocated or launched: 1 to
/// 256 members, host-to-device only, one destination device, and no
/// destination overlapping another member's destination or any source.
std::variant<GroupRequest, TransferError> prepareDispatchGroup(const std::vector<GroupEntry> &entries);
/// Enqueue every member on `backend` after one wait on the caller stream,
/// then order the caller stream after all of them. Blocks until the group
/// completed unless options.asyncCompletion; `completionEvent` (an event of
/// the sb_cuda layer, or null) is recorded after the last member either way.
/// Marks the group consumed before launching; never retries a member.
std::optional<TransferError> executeGroup(GroupRequest &group, CudaBackend &backend, const TransferOptions &options,
                                          void *completionEvent);

} // namespace dispatch
} // namespace reloc

#endif
