// Layout-only (wire v0) transfers: view validation and execution on a
// CudaBackend; see include/reloc/Transfer.h. The admitted views, the checks
// and their error codes follow the reference's contract
// (libreloc/src/Transfer.cpp:65-290, executeTransfer :493): views are
// non-empty with non-negative, non-broadcast, non-overlapping strides; the
// plan's reads must lie in the source span and its writes in a dense
// destination of exactly the plan's byte count. Execution differs: the plan
// runs as a stage-free fused kernel on the GPU instead of a host gather.
#include "reloc/Transfer.h"

#include "reloc/CudaBackend.h"
#include "reloc/Dispatch.h"

#include <algorithm>
#include <limits>

namespace reloc {
namespace {

TransferError terr(const char *code, std::string msg) { return TransferError{code, std::move(msg)}; }

bool mulChecked(int64_t a, int64_t b, int64_t &out) { return !__builtin_mul_overflow(a, b, &out); }
bool addChecked(int64_t a, int64_t b, int64_t &out) { return !__builtin_add_overflow(a, b, &out); }

std::string capitalized(const char *role) {
  std::string s(role ? role : "view");
  if (!s.empty() && s[0] >= 'a' && s[0] <= 'z')
    s[0] = static_cast<char>(s[0] - 'a' + 'A');
  return s;
}

/// Elements of `extents` (all >= 1 after viewSpanBytes), overflow-checked.
bool elements(const std::vector<int64_t> &extents, int64_t &out) {
  out = 1;
  for (int64_t e : extents)
    if (!mulChecked(out, e, out))
      return false;
  return true;
}

/// Row-major dense with respect to its own extents (unit axes ignored).
bool dense(const BufferView &v) {
  int64_t expect = 1;
  for (size_t k = v.extents.size(); k-- > 0;) {
    if (v.extents[k] != 1 && v.strides[k] != expect)
      return false;
    if (!mulChecked(expect, v.extents[k], expect))
      return false;
  }
  return true;
}

std::optional<TransferError> kindsFit(const BufferView *source, const BufferView *destination,
                                      TransferDirection direction) {
  // The device end of a transfer is CUDA memory; the other end is host memory.
  if (direction == TransferDirection::HostToDevice && source && source->kind == MemoryKind::Cuda)
    return terr("direction_mismatch", "a host-to-device source must be host memory");
  if (direction == TransferDirection::DeviceToHost && destination && destination->kind == MemoryKind::Cuda)
    return terr("direction_mismatch", "a device-to-host destination must be host memory");
  return std::nullopt;
}

std::optional<TransferError> planReadsFit(const BoundPlan &b, const BufferView &source, size_t spanBytes) {
  if (b.extents.empty() || b.extents.size() != b.srcStrides.size() || b.extents.size() != b.dstStrides.size())
    return terr("plan_mismatch", "bound plan has inconsistent axes");
  if (b.typed)
    return terr("typed_unsupported", "bound plan is the layout of a typed plan; run it through typed dispatch");
  if (b.elementSize == 0 || b.elementSize != source.elementSize)
    return terr("plan_mismatch", "the plan's element size differs from the source view's");
  int64_t planCells = 0, viewCells = 0;
  if (!elements(b.extents, planCells) || !elements(source.extents, viewCells))
    return terr("integer_overflow", "element count overflows");
  if (planCells != viewCells)
    return terr("plan_mismatch", "the plan moves " + std::to_string(planCells) + " elements, the source view holds " +
                                     std::to_string(viewCells));
  int64_t last = 0; // largest element offset the plan reads
  for (size_t k = 0; k < b.extents.size(); ++k) {
    if (b.srcStrides[k] < 0)
      return terr("plan_mismatch", "the plan has a negative source stride");
    int64_t reach = 0;
    if (!mulChecked(b.extents[k] - 1, b.srcStrides[k], reach) || !addChecked(last, reach, last))
      return terr("integer_overflow", "the plan's source reach overflows");
  }
  int64_t need = 0;
  if (!mulChecked(last + 1, static_cast<int64_t>(b.elementSize), need))
    return terr("integer_overflow", "the plan's source footprint overflows");
  if (static_cast<size_t>(need) > spanBytes)
    return terr("plan_mismatch", "the plan reads " + std::to_string(need) + " bytes; the source view spans " +
                                     std::to_string(spanBytes));
  return std::nullopt;
}

std::optional<TransferError> planWritesFit(const BoundPlan &b, const BufferView &destination, size_t spanBytes) {
  if (b.elementSize != destination.elementSize)
    return terr("plan_mismatch", "the plan's element size differs from the destination view's");
  if (!dense(destination))
    return terr("unsupported_layout", "the destination view must be dense row-major");
  if (b.totalBytes <= 0)
    return terr("plan_mismatch", "the bound plan has no destination footprint");
  if (spanBytes != static_cast<size_t>(b.totalBytes))
    return terr("plan_mismatch", "the destination view spans " + std::to_string(spanBytes) +
                                     " bytes; the plan writes " + std::to_string(b.totalBytes));
  std::vector<int64_t> padded = b.extents;
  for (const PadRegion &p : b.padRegions) {
    if (p.axis >= padded.size() || p.lo < 0 || p.hi < 0)
      return terr("plan_mismatch", "the bound plan has an invalid pad region");
    if (!addChecked(padded[p.axis], p.lo, padded[p.axis]) || !addChecked(padded[p.axis], p.hi, padded[p.axis]))
      return terr("integer_overflow", "a padded extent overflows");
  }
  int64_t last = 0;
  for (size_t k = 0; k < padded.size(); ++k) {
    if (b.dstStrides[k] < 0)
      return terr("plan_mismatch", "the plan has a negative destination stride");
    int64_t reach = 0;
    if (!mulChecked(padded[k] - 1, b.dstStrides[k], reach) || !addChecked(last, reach, last))
      return terr("integer_overflow", "the plan's destination reach overflows");
  }
  int64_t need = 0;
  if (!mulChecked(last + 1, static_cast<int64_t>(b.elementSize), need))
    return terr("integer_overflow", "the plan's destination footprint overflows");
  if (need > b.totalBytes)
    return terr("plan_mismatch", "the plan writes beyond its declared destination footprint");
  return std::nullopt;
}

} // namespace

std::variant<size_t, TransferError> viewSpanBytes(const BufferView &v, const char *role) {
  const std::string who = capitalized(role);
  if (v.base == 0)
    return terr("invalid_view", who + " base pointer is null");
  if (v.elementSize == 0)
    return terr("invalid_view", who + " element size is zero");
  if (v.extents.empty())
    return terr("invalid_view", who + " has rank zero");
  if (v.extents.size() != v.strides.size())
    return terr("invalid_view", who + " extents and strides differ in rank");
  if (v.kind == MemoryKind::Cuda && v.device < 0)
    return terr("invalid_view", who + " is CUDA memory without a device ordinal");
  if (v.kind == MemoryKind::Host && v.device >= 0)
    return terr("invalid_view", who + " is host memory but names a CUDA device");
  // Injective addressing: walk the moving axes by increasing stride; each
  // stride must step past everything the smaller ones reach.
  std::vector<std::pair<int64_t, int64_t>> moving; // (stride, extent) of axes with extent > 1
  for (size_t k = 0; k < v.extents.size(); ++k) {
    if (v.extents[k] < 1)
      return terr("invalid_view", who + " has an extent below one");
    if (v.strides[k] < 0)
      return terr("unsupported_layout", who + " has a negative stride");
    if (v.extents[k] == 1)
      continue;
    if (v.strides[k] == 0)
      return terr("unsupported_layout", who + " broadcasts an axis (stride zero)");
    moving.emplace_back(v.strides[k], v.extents[k]);
  }
  std::sort(moving.begin(), moving.end());
  int64_t reach = 0;
  for (const auto &axis : moving) {
    if (axis.first <= reach)
      return terr("unsupported_layout", who + " has overlapping strides");
    int64_t r = 0;
    if (!mulChecked(axis.second - 1, axis.first, r) || !addChecked(reach, r, reach))
      return terr("integer_overflow", who + " span overflows");
  }
  int64_t bytes = 0;
  if (!mulChecked(reach + 1, static_cast<int64_t>(v.elementSize), bytes) ||
      v.offsetBytes > static_cast<size_t>(std::numeric_limits<int64_t>::max() - bytes))
    return terr("integer_overflow", who + " byte span overflows");
  const size_t end = v.offsetBytes + static_cast<size_t>(bytes);
  if (end > v.capacityBytes)
    return terr("insufficient_capacity", who + " needs " + std::to_string(end) +
                                             " bytes from its allocation base; " +
                                             std::to_string(v.capacityBytes) + " are declared");
  return static_cast<size_t>(bytes);
}

std::variant<size_t, TransferError> validateTransferSource(const BoundPlan &bound, const BufferView &source,
                                                           TransferDirection direction) {
  if (auto e = kindsFit(&source, nullptr, direction))
    return *e;
  auto span = viewSpanBytes(source, "source");
  if (auto *e = std::get_if<TransferError>(&span))
    return *e;
  if (auto e = planReadsFit(bound, source, std::get<size_t>(span)))
    return *e;
  return std::get<size_t>(span);
}

std::variant<TransferRequest, TransferError> validateTransfer(const BoundPlan &bound, const BufferView &source,
                                                              const BufferView &destination,
                                                              TransferDirection direction) {
  if (auto e = kindsFit(&source, &destination, direction))
    return *e;
  auto sourceSpan = validateTransferSource(bound, source, direction);
  if (auto *e = std::get_if<TransferError>(&sourceSpan))
    return *e;
  auto destinationSpan = viewSpanBytes(destination, "destination");
  if (auto *e = std::get_if<TransferError>(&destinationSpan))
    return *e;
  if (auto e = planWritesFit(bound, destination, std::get<size_t>(destinationSpan)))
    return *e;
  TransferRequest r;
  r.bound = bound;
  r.source = source;
  r.destination = destination;
  r.direction = direction;
  r.sourceSpanBytes = std::get<size_t>(sourceSpan);
  r.destinationBytes = static_cast<size_t>(bound.totalBytes);
  return r;
}

std::optional<TransferError> executeTransfer(TransferRequest &request, CopyBackend &backend,
                                             const TransferOptions &options) {
  if (request.consumed)
    return terr("already_executed", "transfer requests are single-use");
  // The request's fields are public: prove them again before anything runs.
  auto checked = validateTransfer(request.bound, request.source, request.destination, request.direction);
  if (auto *e = std::get_if<TransferError>(&checked))
    return *e;
  auto *cuda = dynamic_cast<CudaBackend *>(&backend);
  if (!cuda)
    return terr("backend_mismatch", "layout transfers run on the GPU and need a CudaBackend");
  const bool d2h = request.direction == TransferDirection::DeviceToHost;
  const BufferView &deviceEnd = d2h ? request.source : request.destination;
  if (deviceEnd.kind != MemoryKind::Cuda)
    return terr("direction_mismatch", std::string("the ") + (d2h ? "source" : "destination") +
                                          " of this direction must be CUDA memory");
  if (deviceEnd.device != cuda->device())
    return terr("device_mismatch", "the device end lives on cuda:" + std::to_string(deviceEnd.device) +
                                       ", the backend on cuda:" + std::to_string(cuda->device()));
  auto tmpl = dispatch::prepareTransferTemplate(request.bound, request.direction);
  if (auto *e = std::get_if<TransferError>(&tmpl))
    return *e;
  const auto &t = std::get<dispatch::DispatchTemplate>(tmpl);
  // The template's ends as dense 1-D views over the same allocations: the
  // span the plan reads (from the source view's element 0, inside the
  // validated source span) and the dense destination.
  BufferView src = request.source, dst = request.destination;
  src.extents = t.program.plan.sourceExtents;
  src.strides = {1};
  dst.extents = t.program.plan.resultExtents;
  dst.strides = {1};
  auto prepared = dispatch::prepareDispatch(t, src, dst);
  if (auto *e = std::get_if<TransferError>(&prepared))
    return *e;
  request.consumed = true;
  return dispatch::executeDispatch(std::get<dispatch::DispatchRequest>(prepared), *cuda, options);
}

} // namespace reloc
