// Capability rows, selection, request validation and execution for the B200
// rows; see include/reloc/Dispatch.h. Contracts follow the reference's
// libreloc/src/Dispatch.cpp (queryCapability :1382-1533, select :1147,
// prepareDispatch :1585-1620, executeDispatch :1983-2048): pure capability,
// policy over eligible rows only, single-use requests, errors by value, no
// second path after data dispatch.
#include "reloc/Dispatch.h"
#include "reloc/CudaBackend.h"

#include "device_plan.hpp"
#include "sb_cuda.h"

#include <cstring>

namespace reloc {
namespace dispatch {
namespace {

TransferError terr(const char *code, std::string msg) { return TransferError{code, std::move(msg)}; }

const char *const kCpuExcluded = "the B200 executor runs no supported plan on the CPU";

Implementation b200Row(const typed::Program &p, const char *variant, const b200::Lowered *l, bool d2h = false) {
  Implementation row;
  row.id = d2h ? kB200FusedD2H : kB200FusedH2D;
  row.variant = variant;
  // H2D: the raw source crosses the link; D2H: the finished result does
  row.wireBoundary = d2h ? static_cast<uint32_t>(p.stages.size()) : 0;
  row.wireResultLayout = d2h;
  row.wireBytes = d2h ? p.plan.destinationBytes : p.plan.sourceBytes;
  row.deviceTempBytes = 0;
  row.method = "B";
  (void)l;
  return row;
}

} // namespace

Capability queryCapability(const typed::Program &p, TransferDirection direction, bool cuda) {
  Capability cap;
  const uint32_t n = static_cast<uint32_t>(p.stages.size());
  cap.excluded.push_back({kCpuReference, kCpuExcluded});
  for (uint32_t k = 0; k <= n; ++k)
    cap.excluded.push_back({std::string(kCpuStagesCudaStages) + "@" + std::to_string(k), kCpuExcluded});
  cap.excluded.push_back({kCudaDequantRelocate, "superseded by b200_fused_h2d"});
  cap.excluded.push_back({kCudaRelocateF32, "superseded by b200_fused_h2d"});
  const bool d2h = direction == TransferDirection::DeviceToHost;
  const char *id = d2h ? kB200FusedD2H : kB200FusedH2D;
  cap.excluded.push_back({d2h ? kB200FusedH2D : kB200FusedD2H, "the other transfer direction"});
  if (!cuda) {
    cap.excluded.push_back({id, "no CUDA device end"});
    return cap;
  }
  auto lowered = b200::lower(p);
  if (auto *e = std::get_if<TransferError>(&lowered)) {
    cap.excluded.push_back({id, e->code + ": " + e->message});
    return cap;
  }
  const auto &l = std::get<b200::Lowered>(lowered);
  cap.eligible.push_back(b200Row(p, "", &l, d2h));
  cap.eligible.push_back(b200Row(p, "dma_ring", &l, d2h));
  cap.eligible.push_back(b200Row(p, "zero_copy", &l, d2h));
  return cap;
}

std::variant<Selection, TransferError> selectImplementation(const typed::Program &p, TransferDirection direction,
                                                            const Options &o) {
  const Capability cap = queryCapability(p, direction, o.cuda);
  Selection sel;
  if (!o.implementation.empty()) {
    for (const Implementation &row : cap.eligible)
      if (row.label() == o.implementation) {
        sel.row = row;
        sel.policy = "explicit";
        sel.reason = "explicit";
        return sel;
      }
    std::string why = "not an eligible row";
    for (const Exclusion &e : cap.excluded)
      if (e.id == o.implementation)
        why = e.reason;
    return terr("implementation_unavailable", o.implementation + ": " + why);
  }
  if (o.policy == Policy::OriginalCpu)
    return terr("implementation_unavailable", std::string("original_cpu: ") + kCpuExcluded);
  if (cap.eligible.empty()) {
    std::string why;
    for (const Exclusion &e : cap.excluded)
      if (e.id == (direction == TransferDirection::DeviceToHost ? kB200FusedD2H : kB200FusedH2D))
        why = e.reason;
    return terr("implementation_unavailable", "no eligible row: " + why);
  }
  sel.row = cap.eligible.front();
  sel.policy = "auto";
  sel.reason = "b200_gpu_only";
  return sel;
}

std::variant<DispatchTemplate, TransferError> prepareDispatchTemplate(const TypedBoundPlan &plan,
                                                                      TransferDirection direction, const Options &o) {
  auto prog = typed::prepareProgram(plan);
  if (auto *e = std::get_if<typed::ExecutionError>(&prog))
    return terr(e->code.c_str(), e->message);
  DispatchTemplate t;
  t.program = std::get<typed::Program>(std::move(prog));
  t.direction = direction;
  t.cuda = o.cuda;
  t.capability = queryCapability(t.program, direction, o.cuda);
  auto sel = selectImplementation(t.program, direction, o);
  if (auto *e = std::get_if<TransferError>(&sel))
    return *e;
  t.selection = std::get<Selection>(std::move(sel));
  auto lowered = b200::lower(t.program);
  if (auto *e = std::get_if<TransferError>(&lowered))
    return *e;
  t.lowered = std::make_shared<const b200::Lowered>(std::get<b200::Lowered>(std::move(lowered)));
  return t;
}

namespace {

/// The views must be the plan's dense tensors: row-major, the bound extents,
/// the boundary element width, enough capacity.
std::optional<TransferError> checkView(const BufferView &v, const std::vector<int64_t> &extents, uint32_t width,
                                       int64_t bytes, MemoryKind kind, const char *role) {
  if (v.kind != kind)
    return terr("direction_mismatch", std::string(role) + " memory kind does not match the transfer direction");
  if (v.base == 0)
    return terr("invalid_view", std::string(role) + " base is null");
  if (v.elementSize != width)
    return terr("plan_mismatch", std::string(role) + " element size " + std::to_string(v.elementSize) +
                                     " differs from the plan's " + std::to_string(width));
  if (v.extents != extents)
    return terr("plan_mismatch", std::string(role) + " extents differ from the bound plan");
  if (v.strides.size() != extents.size())
    return terr("invalid_view", std::string(role) + " strides and extents differ in rank");
  int64_t expect = 1;
  for (size_t k = extents.size(); k-- > 0;) {
    if (extents[k] != 1 && v.strides[k] != expect)
      return terr("unsupported_layout", std::string(role) + " must be dense row-major");
    expect *= extents[k];
  }
  if (v.offsetBytes > v.capacityBytes || static_cast<int64_t>(v.capacityBytes - v.offsetBytes) < bytes)
    return terr("insufficient_capacity", std::string(role) + " allocation is smaller than the plan's " +
                                             std::to_string(bytes) + " bytes");
  return std::nullopt;
}

} // namespace

std::variant<DispatchRequest, TransferError> prepareDispatch(const DispatchTemplate &t, const BufferView &src,
                                                             const BufferView &dst) {
  const bool d2h = t.direction == TransferDirection::DeviceToHost;
  const typed::Program &p = t.program;
  const uint32_t n = static_cast<uint32_t>(p.stages.size());
  if (auto e = checkView(src, p.plan.sourceExtents, typed::widthAt(p, 0), p.plan.sourceBytes,
                         d2h ? MemoryKind::Cuda : MemoryKind::Host, "source"))
    return *e;
  if (auto e = checkView(dst, p.plan.resultExtents, typed::widthAt(p, n), p.plan.destinationBytes,
                         d2h ? MemoryKind::Host : MemoryKind::Cuda, "destination"))
    return *e;
  DispatchRequest r;
  r.program = p;
  r.source = src;
  r.destination = dst;
  r.direction = t.direction;
  r.selected = t.selection.row;
  r.lowered = t.lowered;
  Report &rep = r.report;
  rep.implementation = t.selection.row.label();
  rep.policy = t.selection.policy;
  rep.placementReason = t.selection.reason;
  rep.method = t.selection.row.method;
  rep.wireBoundary = t.selection.row.wireBoundary;
  rep.sourceBytes = p.plan.sourceBytes;
  rep.wireBytes = t.selection.row.wireBytes;
  rep.destinationBytes = p.plan.destinationBytes;
  rep.parameterBytes = p.plan.parameterBytes;
  return r;
}

std::variant<DispatchRequest, TransferError> prepareDispatch(const TypedBoundPlan &plan, const BufferView &src,
                                                             const BufferView &dst, TransferDirection direction,
                                                             const Options &o) {
  auto t = prepareDispatchTemplate(plan, direction, o);
  if (auto *e = std::get_if<TransferError>(&t))
    return *e;
  return prepareDispatch(std::get<DispatchTemplate>(t), src, dst);
}

namespace {

Route routeOf(const Implementation &row, const TransferOptions &o) {
  if (row.variant == "dma_ring")
    return Route::DmaRing;
  if (row.variant == "zero_copy")
    return Route::ZeroCopy;
  return o.route;
}

/// Shared tail of an execution: signal the caller stream, record
/// `completionEvent`, then (blocking, or when a status word or a route timing
/// must be read) wait, check the context's fault word and the status word,
/// and learn the route timing. An asynchronous execution returns once
/// enqueued; the fault word then still reports any earlier execution of this
/// context whose kernels have finished (the word is host memory: reading it
/// costs no CUDA call), and a later call or the completion reports this one.
std::optional<TransferError> finish(bool needsStatus, const std::string &classKey, CudaBackend &b,
                                    const TransferOptions &o, bool timed, Route route, int64_t bytes,
                                    void *completionEvent = nullptr, bool copyUsed = true) {
  if (!b.signalStream(o.callerStream, o.hasCallerStream, copyUsed))
    return terr("backend_failure", b.error());
  int rc;
  if (completionEvent) {
    if ((rc = sbc_event_record(completionEvent, b.computeStream()))) {
      b.fail("cudaEventRecord(completion)", rc);
      return terr("backend_failure", b.error());
    }
    ++b.eventRecords;
  }
  if (o.asyncCompletion && !needsStatus && !timed) {
    if (!completionEvent && !b.healthy())
      return terr("backend_failure", b.error());
    return std::nullopt;
  }
  if ((rc = sbc_event_synchronize(b.doneEvent()))) {
    b.fail("completion", rc);
    return terr("backend_failure", b.error());
  }
  if (!completionEvent && !b.healthy())
    return terr("backend_failure", b.error());
  if (timed) {
    float ms = 0;
    if (sbc_event_elapsed_ms(b.startEvent(), b.stopEvent(), &ms) == 0 && bytes > 0) {
      auto &s = b.routeStats[classKey];
      const double spb = (ms * 1e-3) / static_cast<double>(bytes);
      if (route == Route::DmaRing) {
        s.dmaSecondsPerByte = spb;
        ++s.dmaSamples;
      } else if (route == Route::ZeroCopy) {
        s.zeroCopySecondsPerByte = spb;
        ++s.zeroCopySamples;
      }
    }
  }
  if (needsStatus) {
    if ((rc = sbc_memcpy_d2h_async(b.statusHost(), b.statusWord(), 4, b.computeStream())) ||
        (rc = sbc_stream_synchronize(b.computeStream()))) {
      b.fail("status readback", rc);
      return terr("backend_failure", b.error());
    }
    if (*b.statusHost())
      return terr("channel_out_of_range", "a channel index fell outside its parameter table");
  }
  return std::nullopt;
}

/// Enqueue one request's copies and kernels (after the caller-stream wait,
/// before the completion). `timed`: bracket it with the route-timing events.
std::optional<TransferError> launch(DispatchRequest &req, CudaBackend &b, const TransferOptions &o, bool timed,
                                    Route &route) {
  const b200::Lowered &l = *req.lowered;
  const void *src = reinterpret_cast<const void *>(req.source.base + req.source.offsetBytes);
  void *dst = reinterpret_cast<void *>(req.destination.base + req.destination.offsetBytes);
  TransferOptions ro = o;
  ro.route = routeOf(req.selected, o);
  const bool d2h = req.direction == TransferDirection::DeviceToHost;
  route = d2h ? b200::chooseRouteD2H(l, dst, ro) : b200::chooseRoute(l, b, src, ro);
  if (timed)
    sbc_event_record(b.startEvent(), b.copyStream());
  b200::RunStats st;
  const uint64_t copies0 = b.copyCalls, launches0 = b.kernelLaunches;
  if (auto e = d2h ? b200::runD2H(l, b, src, dst, route, ro, st)
                   : b200::runH2D(l, b, src, dst, route, b200::RowWindow{}, ro, st))
    return e;
  if (timed)
    sbc_event_record(b.stopEvent(), b.computeStream());
  Report &rep = req.report;
  rep.executed = true;
  rep.route = st.route;
  rep.deviceKernel = st.kernel;
  rep.hostPipeline = st.route;
  rep.hostChunks = st.chunks;
  rep.hostChunkBytes = st.chunkBytes;
  rep.hostBuffers = st.buffers;
  rep.payloadBytesTransferred = st.payloadBytes + static_cast<int64_t>(l.paramBlob.size());
  rep.kernelLaunches = b.kernelLaunches - launches0;
  rep.copyCalls = b.copyCalls - copies0;
  rep.implementation = req.selected.variant.empty() ? req.selected.id + "@" + st.route : req.selected.label();
  return std::nullopt;
}

} // namespace

int executionDevice(const DispatchRequest &req) {
  return req.direction == TransferDirection::DeviceToHost ? req.source.device : req.destination.device;
}

std::optional<TransferError> executeDispatch(DispatchRequest &req, CudaBackend &b, const TransferOptions &o) {
  if (req.consumed)
    return terr("already_executed", "dispatch requests are single-use");
  req.consumed = true;
  if (!req.lowered)
    return terr("implementation_unavailable", "request has no lowered program");
  if (executionDevice(req) != b.device())
    return terr("device_mismatch", "the device end lives on cuda:" + std::to_string(executionDevice(req)) +
                                       ", the context on cuda:" + std::to_string(b.device()));
  if (!b.healthy())
    return terr("backend_failure", b.error());
  if (!b.activate())
    return terr("backend_failure", b.error());
  if (o.hasCallerStream && !b.waitStream(o.callerStream))
    return terr("backend_failure", b.error());
  // Auto mode learns each H2D route's cost per plan class from event
  // timings: every execution until both routes are measured, then one in 64,
  // and the slower route is measured again after 4, 16 and then every 128
  // executions, so a cold early sample (ring allocation, first touch of the
  // source, a link leaving its idle state) does not decide for good.
  bool timed = false;
  CudaBackend::RouteStats *rs = nullptr;
  if (routeOf(req.selected, o) == Route::Auto && !o.asyncCompletion &&
      req.direction == TransferDirection::HostToDevice) {
    rs = &b.routeStats[req.lowered->classKey];
    const bool known = rs->known();
    const uint32_t n = known ? ++rs->executions : 0;
    rs->probe = known && (n == 4 || n == 16 || (n & 127u) == 64);
    timed = !known || rs->probe || (n & 63u) == 0;
  }
  Route route = Route::Auto;
  const uint64_t copies0 = b.copyCalls;
  auto e = launch(req, b, o, timed, route);
  if (rs)
    rs->probe = false; // only this execution
  if (e)
    return e;
  return finish(req.lowered->needsStatus, req.lowered->classKey, b, o, timed, route, req.program.plan.sourceBytes,
                nullptr, timed || b.copyCalls != copies0);
}

std::optional<TransferError> executeDispatch(DispatchRequest &req, CopyBackend &backend, const TransferOptions &o) {
  auto *cuda = dynamic_cast<CudaBackend *>(&backend);
  if (!cuda)
    return terr("backend_mismatch", "row " + req.selected.label() + " needs a CudaBackend");
  return executeDispatch(req, *cuda, o);
}

std::variant<DispatchTemplate, TransferError> prepareTransferTemplate(const BoundPlan &l,
                                                                      TransferDirection direction) {
  if (l.typed)
    return terr("typed_unsupported", "layout transfers take a layout-only (v0) bound plan");
  if (l.extents.empty() || l.extents.size() != l.srcStrides.size() || l.extents.size() != l.dstStrides.size())
    return terr("plan_mismatch", "bound plan has inconsistent axes");
  if (l.padRegions.size() > 1)
    for (const PadRegion &p : l.padRegions)
      if (p.fillBits != l.padRegions.front().fillBits)
        return terr("mixed_fills_unsupported", "v0 plans carry a single fill value");
  // The plan as a stage-free typed program: a dense 1-D source of the plan's
  // source span, a dense 1-D result of its padded element count.
  TypedBoundPlan t;
  t.layout = l;
  const ElementType et{ElementTypeKind::Integer, l.elementSize * 8};
  int64_t span = 1;
  for (size_t k = 0; k < l.extents.size(); ++k)
    span += (l.extents[k] - 1) * l.srcStrides[k];
  t.sourceExtents = {span};
  t.resultExtents = {l.totalBytes / static_cast<int64_t>(l.elementSize)};
  t.sourceType = t.resultType = et;
  for (const PadRegion &p : l.padRegions)
    t.fills.push_back(TypedFill{static_cast<uint32_t>(p.axis), 0, et, p.fillBits});
  t.cuts.push_back(StageFootprint{0, et, t.resultExtents[0], l.totalBytes});
  t.sourceBytes = span * l.elementSize;
  t.destinationBytes = l.totalBytes;
  t.requirements = {"layout_transfer"};
  Options o;
  o.cuda = true;
  return prepareDispatchTemplate(t, direction, o);
}

std::optional<TransferError> executeSourceRows(const DispatchTemplate &t, CudaBackend &b, const void *rows,
                                               int64_t rowBegin, int64_t rowEnd, void *dst, const TransferOptions &o,
                                               Report &rep) {
  if (!t.lowered)
    return terr("implementation_unavailable", "template has no lowered program");
  if (!b.healthy())
    return terr("backend_failure", b.error());
  if (!b.activate())
    return terr("backend_failure", b.error());
  if (o.hasCallerStream && !b.waitStream(o.callerStream))
    return terr("backend_failure", b.error());
  b200::RunStats st;
  const uint64_t launches0 = b.kernelLaunches;
  if (auto e = b200::runSourceRows(*t.lowered, b, rows, rowBegin, rowEnd, dst, st))
    return e;
  rep.executed = true;
  rep.route = st.route;
  rep.deviceKernel = st.kernel;
  rep.kernelLaunches = b.kernelLaunches - launches0;
  rep.sourceBytes = t.program.plan.sourceBytes;
  rep.destinationBytes = t.program.plan.destinationBytes;
  return finish(t.lowered->needsStatus, t.lowered->classKey, b, o, false, Route::Auto, 0);
}

std::optional<TransferError> executeSourceShards(const DispatchTemplate &t, CudaBackend &b,
                                                 const void *const *shards, const int64_t *bounds, int n, void *dst,
                                                 const TransferOptions &o, Report &rep) {
  if (!t.lowered)
    return terr("implementation_unavailable", "template has no lowered program");
  if (!b.healthy())
    return terr("backend_failure", b.error());
  if (!b.activate())
    return terr("backend_failure", b.error());
  if (o.hasCallerStream && !b.waitStream(o.callerStream))
    return terr("backend_failure", b.error());
  b200::RunStats st;
  const uint64_t launches0 = b.kernelLaunches;
  if (auto e = b200::runSourceShards(*t.lowered, b, shards, bounds, n, dst, st))
    return e;
  rep.executed = true;
  rep.route = st.route;
  rep.deviceKernel = st.kernel;
  rep.kernelLaunches = b.kernelLaunches - launches0;
  rep.sourceBytes = t.program.plan.sourceBytes;
  rep.destinationBytes = t.program.plan.destinationBytes;
  return finish(t.lowered->needsStatus, t.lowered->classKey, b, o, false, Route::Auto, 0);
}

std::variant<GroupRequest, TransferError> prepareDispatchGroup(const std::vector<GroupEntry> &entries) {
  if (entries.empty() || entries.size() > 256)
    return terr("invalid_options", "a group must contain between 1 and 256 members");
  GroupRequest g;
  std::vector<std::pair<uintptr_t, uintptr_t>> dsts, srcs;
  for (size_t i = 0; i < entries.size(); ++i) {
    const GroupEntry &e = entries[i];
    const std::string who = "group member " + std::to_string(i) + ": ";
    if (!e.plan)
      return terr("invalid_options", who + "no plan");
    if (e.direction != TransferDirection::HostToDevice)
      return terr("implementation_unavailable", who + "device-to-host transfers are outside this executor");
    auto r = prepareDispatch(*e.plan, e.source, e.destination);
    if (auto *err = std::get_if<TransferError>(&r))
      return terr(err->code.c_str(), who + err->message);
    DispatchRequest req = std::move(std::get<DispatchRequest>(r));
    if (g.device < 0)
      g.device = req.destination.device;
    else if (req.destination.device != g.device)
      return terr("device_mismatch", who + "destination on cuda:" + std::to_string(req.destination.device) +
                                         ", the group on cuda:" + std::to_string(g.device));
    // prepareDispatch admits dense row-major views only: their spans are the plan's byte counts
    const size_t sspan = static_cast<size_t>(req.program.plan.sourceBytes);
    const size_t dspan = static_cast<size_t>(req.program.plan.destinationBytes);
    const uintptr_t s0 = req.source.base + req.source.offsetBytes, d0 = req.destination.base + req.destination.offsetBytes;
    srcs.push_back({s0, s0 + sspan});
    dsts.push_back({d0, d0 + dspan});
    g.report.outputBytes += dspan;
    g.items.push_back(std::move(req));
  }
  auto overlap = [](const std::pair<uintptr_t, uintptr_t> &a, const std::pair<uintptr_t, uintptr_t> &b) {
    return a.first < b.second && b.first < a.second;
  };
  for (size_t i = 0; i < dsts.size(); ++i)
    for (size_t j = 0; j < dsts.size(); ++j) {
      if (j > i && overlap(dsts[i], dsts[j]))
        return terr("invalid_view", "group members " + std::to_string(i) + " and " + std::to_string(j) +
                                        " write overlapping destinations");
      if (overlap(dsts[i], srcs[j]))
        return terr("invalid_view", "the destination of group member " + std::to_string(i) +
                                        " overlaps the source of member " + std::to_string(j));
    }
  g.reports.resize(g.items.size());
  return g;
}

std::optional<TransferError> executeGroup(GroupRequest &g, CudaBackend &b, const TransferOptions &o,
                                          void *completionEvent) {
  if (g.consumed)
    return terr("already_executed", "dispatch groups are single-use");
  g.consumed = true;
  if (g.device != b.device())
    return terr("device_mismatch", "group destinations live on cuda:" + std::to_string(g.device) +
                                       ", the context on cuda:" + std::to_string(b.device()));
  for (const DispatchRequest &r : g.items)
    if (r.consumed || !r.lowered)
      return terr("already_executed", "a group member was already executed");
  if (!b.healthy())
    return terr("backend_failure", b.error());
  if (!b.activate())
    return terr("backend_failure", b.error());
  const uint64_t copies0 = b.copyCalls, launches0 = b.kernelLaunches, records0 = b.eventRecords,
                 waits0 = b.eventWaits, callers0 = b.callerWaits;
  if (o.hasCallerStream && !b.waitStream(o.callerStream))
    return terr("backend_failure", b.error());
  // One status word serves the whole group: cleared once here, not per member.
  bool needsStatus = false;
  for (const DispatchRequest &r : g.items)
    needsStatus = needsStatus || r.lowered->needsStatus;
  if (needsStatus) {
    const int rc = sbc_fill(b.statusWord(), 1, 4, 0, b.computeStream());
    if (rc) {
      b.fail("status reset", rc);
      return terr("backend_failure", b.error());
    }
  }
  struct Keep {
    CudaBackend &b;
    ~Keep() { b.keepStatus = false; }
  } keep{b};
  b.keepStatus = true;
  for (size_t i = 0; i < g.items.size(); ++i) {
    DispatchRequest &r = g.items[i];
    r.consumed = true;
    Route route = Route::Auto;
    if (auto e = launch(r, b, o, false, route)) {
      g.failed = true;
      return terr(e->code.c_str(), "group member " + std::to_string(i) + ": " + e->message);
    }
    g.reports[i] = r.report;
  }
  b.keepStatus = false;
  GroupReport &gr = g.report;
  gr.copyCalls = b.copyCalls - copies0;
  gr.payloadCopyCalls = gr.copyCalls;
  gr.kernelLaunches = b.kernelLaunches - launches0;
  auto e = finish(needsStatus, std::string(), b, o, false, Route::Auto, 0, completionEvent);
  gr.eventRecords = b.eventRecords - records0;
  gr.eventWaits = b.eventWaits - waits0;
  gr.callerWaits = b.callerWaits - callers0;
  if (e)
    g.failed = true;
  return e;
}

std::optional<TransferError> executeWindow(const DispatchTemplate &t, CudaBackend &b, const void *src, bool hostSource,
                                           void *dst, int64_t rowBegin, int64_t rowEnd, const TransferOptions &o,
                                           Report &rep) {
  if (!t.lowered)
    return terr("implementation_unavailable", "template has no lowered program");
  if (!b.healthy())
    return terr("backend_failure", b.error());
  if (!b.activate())
    return terr("backend_failure", b.error());
  const b200::Lowered &l = *t.lowered;
  if (rowBegin < 0 || rowEnd > l.padded[0] || rowEnd < rowBegin)
    return terr("invalid_options", "row window outside the padded result rows [0, " + std::to_string(l.padded[0]) +
                                       ")");
  if (rowEnd == rowBegin)
    return std::nullopt;
  if (o.hasCallerStream && !b.waitStream(o.callerStream))
    return terr("backend_failure", b.error());
  b200::RunStats st;
  const uint64_t copies0 = b.copyCalls, launches0 = b.kernelLaunches;
  std::optional<TransferError> e;
  if (hostSource) {
    TransferOptions ro = o;
    ro.route = routeOf(t.selection.row, o);
    if (ro.route == Route::Auto)
      ro.route = Route::DmaRing;
    e = b200::runH2D(l, b, src, dst, ro.route, b200::RowWindow{rowBegin, rowEnd}, ro, st);
  } else {
    st.route = "device";
    e = b200::runDevice(l, b, src, dst, b200::RowWindow{rowBegin, rowEnd}, st);
  }
  if (e)
    return e;
  rep.executed = true;
  rep.route = st.route;
  rep.deviceKernel = st.kernel;
  rep.hostChunks = st.chunks;
  rep.hostChunkBytes = st.chunkBytes;
  rep.hostBuffers = st.buffers;
  rep.payloadBytesTransferred = st.payloadBytes + static_cast<int64_t>(l.paramBlob.size());
  rep.kernelLaunches = b.kernelLaunches - launches0;
  rep.copyCalls = b.copyCalls - copies0;
  rep.sourceBytes = t.program.plan.sourceBytes;
  rep.destinationBytes = t.program.plan.destinationBytes;
  return finish(l.needsStatus, l.classKey, b, o, false, Route::Auto, 0);
}

} // namespace dispatch
} // namespace reloc
