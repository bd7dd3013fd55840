// The drop-in C-ABI (include/sym_b200.h) over the C++ runtime.
#include "sym_b200.h"

#include "reloc/Bind.h"
#include "reloc/CudaBackend.h"
#include "reloc/Decode.h"
#include "reloc/Dispatch.h"
#include "reloc/DispatchResources.h"
#include "reloc/TypedValue.h"

#include "device_plan.hpp"
#include "sb_cuda.h"
#include "static_scratch.h"

#include <cstdio>
#include <cstring>
#include <sstream>
#include <string>
#include <variant>

using namespace reloc;

struct sb_plan {
  bool typed = false;
  RelocationPlan layout;
  TypedRelocationPlan plan;
};

struct sb_bound {
  bool typed = false;
  BoundPlan layout;
  TypedBoundPlan bound;
  std::optional<typed::Program> program;
  std::string programError;
};

struct sb_template {
  dispatch::DispatchTemplate t;
};

struct sb_request {
  dispatch::DispatchRequest r;
};

struct sb_resources {
  dispatch::Resources res;
  sb_resources(size_t a, size_t b, unsigned c) : res(a, b, c) {}
};

struct sb_group {
  dispatch::GroupRequest g;
};

struct sb_completion {
  std::shared_ptr<dispatch::Resources> ephemeral; // private context when the caller passed none
  std::shared_ptr<dispatch::Completion> c;
  ~sb_completion() { c.reset(); } // drains before the private context goes
};

namespace {

const char *kVersion = "sym_b200 0.1.0 (libreloc wire v0/v1, sm_100a)";

int setErr(sb_error *err, const std::string &code, const std::string &msg, int64_t offset = -1) {
  if (err) {
    std::snprintf(err->code, sizeof err->code, "%s", code.c_str());
    std::snprintf(err->message, sizeof err->message, "%s", msg.c_str());
    err->offset = offset;
  }
  return 1;
}

int putJson(const std::string &s, char *buf, size_t cap) {
  if (buf && cap) {
    const size_t n = s.size() < cap - 1 ? s.size() : cap - 1;
    std::memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
  return static_cast<int>(s.size());
}

std::string q(const std::string &s) {
  std::string o = "\"";
  for (char c : s) {
    if (c == '"' || c == '\\')
      o += '\\';
    // Control and non-ASCII bytes are escaped byte-wise (names are opaque
    // wire bytes, not necessarily UTF-8).
    if (static_cast<unsigned char>(c) < 0x20 || static_cast<unsigned char>(c) >= 0x80) {
      char b[8];
      std::snprintf(b, sizeof b, "\\u%04x", static_cast<unsigned char>(c));
      o += b;
      continue;
    }
    o += c;
  }
  return o + "\"";
}

template <typename T> std::string list(const std::vector<T> &v) {
  std::ostringstream os;
  os << "[";
  for (size_t i = 0; i < v.size(); ++i)
    os << (i ? "," : "") << v[i];
  os << "]";
  return os.str();
}

std::string dtypeName(ElementType t) {
  switch (t.kind) {
  case ElementTypeKind::Float:
    return t.bitwidth == 16 ? "float16" : t.bitwidth == 32 ? "float32" : "float64";
  case ElementTypeKind::BFloat:
    return "bfloat16";
  case ElementTypeKind::Integer:
    return "int" + std::to_string(t.bitwidth);
  case ElementTypeKind::Index:
    return "index";
  }
  return "unknown";
}

bool parseDtype(const char *name, ElementType &out) {
  const std::string s(name ? name : "");
  if (s == "float32") out = {ElementTypeKind::Float, 32};
  else if (s == "float16") out = {ElementTypeKind::Float, 16};
  else if (s == "float64") out = {ElementTypeKind::Float, 64};
  else if (s == "bfloat16") out = {ElementTypeKind::BFloat, 16};
  else if (s == "int8") out = {ElementTypeKind::Integer, 8};
  else if (s == "int16") out = {ElementTypeKind::Integer, 16};
  else if (s == "int32") out = {ElementTypeKind::Integer, 32};
  else if (s == "int64") out = {ElementTypeKind::Integer, 64};
  else return false;
  return true;
}

std::string layoutJson(const BoundPlan &b) {
  std::ostringstream os;
  os << "{\"extents\":" << list(b.extents) << ",\"src_strides\":" << list(b.srcStrides)
     << ",\"dst_strides\":" << list(b.dstStrides) << ",\"element_size\":" << b.elementSize
     << ",\"total_bytes\":" << b.totalBytes << ",\"L\":" << b.L << ",\"typed\":" << (b.typed ? "true" : "false")
     << ",\"no_copy\":" << (b.noCopy ? "true" : "false") << ",\"perm\":" << list(b.perm) << ",\"pads\":[";
  for (size_t i = 0; i < b.padRegions.size(); ++i) {
    const PadRegion &p = b.padRegions[i];
    os << (i ? "," : "") << "{\"axis\":" << p.axis << ",\"lo\":" << p.lo << ",\"hi\":" << p.hi
       << ",\"fill\":" << p.fillBits << "}";
  }
  static const char *strategies[] = {"auto", "view_no_copy", "single_thread_simd", "multi_thread_tiled",
                                     "chunked_pipeline"};
  os << "],\"strategy\":\"" << strategies[static_cast<int>(b.strategy)] << "\"}";
  return os.str();
}

std::string exprJson(const ExprStream &e) {
  std::ostringstream os;
  os << "[";
  for (size_t i = 0; i < e.size(); ++i)
    os << (i ? "," : "") << "[" << static_cast<int>(e[i].op) << "," << e[i].value << "]";
  os << "]";
  return os.str();
}

std::string paramJson(const StageParam &p) {
  if (p.kind == ParamKind::None)
    return "null";
  std::ostringstream os;
  os << "{\"kind\":" << (p.kind == ParamKind::Inline ? "\"inline\"" : "\"binding\"") << ",\"rank\":" << int(p.rank)
     << ",\"dtype\":" << q(dtypeName(p.elementType));
  if (p.kind == ParamKind::Binding)
    os << ",\"name\":" << q(p.bindingName);
  else
    os << ",\"count\":" << p.inlineBits.size();
  os << "}";
  return os.str();
}

std::string boundJson(const sb_bound &b) {
  if (!b.typed)
    return layoutJson(b.layout);
  const TypedBoundPlan &t = b.bound;
  std::ostringstream os;
  os << "{\"layout\":" << layoutJson(t.layout) << ",\"source_extents\":" << list(t.sourceExtents)
     << ",\"result_extents\":" << list(t.resultExtents) << ",\"source_dtype\":" << q(dtypeName(t.sourceType))
     << ",\"result_dtype\":" << q(dtypeName(t.resultType)) << ",\"source_bytes\":" << t.sourceBytes
     << ",\"destination_bytes\":" << t.destinationBytes << ",\"parameter_bytes\":" << t.parameterBytes
     << ",\"symbols\":" << list(t.symbols) << ",\"requirements\":[";
  for (size_t i = 0; i < t.requirements.size(); ++i)
    os << (i ? "," : "") << q(t.requirements[i]);
  os << "],\"cuts\":[";
  for (size_t i = 0; i < t.cuts.size(); ++i)
    os << (i ? "," : "") << "{\"boundary\":" << t.cuts[i].boundary << ",\"dtype\":" << q(dtypeName(t.cuts[i].elementType))
       << ",\"elements\":" << t.cuts[i].elements << ",\"bytes\":" << t.cuts[i].bytes << "}";
  os << "],\"stages\":[";
  for (size_t k = 0; k < t.stages.size(); ++k) {
    const BoundStage &s = t.stages[k];
    os << (k ? "," : "") << "{\"transform\":" << int(s.transform) << ",\"policy\":" << int(s.policy)
       << ",\"input_dtype\":" << q(dtypeName(s.input.type)) << ",\"output_dtype\":" << q(dtypeName(s.output.type))
       << ",\"shape\":" << list(s.shape) << ",\"axis\":" << s.axis
       << ",\"channel_tokens\":" << (s.hasChannel ? exprJson(s.channel) : "null");
    if (b.program) {
      const typed::StageArithmetic &a = b.program->stages[k];
      std::vector<uint32_t> sc, inv;
      for (float f : a.scale) {
        uint32_t u;
        std::memcpy(&u, &f, 4);
        sc.push_back(u);
      }
      for (float f : a.invScale) {
        uint32_t u;
        std::memcpy(&u, &f, 4);
        inv.push_back(u);
      }
      os << ",\"per_channel\":" << (a.perChannel ? "true" : "false")
         << ",\"channel_is_dim\":" << (a.channelIsDim ? "true" : "false") << ",\"channel_dim\":" << a.channelDim
         << ",\"channel_length\":" << a.channelLength << ",\"scale_bits\":" << list(sc)
         << ",\"inv_scale_bits\":" << list(inv) << ",\"zero_point\":" << list(a.zeroPoint);
    }
    os << "}";
  }
  os << "]";
  if (!b.program)
    os << ",\"program_error\":" << q(b.programError);
  os << "}";
  return os.str();
}

std::string capabilityJson(const dispatch::Capability &c) {
  std::ostringstream os;
  os << "{\"eligible\":[";
  for (size_t i = 0; i < c.eligible.size(); ++i) {
    const auto &r = c.eligible[i];
    os << (i ? "," : "") << "{\"implementation\":" << q(r.label()) << ",\"wire_boundary\":" << r.wireBoundary
       << ",\"wire_bytes\":" << r.wireBytes << ",\"device_temp_bytes\":" << r.deviceTempBytes
       << ",\"method\":" << q(r.method) << "}";
  }
  os << "],\"excluded\":[";
  for (size_t i = 0; i < c.excluded.size(); ++i)
    os << (i ? "," : "") << "{\"implementation\":" << q(c.excluded[i].id) << ",\"reason\":" << q(c.excluded[i].reason)
       << "}";
  os << "]}";
  return os.str();
}

std::string reportJson(const dispatch::Report &r) {
  std::ostringstream os;
  os << "{\"implementation\":" << q(r.implementation) << ",\"policy\":" << q(r.policy)
     << ",\"placement_reason\":" << q(r.placementReason) << ",\"method\":" << q(r.method)
     << ",\"wire_boundary\":" << r.wireBoundary << ",\"source_bytes\":" << r.sourceBytes
     << ",\"wire_bytes\":" << r.wireBytes << ",\"destination_bytes\":" << r.destinationBytes
     << ",\"parameter_bytes\":" << r.parameterBytes << ",\"payload_bytes_transferred\":" << r.payloadBytesTransferred
     << ",\"device_temp_bytes\":" << r.deviceTempBytes << ",\"artifact_version\":" << r.artifactVersion
     << ",\"executed\":" << (r.executed ? "true" : "false") << ",\"host_pipeline\":" << q(r.hostPipeline)
     << ",\"host_kernel\":" << q(r.hostKernel) << ",\"host_chunks\":" << r.hostChunks
     << ",\"host_chunk_bytes\":" << r.hostChunkBytes << ",\"host_buffers\":" << r.hostBuffers
     << ",\"route\":" << q(r.route) << ",\"device_kernel\":" << q(r.deviceKernel)
     << ",\"kernel_launches\":" << r.kernelLaunches << ",\"copy_calls\":" << r.copyCalls << "}";
  return os.str();
}

BufferView toView(const sb_view &v) {
  BufferView b;
  b.base = static_cast<uintptr_t>(v.base);
  b.capacityBytes = static_cast<size_t>(v.capacity_bytes);
  b.offsetBytes = static_cast<size_t>(v.offset_bytes);
  b.kind = v.kind == 1 ? MemoryKind::Cuda : MemoryKind::Host;
  b.device = v.device;
  b.elementSize = v.element_size;
  const int r = v.rank < 0 ? 0 : (v.rank > 8 ? 8 : v.rank);
  b.extents.assign(v.extents, v.extents + r);
  b.strides.assign(v.strides, v.strides + r);
  return b;
}

TransferOptions toOptions(const sb_options *o) {
  TransferOptions t;
  if (!o)
    return t;
  t.nBuffers = o->n_buffers > 0 ? o->n_buffers : 4;
  t.route = o->route == 1 ? Route::DmaRing : o->route == 2 ? Route::ZeroCopy : o->route == 3 ? Route::Staged
                                                                                              : Route::Auto;
  t.chunkSizeOverride = static_cast<size_t>(o->chunk_bytes);
  t.hasCallerStream = o->has_caller_stream != 0;
  t.callerStream = o->caller_stream;
  t.asyncCompletion = o->async_completion != 0;
  return t;
}

SymbolMap symbolsOf(int32_t n, const char *const *names, const int64_t *values) {
  SymbolMap m;
  for (int32_t i = 0; i < n; ++i)
    m[names[i]] = values[i];
  return m;
}

} // namespace

extern "C" {

const char *sb_version(void) { return kVersion; }
uint64_t sb_kernel_launches(void) { return sbc_launch_count(); }

int sb_wire_version(const uint8_t *data, size_t size) {
  auto v = peekWireVersion(data, size);
  return v ? static_cast<int>(*v) : -1;
}

int sb_load_plan(const uint8_t *data, size_t size, sb_plan **out, sb_error *err) {
  auto r = decodePlan(data, size);
  if (auto *e = std::get_if<DecodeError>(&r))
    return setErr(err, "decode_error", e->message, static_cast<int64_t>(e->offset));
  auto *p = new sb_plan();
  p->layout = std::get<RelocationPlan>(std::move(r));
  *out = p;
  return 0;
}

int sb_load_typed_plan(const uint8_t *data, size_t size, sb_plan **out, sb_error *err) {
  auto r = decodeTypedPlan(data, size);
  if (auto *e = std::get_if<DecodeError>(&r))
    return setErr(err, "decode_error", e->message, static_cast<int64_t>(e->offset));
  auto *p = new sb_plan();
  p->typed = true;
  p->plan = std::get<TypedRelocationPlan>(std::move(r));
  *out = p;
  return 0;
}

int sb_plan_describe(const sb_plan *p, char *json, size_t cap) {
  std::ostringstream os;
  const RelocationPlan &lay = p->typed ? p->plan.layout : p->layout;
  os << "{\"typed\":" << (p->typed ? "true" : "false") << ",\"symbols\":[";
  for (size_t i = 0; i < lay.symbols.size(); ++i)
    os << (i ? "," : "") << q(lay.symbols[i]);
  os << "],\"num_axes\":" << lay.axes.size() << ",\"no_copy\":" << (lay.noCopy ? "true" : "false")
     << ",\"element_size\":" << lay.dst.elementType.bitwidth / 8;
  if (p->typed) {
    const TypedRelocationPlan &t = p->plan;
    os << ",\"source_dtype\":" << q(dtypeName(t.source.elementType))
       << ",\"result_dtype\":" << q(dtypeName(t.result.elementType)) << ",\"source_rank\":" << t.source.extents.size()
       << ",\"result_rank\":" << t.result.extents.size() << ",\"fills\":" << t.fills.size() << ",\"stages\":[";
    static const char *tr[] = {"cast", "quantize", "dequantize"};
    static const char *po[] = {"ieee_rne", "exact", "symmetric_rne", "affine"};
    for (size_t k = 0; k < t.stages.size(); ++k) {
      const ValueStage &s = t.stages[k];
      os << (k ? "," : "") << "{\"transform\":" << q(tr[int(s.transform)]) << ",\"policy\":" << q(po[int(s.policy)])
         << ",\"input_dtype\":" << q(dtypeName(s.input.type)) << ",\"output_dtype\":" << q(dtypeName(s.output.type))
         << ",\"input_signed\":" << (s.input.signedness == Signedness::Signed ? "true" : "false")
         << ",\"output_signed\":" << (s.output.signedness == Signedness::Signed ? "true" : "false")
         << ",\"rank\":" << s.shape.size() << ",\"axis\":" << s.axis
         << ",\"has_channel\":" << (s.hasChannel ? "true" : "false") << ",\"scale\":" << paramJson(s.scale)
         << ",\"zero_point\":" << paramJson(s.zeroPoint) << "}";
    }
    os << "],\"parameters\":[";
    std::vector<std::string> seen;
    bool first = true;
    for (size_t k = 0; k < t.stages.size(); ++k)
      for (int role = 0; role < 2; ++role) {
        const StageParam &sp = role == 0 ? t.stages[k].scale : t.stages[k].zeroPoint;
        if (sp.kind != ParamKind::Binding)
          continue;
        bool dup = false;
        for (auto &n : seen)
          dup |= n == sp.bindingName;
        if (dup)
          continue;
        seen.push_back(sp.bindingName);
        os << (first ? "" : ",") << "{\"name\":" << q(sp.bindingName) << ",\"dtype\":" << q(dtypeName(sp.elementType))
           << ",\"rank\":" << int(sp.rank) << ",\"stage\":" << k << ",\"role\":" << (role == 0 ? "\"scale\"" : "\"zero_point\"")
           << ",\"extents\":[";
        for (size_t e = 0; e < sp.bindingExtents.size(); ++e)
          os << (e ? "," : "") << exprJson(sp.bindingExtents[e]);
        os << "]}";
        first = false;
      }
    os << "]";
  }
  os << "}";
  return putJson(os.str(), json, cap);
}

void sb_plan_free(sb_plan *p) { delete p; }

int sb_bind(const sb_plan *p, int32_t nsym, const char *const *names, const int64_t *values, sb_bound **out,
            sb_error *err) {
  if (p->typed)
    return setErr(err, "bind_error", "bind expects a layout-only (v0) plan; use bind_typed");
  auto r = reloc::bind(p->layout, symbolsOf(nsym, names, values));
  if (auto *e = std::get_if<BindError>(&r))
    return setErr(err, "bind_error", e->message);
  auto *b = new sb_bound();
  b->layout = std::get<BoundPlan>(std::move(r));
  *out = b;
  return 0;
}

int sb_bind_typed(const sb_plan *p, int32_t nsym, const char *const *names, const int64_t *values, int32_t nparam,
                  const char *const *pnames, const char *const *pdtypes, const int32_t *pranks,
                  const int64_t *pextents, const void *const *pbytes, const size_t *plens, sb_bound **out,
                  sb_error *err) {
  if (!p->typed)
    return setErr(err, "bind_error", "bind_typed expects a typed (v1) plan");
  ParameterMap params;
  for (int32_t i = 0; i < nparam; ++i) {
    ParameterValue v;
    if (!parseDtype(pdtypes[i], v.elementType))
      return setErr(err, "bind_error", std::string("unknown parameter dtype ") + (pdtypes[i] ? pdtypes[i] : ""));
    if (pranks[i] == 1)
      v.extents.push_back(pextents[i]);
    const auto *bytes = static_cast<const uint8_t *>(pbytes[i]);
    v.bytes.assign(bytes, bytes + plens[i]);
    params[pnames[i]] = std::move(v);
  }
  auto r = bindTyped(p->plan, symbolsOf(nsym, names, values), params);
  if (auto *e = std::get_if<BindError>(&r))
    return setErr(err, "bind_error", e->message);
  auto *b = new sb_bound();
  b->typed = true;
  b->bound = std::get<TypedBoundPlan>(std::move(r));
  auto prog = typed::prepareProgram(b->bound);
  if (auto *e = std::get_if<typed::ExecutionError>(&prog))
    b->programError = e->code + ": " + e->message;
  else
    b->program = std::get<typed::Program>(std::move(prog));
  *out = b;
  return 0;
}

int sb_bound_describe(const sb_bound *b, char *json, size_t cap) { return putJson(boundJson(*b), json, cap); }
void sb_bound_free(sb_bound *b) { delete b; }

int sb_query_capability(const sb_bound *b, int32_t direction, int32_t cuda, char *json, size_t cap, sb_error *err) {
  if (!b->typed)
    return setErr(err, "typed_unsupported", "capability is defined for typed plans");
  if (!b->program)
    return setErr(err, "unsupported_stage", b->programError);
  auto c = dispatch::queryCapability(*b->program,
                                     direction ? TransferDirection::DeviceToHost : TransferDirection::HostToDevice,
                                     cuda != 0);
  putJson(capabilityJson(c), json, cap);
  return 0;
}

int sb_prepare_dispatch_template(const sb_bound *b, int32_t direction, int32_t policy, const char *implementation,
                                 sb_template **out, sb_error *err) {
  if (!b->typed)
    return setErr(err, "typed_unsupported", "dispatch templates are defined for typed plans");
  dispatch::Options o;
  o.cuda = true;
  o.policy = policy == 1 ? dispatch::Policy::OriginalCpu : dispatch::Policy::Auto;
  if (implementation)
    o.implementation = implementation;
  auto t = dispatch::prepareDispatchTemplate(
      b->bound, direction ? TransferDirection::DeviceToHost : TransferDirection::HostToDevice, o);
  if (auto *e = std::get_if<TransferError>(&t))
    return setErr(err, e->code, e->message);
  *out = new sb_template{std::get<dispatch::DispatchTemplate>(std::move(t))};
  return 0;
}

int sb_prepare_transfer_template(const sb_bound *b, sb_template **out, sb_error *err) {
  if (b->typed)
    return setErr(err, "typed_unsupported", "layout transfers take a layout-only (v0) bound plan");
  auto r = dispatch::prepareTransferTemplate(b->layout, TransferDirection::HostToDevice);
  if (auto *e = std::get_if<TransferError>(&r))
    return setErr(err, e->code, e->message);
  *out = new sb_template{std::get<dispatch::DispatchTemplate>(std::move(r))};
  return 0;
}

int sb_template_describe(const sb_template *t, char *json, size_t cap) {
  std::ostringstream os;
  os << "{\"capability\":" << capabilityJson(t->t.capability) << ",\"selection\":{\"implementation\":"
     << q(t->t.selection.row.label()) << ",\"policy\":" << q(t->t.selection.policy)
     << ",\"placement_reason\":" << q(t->t.selection.reason) << "}";
  if (t->t.lowered) {
    const b200::Lowered &l = *t->t.lowered;
    os << ",\"device_kernel\":" << q(b200::familyName(l.family)) << ",\"rows_chunkable\":"
       << (l.rowsChunkable ? "true" : "false") << ",\"source_outer_axis\":" << l.srcOuter
       << ",\"padded_rows\":" << l.padded[0] << ",\"dense_cover\":" << (l.denseCover ? "true" : "false")
       << ",\"row_bytes\":" << l.desc.dst_strides[0] * l.desc.dst_width;
  }
  os << "}";
  return putJson(os.str(), json, cap);
}

void sb_template_free(sb_template *t) { delete t; }

int sb_prepare_dispatch(const sb_template *t, const sb_view *src, const sb_view *dst, sb_request **out,
                        sb_error *err) {
  auto r = dispatch::prepareDispatch(t->t, toView(*src), toView(*dst));
  if (auto *e = std::get_if<TransferError>(&r))
    return setErr(err, e->code, e->message);
  *out = new sb_request{std::get<dispatch::DispatchRequest>(std::move(r))};
  return 0;
}

int sb_execute_dispatch(sb_request *req, sb_resources *res, const sb_options *opts, char *report, size_t cap,
                        sb_error *err) {
  const TransferOptions o = toOptions(opts);
  const int device = dispatch::executionDevice(req->r);
  TransferOutcome out;
  if (res) {
    out = res->res.execute(req->r, device, 2, o, nullptr);
  } else {
    dispatch::Resources local(0, 0, 1);
    out = local.execute(req->r, device, 2, o, nullptr);
  }
  putJson(reportJson(req->r.report), report, cap);
  if (out.error)
    return setErr(err, out.error->code, out.error->message);
  return 0;
}

void sb_request_free(sb_request *r) { delete r; }

int sb_execute_rows(const sb_template *t, sb_resources *res, int32_t device, const void *src, int32_t host_source,
                    void *dst, int64_t row_begin, int64_t row_end, const sb_options *opts, char *report, size_t cap,
                    sb_error *err) {
  const TransferOptions o = toOptions(opts);
  dispatch::Report rep;
  rep.implementation = t->t.selection.row.label();
  rep.policy = t->t.selection.policy;
  auto fn = [&](CudaBackend &b) {
    return dispatch::executeWindow(t->t, b, src, host_source != 0, dst, row_begin, row_end, o, rep);
  };
  TransferOutcome out;
  if (res) {
    out = res->res.withContext(device, fn, !o.asyncCompletion);
  } else {
    dispatch::Resources local(0, 0, 1);
    out = local.withContext(device, fn);
  }
  putJson(reportJson(rep), report, cap);
  if (out.error)
    return setErr(err, out.error->code, out.error->message);
  return 0;
}

int sb_execute_source_rows(const sb_template *t, sb_resources *res, int32_t device, const void *src,
                           int64_t row_begin, int64_t row_end, void *dst, const sb_options *opts, char *report,
                           size_t cap, sb_error *err) {
  const TransferOptions o = toOptions(opts);
  dispatch::Report rep;
  rep.implementation = t->t.selection.row.label();
  rep.policy = t->t.selection.policy;
  auto fn = [&](CudaBackend &b) {
    return dispatch::executeSourceRows(t->t, b, src, row_begin, row_end, dst, o, rep);
  };
  TransferOutcome out;
  if (res) {
    out = res->res.withContext(device, fn, !o.asyncCompletion);
  } else {
    dispatch::Resources local(0, 0, 1);
    out = local.withContext(device, fn);
  }
  putJson(reportJson(rep), report, cap);
  if (out.error)
    return setErr(err, out.error->code, out.error->message);
  return 0;
}

int sb_execute_source_shards(const sb_template *t, sb_resources *res, int32_t device, const void *const *srcs,
                             const int64_t *row_bounds, int32_t n, void *dst, const sb_options *opts, char *report,
                             size_t cap, sb_error *err) {
  const TransferOptions o = toOptions(opts);
  dispatch::Report rep;
  rep.implementation = t->t.selection.row.label();
  rep.policy = t->t.selection.policy;
  auto fn = [&](CudaBackend &b) {
    return dispatch::executeSourceShards(t->t, b, srcs, row_bounds, n, dst, o, rep);
  };
  TransferOutcome out;
  if (res) {
    out = res->res.withContext(device, fn, !o.asyncCompletion);
  } else {
    dispatch::Resources local(0, 0, 1);
    out = local.withContext(device, fn);
  }
  putJson(reportJson(rep), report, cap);
  if (out.error)
    return setErr(err, out.error->code, out.error->message);
  return 0;
}

int sb_ipc_handle(void *device_ptr, uint8_t handle[64], uint64_t *offset, sb_error *err) {
  size_t off = 0;
  const int rc = sbc_ipc_get_handle(device_ptr, handle, &off);
  *offset = off;
  if (rc)
    return setErr(err, "backend_failure", std::string("cudaIpcGetMemHandle: ") + sbc_error_string(rc));
  return 0;
}

int sb_ipc_open(const uint8_t handle[64], int32_t device, void **device_ptr, sb_error *err) {
  int rc = sbc_set_device(device);
  if (!rc)
    rc = sbc_ipc_open_handle(handle, device_ptr);
  if (rc)
    return setErr(err, "backend_failure", std::string("cudaIpcOpenMemHandle: ") + sbc_error_string(rc));
  return 0;
}

int sb_ipc_close(void *device_ptr, sb_error *err) {
  const int rc = sbc_ipc_close_handle(device_ptr);
  if (rc)
    return setErr(err, "backend_failure", std::string("cudaIpcCloseMemHandle: ") + sbc_error_string(rc));
  return 0;
}

int sb_execute_h2d_static(const sb_template *t, const void *source, void *destination, void *stream,
                          sb_error *err) {
  if (!t->t.lowered)
    return setErr(err, "implementation_unavailable", "template has no lowered program");
  if (!source || !destination)
    return setErr(err, "invalid_view", "source and destination must be non-null");
  // The scratch used is the current device's: the destination must live there.
  int current = -1, kind = 0, owner = -1;
  if (sbc_get_device(&current) == 0 && sbc_pointer_info(destination, &kind, &owner) == 0 && kind == 2 &&
      owner != current)
    return setErr(err, "device_mismatch", "the destination lives on cuda:" + std::to_string(owner) +
                                              ", the current device is cuda:" + std::to_string(current));
  void *scratch = nullptr;
  size_t bytes = 0;
  const int rc = sbc_static_scratch(&scratch, &bytes);
  if (rc)
    return setErr(err, "backend_failure", std::string("static scratch: ") + sbc_error_string(rc));
  auto e = b200::runH2DStatic(*t->t.lowered, source, destination, stream, static_cast<uint8_t *>(scratch), bytes);
  if (e)
    return setErr(err, e->code, e->message);
  return 0;
}

int sb_resources_create(uint64_t max_retained_bytes, uint64_t max_live_bytes, uint32_t max_contexts,
                        sb_resources **out, sb_error *err) {
  (void)err;
  *out = new sb_resources(static_cast<size_t>(max_retained_bytes), static_cast<size_t>(max_live_bytes),
                          max_contexts ? max_contexts : 8);
  return 0;
}

int sb_resources_stats(const sb_resources *r, char *json, size_t cap) {
  const dispatch::ResourceStats s = r->res.stats();
  std::ostringstream os;
  os << "{\"requests\":" << s.requests << ",\"hits\":" << s.hits << ",\"contexts\":" << s.contexts
     << ",\"device_allocations\":" << s.deviceAllocations << ",\"retained_bytes\":" << s.retainedBytes
     << ",\"device_bytes\":" << s.deviceBytes << ",\"copy_calls\":" << s.copyCalls
     << ",\"event_records\":" << s.eventRecords << ",\"event_waits\":" << s.eventWaits
     << ",\"caller_waits\":" << s.callerWaits << ",\"kernel_launches\":" << s.kernelLaunches
     << ",\"closed\":" << (s.closed ? "true" : "false") << ",\"quarantined\":" << (s.quarantined ? "true" : "false")
     << ",\"retained_limit\":" << s.retainedLimit << ",\"live_limit\":" << s.liveLimit
     << ",\"context_limit\":" << s.contextLimit << ",\"peak_live_bytes\":" << s.peakLiveBytes
     << ",\"releases\":" << s.releases << ",\"evictions\":" << s.evictions
     << ",\"retirements\":" << s.retirements << "}";
  return putJson(os.str(), json, cap);
}

int sb_resources_streams(sb_resources *r, int32_t device, void **copy_stream, void **compute_stream,
                         sb_error *err) {
  auto out = r->res.withContext(
      device,
      [&](CudaBackend &b) -> std::optional<TransferError> {
        *copy_stream = b.copyStream();
        *compute_stream = b.computeStream();
        return std::nullopt;
      },
      false); // a query: queued work stays as it is
  if (out.error)
    return setErr(err, out.error->code, out.error->message);
  return 0;
}

void sb_resources_set_acquire_timeout(sb_resources *r, int64_t ms) { r->res.setAcquireTimeout(ms); }

int sb_resources_clear(sb_resources *r, sb_error *err) {
  if (auto e = r->res.clear())
    return setErr(err, e->code, e->message);
  return 0;
}

int sb_resources_close(sb_resources *r, sb_error *err) {
  if (auto e = r->res.close())
    return setErr(err, e->code, e->message);
  return 0;
}

void sb_resources_free(sb_resources *r) { delete r; }

int sb_prepare_dispatch_group(const sb_group_entry *entries, size_t count, sb_group **out, sb_error *err) {
  std::vector<dispatch::GroupEntry> es;
  es.reserve(count);
  for (size_t i = 0; i < count; ++i) {
    dispatch::GroupEntry e;
    e.plan = entries[i].plan ? &entries[i].plan->t : nullptr;
    e.source = toView(entries[i].source);
    e.destination = toView(entries[i].destination);
    e.direction = entries[i].direction == 1 ? TransferDirection::DeviceToHost : TransferDirection::HostToDevice;
    es.push_back(std::move(e));
  }
  auto r = dispatch::prepareDispatchGroup(es);
  if (auto *e = std::get_if<TransferError>(&r))
    return setErr(err, e->code, e->message);
  *out = new sb_group{std::get<dispatch::GroupRequest>(std::move(r))};
  return 0;
}

int sb_group_report(const sb_group *grp, char *json, size_t cap) {
  const dispatch::GroupRequest &g = grp->g;
  const dispatch::GroupReport &r = g.report;
  std::ostringstream os;
  int64_t src = 0, wire = 0, dst = 0, payload = 0;
  for (const auto &rep : g.reports) {
    src += rep.sourceBytes;
    wire += rep.wireBytes;
    dst += rep.destinationBytes;
    payload += rep.payloadBytesTransferred;
  }
  os << "{\"logical_transfers\":" << g.items.size() << ",\"device\":" << g.device
     << ",\"consumed\":" << (g.consumed ? "true" : "false") << ",\"failed\":" << (g.failed ? "true" : "false")
     << ",\"payload_copy_calls\":" << r.payloadCopyCalls << ",\"parameter_uploads\":" << r.parameterUploads
     << ",\"parameter_reuses\":" << r.parameterReuses << ",\"parameter_upload_bytes\":" << r.parameterUploadBytes
     << ",\"host_transform_bytes\":" << r.hostTransformBytes << ",\"packing_bytes\":" << r.packingBytes
     << ",\"kernel_launches\":" << r.kernelLaunches << ",\"output_bytes\":" << r.outputBytes
     << ",\"copy_calls\":" << r.copyCalls << ",\"event_records\":" << r.eventRecords
     << ",\"event_waits\":" << r.eventWaits << ",\"caller_waits\":" << r.callerWaits
     << ",\"scratch_peak_bytes\":" << r.scratchPeakBytes << ",\"source_bytes\":" << src
     << ",\"wire_bytes\":" << wire << ",\"destination_bytes\":" << dst << ",\"payload_bytes_transferred\":" << payload
     << ",\"items\":[";
  for (size_t i = 0; i < g.reports.size(); ++i) {
    dispatch::Report rep = g.reports[i];
    if (!rep.executed && i < g.items.size())
      rep = g.items[i].report;
    os << (i ? "," : "") << reportJson(rep);
  }
  os << "]}";
  return putJson(os.str(), json, cap);
}

int sb_execute_dispatch_group(sb_group *grp, sb_resources *res, const sb_options *opts, char *report, size_t cap,
                              sb_error *err) {
  const TransferOptions o = toOptions(opts);
  TransferOutcome out;
  if (res) {
    out = res->res.execute(grp->g, o, nullptr);
  } else {
    dispatch::Resources local(0, 0, 1);
    TransferOptions blocking = o;
    blocking.asyncCompletion = false; // the private context ends with this call
    out = local.execute(grp->g, blocking, nullptr);
  }
  sb_group_report(grp, report, cap);
  if (out.error)
    return setErr(err, out.error->code, out.error->message);
  return 0;
}

int sb_submit_dispatch_group(sb_group *grp, sb_resources *res, const sb_options *opts, sb_completion **out,
                             sb_error *err) {
  const TransferOptions o = toOptions(opts);
  auto handle = std::make_unique<sb_completion>();
  dispatch::Resources *owner = res ? &res->res : nullptr;
  if (!owner) {
    handle->ephemeral = std::make_shared<dispatch::Resources>(0, 0, 1);
    owner = handle->ephemeral.get();
  }
  auto r = owner->submit(grp->g, o, nullptr);
  if (auto *e = std::get_if<TransferError>(&r))
    return setErr(err, e->code, e->message);
  handle->c = std::get<std::shared_ptr<dispatch::Completion>>(std::move(r));
  *out = handle.release();
  return 0;
}

void sb_group_free(sb_group *g) { delete g; }

int sb_completion_wait(sb_completion *c, sb_error *err) {
  const TransferOutcome o = c->c->wait();
  if (o.error)
    return setErr(err, o.error->code, o.error->message);
  return 0;
}

int sb_completion_query(sb_completion *c, int32_t *done, sb_error *err) {
  auto r = c->c->query();
  if (auto *e = std::get_if<TransferError>(&r))
    return setErr(err, e->code, e->message);
  *done = std::get<bool>(r) ? 1 : 0;
  return 0;
}

int sb_completion_wait_stream(sb_completion *c, void *stream, sb_error *err) {
  if (auto e = c->c->waitStream(stream))
    return setErr(err, e->code, e->message);
  return 0;
}

void sb_completion_free(sb_completion *c) { delete c; }

} // extern "C"
