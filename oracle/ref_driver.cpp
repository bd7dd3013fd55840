// Test infrastructure only: a C-ABI driver over the reference libreloc CPU
// runtime, compiled together with the reference sources into
// oracle/_ref/libreloc_ref.so by oracle/Makefile. The parity tests and the
// bench's reference arm load it through ctypes (oracle/ref.py); nothing in the
// product links it.
//
// Calls the reference's public API only:
//   decodePlan / decodeTypedPlan / peekWireVersion  (libreloc/include/reloc/Decode.h:35-52)
//   bind / bindTyped                                 (libreloc/include/reloc/Bind.h:111,205)
//   typed::prepareProgram / executeHost / executeHostChunk
//                                                    (libreloc/include/reloc/TypedExecute.h:99-170)
//   executeH2DThreaded                               (libreloc/include/reloc/Execute.h:67)
//   GatherPool                                       (libreloc/include/reloc/GatherPool.h:27)

#include "reloc/Bind.h"
#include "reloc/ChunkSchedule.h"
#include "reloc/Decode.h"
#include "reloc/Execute.h"
#include "reloc/GatherPool.h"
#include "reloc/TypedExecute.h"

#include <cstdio>
#include <cstring>
#include <memory>
#include <sstream>
#include <string>
#include <variant>

namespace {

void put(char *buf, size_t cap, const std::string &text) {
  if (!buf || cap == 0)
    return;
  size_t n = text.size() < cap - 1 ? text.size() : cap - 1;
  std::memcpy(buf, text.data(), n);
  buf[n] = 0;
}

bool parseDtype(const char *name, reloc::ElementType &out) {
  std::string s(name);
  using K = reloc::ElementTypeKind;
  if (s == "float32") out = {K::Float, 32};
  else if (s == "float16") out = {K::Float, 16};
  else if (s == "bfloat16") out = {K::BFloat, 16};
  else if (s == "float64") out = {K::Float, 64};
  else if (s == "int8") out = {K::Integer, 8};
  else if (s == "int16") out = {K::Integer, 16};
  else if (s == "int32") out = {K::Integer, 32};
  else if (s == "int64") out = {K::Integer, 64};
  else return false;
  return true;
}

template <typename T> std::string list(const std::vector<T> &v) {
  std::ostringstream os;
  os << "[";
  for (size_t i = 0; i < v.size(); ++i)
    os << (i ? "," : "") << v[i];
  os << "]";
  return os.str();
}

std::string describeLayout(const reloc::BoundPlan &b) {
  std::ostringstream os;
  os << "{\"extents\":" << list(b.extents)
     << ",\"src_strides\":" << list(b.srcStrides)
     << ",\"dst_strides\":" << list(b.dstStrides)
     << ",\"element_size\":" << b.elementSize
     << ",\"total_bytes\":" << b.totalBytes << ",\"L\":" << b.L
     << ",\"typed\":" << (b.typed ? "true" : "false") << ",\"pads\":[";
  for (size_t i = 0; i < b.padRegions.size(); ++i) {
    const auto &p = b.padRegions[i];
    os << (i ? "," : "") << "{\"axis\":" << p.axis << ",\"lo\":" << p.lo
       << ",\"hi\":" << p.hi << ",\"fill\":" << p.fillBits << "}";
  }
  os << "]}";
  return os.str();
}

struct Typed {
  reloc::typed::Program program;
};

struct Layout {
  reloc::BoundPlan bound;
};

bool buildSymbols(int nsym, const char *const *names, const int64_t *values,
                  reloc::SymbolMap &out) {
  for (int i = 0; i < nsym; ++i)
    out[names[i]] = values[i];
  return true;
}

} // namespace

extern "C" {

int ref_wire_version(const uint8_t *data, size_t size) {
  auto v = reloc::peekWireVersion(data, size);
  return v ? static_cast<int>(*v) : -1;
}

/// Decode only (decoder parity). typed: 0 = decodePlan, 1 = decodeTypedPlan.
/// Returns 0 on success, 1 with the byte offset and message on failure.
int ref_decode(const uint8_t *data, size_t size, int typed,
               uint64_t *offset, char *msg, size_t cap) {
  if (typed) {
    auto r = reloc::decodeTypedPlan(data, size);
    if (auto *e = std::get_if<reloc::DecodeError>(&r)) {
      *offset = e->offset;
      put(msg, cap, e->message);
      return 1;
    }
    return 0;
  }
  auto r = reloc::decodePlan(data, size);
  if (auto *e = std::get_if<reloc::DecodeError>(&r)) {
    *offset = e->offset;
    put(msg, cap, e->message);
    return 1;
  }
  return 0;
}

/// decodeTypedPlan + bindTyped + prepareProgram. Parameters: per parameter a
/// name, dtype name, rank (0/1), extent (rank 1) and little-endian bytes.
void *ref_typed_prepare(const uint8_t *data, size_t size, int nsym,
                        const char *const *names, const int64_t *values,
                        int nparam, const char *const *pnames,
                        const char *const *pdtypes, const int *pranks,
                        const int64_t *pextents, const uint8_t *const *pbytes,
                        const size_t *plens, char *err, size_t cap) {
  auto decoded = reloc::decodeTypedPlan(data, size);
  if (auto *e = std::get_if<reloc::DecodeError>(&decoded)) {
    put(err, cap,
        "decode: offset " + std::to_string(e->offset) + ": " + e->message);
    return nullptr;
  }
  reloc::SymbolMap symbols;
  buildSymbols(nsym, names, values, symbols);
  reloc::ParameterMap params;
  for (int i = 0; i < nparam; ++i) {
    reloc::ParameterValue v;
    if (!parseDtype(pdtypes[i], v.elementType)) {
      put(err, cap, std::string("unknown dtype ") + pdtypes[i]);
      return nullptr;
    }
    if (pranks[i] == 1)
      v.extents.push_back(pextents[i]);
    v.bytes.assign(pbytes[i], pbytes[i] + plens[i]);
    params[pnames[i]] = std::move(v);
  }
  auto bound = reloc::bindTyped(std::get<reloc::TypedRelocationPlan>(decoded),
                                symbols, params);
  if (auto *e = std::get_if<reloc::BindError>(&bound)) {
    put(err, cap, "bind: " + e->message);
    return nullptr;
  }
  auto program =
      reloc::typed::prepareProgram(std::get<reloc::TypedBoundPlan>(bound));
  if (auto *e = std::get_if<reloc::typed::ExecutionError>(&program)) {
    put(err, cap, "program: " + e->code + ": " + e->message);
    return nullptr;
  }
  auto *h = new Typed{std::get<reloc::typed::Program>(std::move(program))};
  return h;
}

/// A JSON description of the bound plan and the checked program.
int ref_typed_describe(void *handle, char *buf, size_t cap) {
  const auto &p = static_cast<Typed *>(handle)->program;
  const auto &b = p.plan;
  std::ostringstream os;
  os << "{\"layout\":" << describeLayout(b.layout)
     << ",\"source_extents\":" << list(b.sourceExtents)
     << ",\"result_extents\":" << list(b.resultExtents)
     << ",\"source_bytes\":" << b.sourceBytes
     << ",\"destination_bytes\":" << b.destinationBytes
     << ",\"parameter_bytes\":" << b.parameterBytes << ",\"cuts\":[";
  for (size_t i = 0; i < b.cuts.size(); ++i)
    os << (i ? "," : "") << "{\"boundary\":" << b.cuts[i].boundary
       << ",\"elements\":" << b.cuts[i].elements
       << ",\"bytes\":" << b.cuts[i].bytes << "}";
  os << "],\"stages\":[";
  for (size_t k = 0; k < p.stages.size(); ++k) {
    const auto &s = p.stages[k];
    std::vector<uint32_t> inv, sc;
    for (float f : s.invScale) {
      uint32_t u;
      std::memcpy(&u, &f, 4);
      inv.push_back(u);
    }
    for (float f : s.scale) {
      uint32_t u;
      std::memcpy(&u, &f, 4);
      sc.push_back(u);
    }
    os << (k ? "," : "") << "{\"transform\":" << int(s.transform)
       << ",\"policy\":" << int(s.policy)
       << ",\"per_channel\":" << (s.perChannel ? "true" : "false")
       << ",\"channel_is_dim\":" << (s.channelIsDim ? "true" : "false")
       << ",\"channel_dim\":" << s.channelDim
       << ",\"channel_length\":" << s.channelLength
       << ",\"scale_bits\":" << list(sc) << ",\"inv_scale_bits\":" << list(inv)
       << ",\"zero_point\":" << list(s.zeroPoint) << "}";
  }
  os << "],\"host_kernel\":\""
     << reloc::typed::hostKernelName(
            reloc::typed::hostKernel(p, 0, static_cast<uint32_t>(p.stages.size())))
     << "\"}";
  put(buf, cap, os.str());
  return static_cast<int>(os.str().size());
}

/// typed::executeHost over all stages, host -> host. threads as executeHost.
int ref_typed_execute(void *handle, const void *src, void *dst,
                      unsigned threads, char *err, size_t cap) {
  const auto &p = static_cast<Typed *>(handle)->program;
  auto e = reloc::typed::executeHost(p, 0, static_cast<uint32_t>(p.stages.size()),
                                     src, dst, nullptr, threads);
  if (e) {
    put(err, cap, e->code + ": " + e->message);
    return 1;
  }
  return 0;
}

/// The same execution over a caller-owned GatherPool (CPU baseline timing).
int ref_typed_execute_pool(void *handle, const void *src, void *dst,
                           void *pool, char *err, size_t cap) {
  const auto &p = static_cast<Typed *>(handle)->program;
  auto e = reloc::typed::executeHost(p, 0, static_cast<uint32_t>(p.stages.size()),
                                     src, dst,
                                     static_cast<reloc::GatherPool *>(pool), 1);
  if (e) {
    put(err, cap, e->code + ": " + e->message);
    return 1;
  }
  return 0;
}

/// typed::executeHostChunk over the physical outer-row window [begin, end) of
/// the bound layout (pad rows included); dst receives only the window.
int ref_typed_execute_rows(void *handle, int64_t begin, int64_t end,
                           const void *src, void *dst, unsigned threads,
                           char *err, size_t cap) {
  const auto &p = static_cast<Typed *>(handle)->program;
  const auto &l = p.plan.layout;
  const uint32_t width = reloc::typed::widthAt(p, static_cast<uint32_t>(p.stages.size()));
  int64_t lo = 0, padded = l.extents.front();
  for (const auto &pad : l.padRegions)
    if (pad.axis == 0) {
      lo = pad.lo;
      padded += pad.lo + pad.hi;
    }
  const int64_t rowBytes = l.dstStrides.front() * width;
  reloc::Chunk chunk;
  chunk.paddedBegin = begin;
  chunk.paddedEnd = end;
  chunk.validBegin = std::min(std::max<int64_t>(begin - lo, 0), l.extents.front());
  chunk.validEnd = std::min(std::max<int64_t>(end - lo, chunk.validBegin), l.extents.front());
  chunk.byteOffset = begin * rowBytes;
  chunk.bytes = static_cast<size_t>((end - begin) * rowBytes);
  (void)padded;
  auto e = reloc::typed::executeHostChunk(
      p, 0, static_cast<uint32_t>(p.stages.size()), src, dst, chunk, nullptr,
      threads);
  if (e) {
    put(err, cap, e->code + ": " + e->message);
    return 1;
  }
  return 0;
}

void ref_typed_free(void *handle) { delete static_cast<Typed *>(handle); }

/// decodePlan + bind (v0 layout plans).
void *ref_layout_prepare(const uint8_t *data, size_t size, int nsym,
                         const char *const *names, const int64_t *values,
                         char *err, size_t cap) {
  auto decoded = reloc::decodePlan(data, size);
  if (auto *e = std::get_if<reloc::DecodeError>(&decoded)) {
    put(err, cap,
        "decode: offset " + std::to_string(e->offset) + ": " + e->message);
    return nullptr;
  }
  reloc::SymbolMap symbols;
  buildSymbols(nsym, names, values, symbols);
  auto bound = reloc::bind(std::get<reloc::RelocationPlan>(decoded), symbols);
  if (auto *e = std::get_if<reloc::BindError>(&bound)) {
    put(err, cap, "bind: " + e->message);
    return nullptr;
  }
  return new Layout{std::get<reloc::BoundPlan>(std::move(bound))};
}

int ref_layout_describe(void *handle, char *buf, size_t cap) {
  std::string s = describeLayout(static_cast<Layout *>(handle)->bound);
  put(buf, cap, s);
  return static_cast<int>(s.size());
}

/// executeH2DThreaded host -> host (fills pads, then gathers).
int ref_layout_execute(void *handle, const void *src, void *dst,
                       unsigned threads) {
  reloc::executeH2DThreaded(static_cast<Layout *>(handle)->bound, src, dst,
                            threads);
  return 0;
}

void ref_layout_free(void *handle) { delete static_cast<Layout *>(handle); }

void *ref_pool_create(unsigned threads) {
  return new reloc::GatherPool(threads);
}
int ref_pool_threads(void *pool) {
  return static_cast<reloc::GatherPool *>(pool)->threadCount();
}
void ref_pool_free(void *pool) { delete static_cast<reloc::GatherPool *>(pool); }

} // extern "C"
