// Symbol binding for v0 layout plans and v1 typed plans.
//
// Guards, messages and axis coalescing follow the reference binder
// (libreloc/src/Bind.cpp:176-385 for bind, :494-700 for bindTyped) so bound
// layouts and diagnostics are identical; see include/reloc/Bind.h.
#include "reloc/Bind.h"
#include "reloc/TypedValue.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <set>

namespace reloc {
namespace {

bool mulOk(int64_t a, int64_t b, int64_t &out) { return !__builtin_mul_overflow(a, b, &out); }

/// Floor division with the two integer-overflow cases reported.
bool floorDivide(int64_t a, int64_t b, int64_t &q, std::string &error) {
  if (b == 0) {
    error = "division by zero";
    return false;
  }
  if (a == std::numeric_limits<int64_t>::min() && b == -1) {
    error = "integer overflow in floordiv";
    return false;
  }
  q = a / b;
  if ((a % b) != 0 && ((a < 0) != (b < 0)))
    --q;
  return true;
}

/// Postfix stack machine shared by the plan and channel contexts.
bool run(const ExprStream &stream, const SymbolValues &symbols, const std::vector<int64_t> *dims, int64_t &out,
         std::string &error) {
  std::vector<int64_t> st;
  st.reserve(stream.size());
  for (const ExprToken &t : stream) {
    switch (t.op) {
    case ExprOp::PushSym:
      if (t.value < 0 || static_cast<size_t>(t.value) >= symbols.size())
        return (error = "symbol index out of range"), false;
      st.push_back(symbols[static_cast<size_t>(t.value)]);
      continue;
    case ExprOp::PushConst:
      st.push_back(t.value);
      continue;
    case ExprOp::PushDim:
      if (!dims)
        return (error = "PUSH_DIM is not valid in a plan expression"), false;
      if (t.value < 0 || static_cast<size_t>(t.value) >= dims->size())
        return (error = "dimension index out of range"), false;
      st.push_back((*dims)[static_cast<size_t>(t.value)]);
      continue;
    default:
      break;
    }
    if (st.size() < 2)
      return (error = "expression stack underflow"), false;
    const int64_t r = st.back();
    st.pop_back();
    const int64_t l = st.back();
    st.pop_back();
    int64_t v = 0;
    switch (t.op) {
    case ExprOp::Add:
      if (__builtin_add_overflow(l, r, &v))
        return (error = "integer overflow in add"), false;
      break;
    case ExprOp::Sub:
      if (__builtin_sub_overflow(l, r, &v))
        return (error = "integer overflow in sub"), false;
      break;
    case ExprOp::Mul:
      if (__builtin_mul_overflow(l, r, &v))
        return (error = "integer overflow in mul"), false;
      break;
    case ExprOp::FloorDiv:
      if (!floorDivide(l, r, v, error))
        return false;
      break;
    case ExprOp::Mod: {
      int64_t q = 0, p = 0;
      if (!floorDivide(l, r, q, error))
        return false;
      if (__builtin_mul_overflow(q, r, &p) || __builtin_sub_overflow(l, p, &v))
        return (error = "integer overflow in mod"), false;
      break;
    }
    default:
      return (error = "unknown expression opcode"), false;
    }
    st.push_back(v);
  }
  if (st.size() != 1)
    return (error = "expression did not evaluate to a single value"), false;
  out = st.back();
  return true;
}

bool field(const ExprStream &s, const SymbolValues &sym, const char *what, int64_t &out, std::string &error) {
  std::string inner;
  if (run(s, sym, nullptr, out, inner))
    return true;
  error = std::string(what) + ": " + inner;
  return false;
}

bool fields(const std::vector<ExprStream> &ss, const SymbolValues &sym, const char *what, std::vector<int64_t> &out,
            std::string &error) {
  out.clear();
  for (const ExprStream &s : ss) {
    int64_t v = 0;
    if (!field(s, sym, what, v, error))
      return false;
    out.push_back(v);
  }
  return true;
}

bool resolve(const std::vector<std::string> &names, const SymbolMap &map, SymbolValues &out, std::string &error) {
  for (const auto &kv : map)
    if (std::find(names.begin(), names.end(), kv.first) == names.end())
      return (error = "unknown symbol in binding: " + kv.first), false;
  out.assign(names.size(), 0);
  for (size_t i = 0; i < names.size(); ++i) {
    auto it = map.find(names[i]);
    if (it == map.end())
      return (error = "unbound symbol: " + names[i]), false;
    out[i] = it->second;
  }
  return true;
}

struct Dim {
  int64_t extent, src, dst;
  bool padded = false;
  int64_t lo = 0, hi = 0;
  uint64_t fill = 0;
};

/// Merge adjacent unpadded axes that are contiguous on both sides, to a
/// fixpoint. `span[c]` counts the original axes each survivor covers.
void coalesce(std::vector<Dim> &dims, std::vector<size_t> &span) {
  for (bool merged = true; merged;) {
    merged = false;
    for (size_t k = 0; k + 1 < dims.size(); ++k) {
      const Dim &o = dims[k], &i = dims[k + 1];
      if (o.padded || i.padded)
        continue;
      int64_t s = 0, d = 0, e = 0;
      if (!mulOk(i.src, i.extent, s) || !mulOk(i.dst, i.extent, d) || !mulOk(o.extent, i.extent, e))
        continue;
      if (o.src != s || o.dst != d)
        continue;
      dims[k] = Dim{e, i.src, i.dst};
      dims.erase(dims.begin() + static_cast<long>(k) + 1);
      span[k] += span[k + 1];
      span.erase(span.begin() + static_cast<long>(k) + 1);
      merged = true;
      break;
    }
  }
}

bool denseDescriptor(const TensorDesc &d, const SymbolValues &sym, const char *what, std::vector<int64_t> &extents,
                     std::string &error) {
  if (!fields(d.extents, sym, what, extents, error))
    return false;
  if (extents.empty())
    return (error = std::string(what) + ": rank must be >= 1"), false;
  for (int64_t e : extents)
    if (e < 1)
      return (error = std::string(what) + ": extents must be >= 1"), false;
  int64_t offset = 0;
  if (!field(d.offset, sym, what, offset, error))
    return false;
  if (offset != 0)
    return (error = std::string(what) + ": only zero offsets are supported"), false;
  if (!d.strides.empty()) {
    std::vector<int64_t> strides;
    if (!fields(d.strides, sym, what, strides, error))
      return false;
    int64_t expect = 1;
    for (size_t k = extents.size(); k-- > 0;) {
      if (strides[k] != expect)
        return (error = std::string(what) + ": only dense row-major strides are supported"), false;
      if (!mulOk(expect, extents[k], expect))
        return (error = std::string(what) + ": stride product overflows"), false;
    }
  }
  return true;
}

int64_t sext(uint64_t bits, uint32_t w) {
  if (w >= 64)
    return static_cast<int64_t>(bits);
  const uint64_t mask = (uint64_t{1} << w) - 1;
  uint64_t v = bits & mask;
  if (v >> (w - 1))
    v |= ~mask;
  return static_cast<int64_t>(v);
}

bool checkValues(const BoundParameter &p, bool isScale, NumericPolicyKind policy, std::string &error) {
  const uint32_t w = typed::byteWidth(p.elementType);
  for (int64_t i = 0; i < p.length; ++i) {
    const uint8_t *e = p.bytes.data() + static_cast<size_t>(i) * w;
    if (isScale) {
      float v;
      std::memcpy(&v, e, 4);
      if (!std::isfinite(v) || !(v > 0.0f))
        return (error = "scale must be finite and strictly positive"), false;
      continue;
    }
    uint64_t bits = 0;
    for (uint32_t b = 0; b < w; ++b)
      bits |= static_cast<uint64_t>(e[b]) << (8 * b);
    const int64_t zp = sext(bits, p.elementType.bitwidth);
    if (zp < -128 || zp > 127)
      return (error = "zero point must lie in [-128, 127]"), false;
    if (policy == NumericPolicyKind::SymmetricRne && zp != 0)
      return (error = "symmetric_rne admits only the zero point 0"), false;
  }
  return true;
}

BoundParameter inlineParameter(const StageParam &p) {
  BoundParameter out;
  out.present = true;
  out.elementType = p.elementType;
  out.length = static_cast<int64_t>(p.inlineBits.size());
  const uint32_t w = typed::byteWidth(p.elementType);
  for (uint64_t bits : p.inlineBits)
    for (uint32_t b = 0; b < w; ++b)
      out.bytes.push_back(static_cast<uint8_t>(bits >> (8 * b)));
  return out;
}

} // namespace

bool evalExpr(const ExprStream &stream, const SymbolValues &symbols, int64_t &out, std::string &error) {
  return run(stream, symbols, nullptr, out, error);
}

bool evalChannel(const ExprStream &stream, const SymbolValues &symbols, const std::vector<int64_t> &dims,
                 int64_t &out, std::string &error) {
  return run(stream, symbols, &dims, out, error);
}

BindResult bind(const RelocationPlan &plan, const SymbolMap &symbolMap, Strategy override) {
  std::string error;
  SymbolValues sym;
  if (!resolve(plan.symbols, symbolMap, sym, error))
    return BindError{error};

  for (const Divisibility &d : plan.divisibility) {
    if (d.divisor <= 0)
      return BindError{"divisibility divisor must be positive"};
    int64_t v = 0;
    if (!field(d.expr, sym, "divisibility expr", v, error))
      return BindError{error};
    if (v % d.divisor != 0)
      return BindError{"divisibility violated: value " + std::to_string(v) + " not divisible by " +
                       std::to_string(d.divisor)};
  }
  if (plan.axes.empty())
    return BindError{"plan must have >= 1 axis (v0)"};

  std::vector<Dim> dims(plan.axes.size());
  for (size_t k = 0; k < plan.axes.size(); ++k) {
    Dim &d = dims[k];
    if (!field(plan.axes[k].extent, sym, "axis extent", d.extent, error) ||
        !field(plan.axes[k].srcStride, sym, "axis src_stride", d.src, error) ||
        !field(plan.axes[k].dstStride, sym, "axis dst_stride", d.dst, error))
      return BindError{error};
    if (d.extent < 1)
      return BindError{"axis extent must be >= 1 (v0 rejects zero/negative)"};
    if (d.src < 0 || d.dst < 0)
      return BindError{"strides must be non-negative in v0"};
  }

  for (const PadFill &pad : plan.padFill) {
    int64_t lo = 0, hi = 0;
    if (!field(pad.lo, sym, "pad lo", lo, error) || !field(pad.hi, sym, "pad hi", hi, error))
      return BindError{error};
    if (pad.dstAxis >= plan.axes.size())
      return BindError{"pad dst_axis out of range"};
    Dim &d = dims[pad.dstAxis];
    d.padded = true;
    d.lo = lo;
    d.hi = hi;
    d.fill = pad.fillBits;
    if (lo < 0 || hi < 0)
      return BindError{"pad width negative"};
    if (plan.runtimePadCheck) {
      if (pad.dstAxis >= plan.dst.extents.size())
        return BindError{"pad dst_axis out of range for dst extents"};
      int64_t dstExtent = 0, sum = 0;
      if (!field(plan.dst.extents[pad.dstAxis], sym, "dst extent", dstExtent, error))
        return BindError{error};
      if (__builtin_add_overflow(d.extent, lo, &sum) || __builtin_add_overflow(sum, hi, &sum))
        return BindError{"overflow in pad-range check"};
      if (sum != dstExtent)
        return BindError{"pad range inconsistent: extent + lo + hi (" + std::to_string(sum) +
                         ") != dst extent (" + std::to_string(dstExtent) + ")"};
    }
  }

  std::vector<size_t> span(dims.size(), 1);
  coalesce(dims, span);
  std::vector<size_t> toCoalesced(plan.axes.size());
  for (size_t c = 0, o = 0; c < span.size(); ++c)
    for (size_t j = 0; j < span[c]; ++j)
      toCoalesced[o++] = c;

  BoundPlan b;
  b.perm = plan.perm;
  const uint32_t bits = plan.dst.elementType.bitwidth;
  if (bits == 0 || bits % 8 != 0)
    return BindError{"element type bitwidth must be a positive multiple of 8 in v0"};
  b.elementSize = bits / 8;
  b.noCopy = plan.noCopy;
  for (const Alignment &a : plan.alignment) {
    if (a.axis >= plan.axes.size())
      return BindError{"alignment axis out of range"};
    b.requiredAlignments.push_back(Alignment{static_cast<uint32_t>(toCoalesced[a.axis]), a.bytes});
  }
  int64_t total = 1;
  for (size_t k = 0; k < dims.size(); ++k) {
    b.extents.push_back(dims[k].extent);
    b.srcStrides.push_back(dims[k].src);
    b.dstStrides.push_back(dims[k].dst);
    int64_t padded = dims[k].extent;
    if (dims[k].padded) {
      b.padRegions.push_back(PadRegion{k, dims[k].lo, dims[k].hi, dims[k].fill});
      if (__builtin_add_overflow(padded, dims[k].lo, &padded) || __builtin_add_overflow(padded, dims[k].hi, &padded))
        return BindError{"overflow computing padded extent"};
    }
    if (__builtin_mul_overflow(total, padded, &total))
      return BindError{"overflow computing total element count"};
  }
  if (__builtin_mul_overflow(total, static_cast<int64_t>(b.elementSize), &b.totalBytes))
    return BindError{"overflow computing total bytes"};
  b.L = (dims.back().src == 1 && dims.back().dst == 1) ? dims.back().extent : 1;

  constexpr int64_t kSingleThreadMax = 256 * 1024, kMultiThreadMax = 256 * 1024 * 1024;
  if (override != Strategy::Auto)
    b.strategy = override;
  else if (b.noCopy)
    b.strategy = Strategy::ViewNoCopy;
  else if (b.totalBytes <= kSingleThreadMax)
    b.strategy = Strategy::SingleThreadSimd;
  else if (b.totalBytes <= kMultiThreadMax)
    b.strategy = Strategy::MultiThreadTiled;
  else
    b.strategy = Strategy::ChunkedPipeline;
  return b;
}

TypedBindResult bindTyped(const TypedRelocationPlan &plan, const SymbolMap &symbolMap,
                          const ParameterMap &parameters) {
  std::string error;
  TypedBoundPlan out;
  BindResult layout = bind(plan.layout, symbolMap);
  if (auto *e = std::get_if<BindError>(&layout))
    return BindError{"layout: " + e->message};
  out.layout = std::get<BoundPlan>(std::move(layout));
  out.layout.typed = true;
  out.fills = plan.fills;
  if (!resolve(plan.layout.symbols, symbolMap, out.symbols, error))
    return BindError{error};
  if (!denseDescriptor(plan.source, out.symbols, "source", out.sourceExtents, error) ||
      !denseDescriptor(plan.result, out.symbols, "result", out.resultExtents, error))
    return BindError{error};
  out.sourceType = plan.source.elementType;
  out.resultType = plan.result.elementType;
  if (typed::byteWidth(out.sourceType) == 0 || typed::byteWidth(out.resultType) == 0)
    return BindError{"element type bitwidth must be a positive multiple of 8"};

  std::set<std::string> used;
  for (const ValueStage &s : plan.stages) {
    BoundStage bs;
    bs.transform = s.transform;
    bs.policy = s.policy;
    bs.input = s.input;
    bs.output = s.output;
    bs.axis = s.axis;
    bs.hasChannel = s.hasChannel;
    bs.channel = s.channel;
    if (!fields(s.shape, out.symbols, "stage shape", bs.shape, error))
      return BindError{error};
    for (int64_t e : bs.shape)
      if (e < 1)
        return BindError{"stage shape extents must be >= 1"};
    if (s.axis >= 0 && static_cast<uint64_t>(s.axis) >= bs.shape.size())
      return BindError{"stage channel axis out of range"};
    const std::pair<const StageParam *, BoundParameter *> roles[] = {{&s.scale, &bs.scale},
                                                                     {&s.zeroPoint, &bs.zeroPoint}};
    for (auto [decl, target] : roles) {
      if (decl->kind == ParamKind::None)
        continue;
      const bool isScale = decl == &s.scale;
      const int64_t expected = decl->rank == 0 ? 1 : bs.shape[static_cast<size_t>(s.axis)];
      const uint32_t width = typed::byteWidth(decl->elementType);
      if (width == 0)
        return BindError{"parameter element type bitwidth must be a positive multiple of 8"};
      if (decl->kind == ParamKind::Inline) {
        *target = inlineParameter(*decl);
        if (target->length != expected)
          return BindError{"inline parameter holds " + std::to_string(target->length) +
                           " values but the channel extent is " + std::to_string(expected)};
      } else {
        const std::string &name = decl->bindingName;
        auto it = parameters.find(name);
        if (it == parameters.end())
          return BindError{"unbound parameter: " + name};
        used.insert(name);
        const ParameterValue &v = it->second;
        if (!typed::sameType(v.elementType, decl->elementType))
          return BindError{"parameter '" + name + "' element type differs from its declaration"};
        if (v.extents.size() != decl->rank)
          return BindError{"parameter '" + name + "' rank differs from its declaration"};
        int64_t declaredLength = 1;
        if (decl->rank == 1 && !field(decl->bindingExtents[0], out.symbols, "parameter extent", declaredLength, error))
          return BindError{error};
        if (declaredLength != expected)
          return BindError{"parameter '" + name + "' declares length " + std::to_string(declaredLength) +
                           " but the channel extent is " + std::to_string(expected)};
        const int64_t have = decl->rank == 0 ? 1 : v.extents[0];
        if (have != expected)
          return BindError{"parameter '" + name + "' has length " + std::to_string(have) +
                           " but the channel extent is " + std::to_string(expected)};
        int64_t need = 0;
        if (!mulOk(expected, static_cast<int64_t>(width), need))
          return BindError{"parameter byte count overflows"};
        if (v.bytes.size() != static_cast<size_t>(need))
          return BindError{"parameter '" + name + "' has " + std::to_string(v.bytes.size()) + " bytes, expected " +
                           std::to_string(need)};
        target->present = true;
        target->elementType = decl->elementType;
        target->length = expected;
        target->bytes = v.bytes;
        target->bindingName = name;
      }
      if (!checkValues(*target, isScale, s.policy, error))
        return BindError{(isScale ? "scale" : "zero_point") + std::string(": ") + error};
      int64_t sum = 0;
      if (__builtin_add_overflow(out.parameterBytes, static_cast<int64_t>(target->bytes.size()), &sum))
        return BindError{"parameter byte total overflows"};
      out.parameterBytes = sum;
    }
    out.stages.push_back(std::move(bs));
  }
  for (const auto &kv : parameters)
    if (!used.count(kv.first))
      return BindError{"unknown parameter in binding: " + kv.first};

  // Footprints per stage boundary; a pad counts from its entry stage on.
  int64_t srcElements = 1;
  for (int64_t e : out.sourceExtents)
    if (!mulOk(srcElements, e, srcElements))
      return BindError{"source element count overflows"};
  if (!mulOk(srcElements, static_cast<int64_t>(typed::byteWidth(out.sourceType)), out.sourceBytes))
    return BindError{"source byte count overflows"};
  std::vector<ExprStream> axisExprs;
  for (const Axis &a : plan.layout.axes)
    axisExprs.push_back(a.extent);
  std::vector<int64_t> axisExtents;
  if (!fields(axisExprs, out.symbols, "layout axis extent", axisExtents, error))
    return BindError{error};
  std::vector<int64_t> padWidth(axisExtents.size(), 0);
  std::vector<uint32_t> padStage(axisExtents.size(), 0);
  for (const PadFill &pad : plan.layout.padFill) {
    if (pad.dstAxis >= axisExtents.size())
      return BindError{"pad dst_axis out of range"};
    int64_t lo = 0, hi = 0, w = 0;
    if (!field(pad.lo, out.symbols, "pad lo", lo, error) || !field(pad.hi, out.symbols, "pad hi", hi, error))
      return BindError{error};
    if (lo < 0 || hi < 0 || __builtin_add_overflow(lo, hi, &w))
      return BindError{"pad widths must be non-negative"};
    padWidth[pad.dstAxis] = w;
    for (const TypedFill &f : plan.fills)
      if (f.dstAxis == pad.dstAxis)
        padStage[pad.dstAxis] = f.stage;
  }
  for (uint32_t boundary = 0; boundary <= plan.stages.size(); ++boundary) {
    StageFootprint cut;
    cut.boundary = boundary;
    cut.elementType = boundary == 0 ? out.sourceType : plan.stages[boundary - 1].output.type;
    cut.elements = 1;
    for (size_t a = 0; a < axisExtents.size(); ++a) {
      int64_t e = axisExtents[a];
      if (padWidth[a] != 0 && padStage[a] <= boundary && __builtin_add_overflow(e, padWidth[a], &e))
        return BindError{"padded extent overflows"};
      if (!mulOk(cut.elements, e, cut.elements))
        return BindError{"stage element count overflows"};
    }
    const uint32_t w = typed::byteWidth(cut.elementType);
    if (w == 0)
      return BindError{"stage element type bitwidth must be a positive multiple of 8"};
    if (!mulOk(cut.elements, static_cast<int64_t>(w), cut.bytes))
      return BindError{"stage byte count overflows"};
    out.cuts.push_back(cut);
  }
  out.destinationBytes = out.cuts.back().bytes;
  if (out.destinationBytes != out.layout.totalBytes)
    return BindError{"layout footprint (" + std::to_string(out.layout.totalBytes) +
                     " bytes) disagrees with the result descriptor (" + std::to_string(out.destinationBytes) +
                     " bytes)"};
  int64_t resElements = 1;
  for (int64_t e : out.resultExtents)
    if (!mulOk(resElements, e, resElements))
      return BindError{"result element count overflows"};
  if (resElements != out.cuts.back().elements)
    return BindError{"result descriptor element count disagrees with the layout"};
  out.requirements = {"typed_execution_dispatch"};
  return out;
}

} // namespace reloc
