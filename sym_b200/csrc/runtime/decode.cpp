// Strict wire decoder for v0 layout plans and v1 typed plans.
//
// Behaviour follows the reference decoder (libreloc/src/Decode.cpp:868-960,
// spec docs/reloc-plan-format.md): the same checks, in the same order, with
// the same byte offsets and messages, so that a caller that reports or tests
// diagnostics sees identical results. The implementation is a cursor with
// first-error-wins recording and one parse function per wire construct.
#include "reloc/Decode.h"
#include "reloc/TypedValue.h"

#include <cmath>
#include <cstring>

namespace reloc {
namespace {

class Cursor {
public:
  Cursor(const uint8_t *data, size_t size) : data_(data), size_(size) {}
  size_t pos() const { return pos_; }
  size_t left() const { return size_ - pos_; }
  bool failAt(size_t at, std::string msg) {
    if (!err_.has_value())
      err_ = DecodeError{at, std::move(msg)};
    return false;
  }
  bool fail(std::string msg) { return failAt(pos_, std::move(msg)); }
  DecodeError error() const { return *err_; }

  template <typename T> bool le(T &out, const char *what) {
    if (left() < sizeof(T))
      return fail(std::string("truncated: expected ") + what);
    uint64_t v = 0;
    for (size_t i = 0; i < sizeof(T); ++i)
      v |= static_cast<uint64_t>(data_[pos_ + i]) << (8 * i);
    pos_ += sizeof(T);
    std::memcpy(&out, &v, sizeof(T)); // little-endian host
    return true;
  }
  bool u8(uint8_t &o) { return le(o, "u8"); }
  bool u32(uint32_t &o) { return le(o, "u32"); }
  bool u64(uint64_t &o) { return le(o, "u64"); }
  bool i64(int64_t &o) {
    uint64_t raw;
    if (!u64(raw))
      return false;
    std::memcpy(&o, &raw, 8);
    return true;
  }
  /// A count that sizes an allocation: never larger than the bytes left.
  bool count(uint32_t &o, const char *what) {
    const size_t at = pos_;
    if (!u32(o))
      return false;
    if (o > left())
      return failAt(at, std::string("count exceeds remaining bytes: ") + what);
    return true;
  }
  bool str(std::string &o) {
    uint32_t n;
    if (!count(n, "string length"))
      return false;
    o.assign(reinterpret_cast<const char *>(data_ + pos_), n);
    pos_ += n;
    return true;
  }
  bool skip(size_t n) {
    if (left() < n)
      return fail("truncated: expected " + std::to_string(n) + " bytes");
    pos_ += n;
    return true;
  }
  const uint8_t *data() const { return data_; }

private:
  const uint8_t *data_;
  size_t size_;
  size_t pos_ = 0;
  std::optional<DecodeError> err_;
};

/// Where an expression is parsed decides which leaf opcodes it may use.
enum class Where { Plan, Inverse, Channel };

bool readExpr(Cursor &c, Where where, size_t nsym, size_t ndim, ExprStream &out) {
  const size_t start = c.pos();
  uint32_t n;
  if (!c.count(n, "expression op_count"))
    return false;
  if (n == 0)
    return c.failAt(start, "empty expression stream");
  out.clear();
  out.reserve(n);
  int64_t depth = 0;
  for (uint32_t i = 0; i < n; ++i) {
    const size_t at = c.pos();
    uint8_t code;
    if (!c.u8(code))
      return false;
    ExprToken tok{static_cast<ExprOp>(code), 0};
    if (code == 0x00 || code == 0x07) { // leaf with a u32 index
      if (code == 0x00 && where == Where::Inverse)
        return c.failAt(at, "PUSH_SYM is not allowed in inverse expressions");
      if (code == 0x07 && where == Where::Plan)
        return c.failAt(at, "PUSH_DIM is only allowed in inverse and channel expressions");
      uint32_t index;
      if (!c.u32(index))
        return false;
      if (code == 0x00 && index >= nsym)
        return c.failAt(at, "PUSH_SYM symbol index out of range");
      if (code == 0x07 && index >= ndim)
        return c.failAt(at, "PUSH_DIM dim index out of range");
      tok.value = index;
      ++depth;
    } else if (code == 0x01) {
      if (!c.i64(tok.value))
        return false;
      ++depth;
    } else if (code >= 0x02 && code <= 0x06) {
      if (depth < 2)
        return c.failAt(at, "expression stack underflow");
      --depth;
    } else {
      return c.failAt(at, "unknown expression opcode");
    }
    out.push_back(tok);
  }
  if (depth != 1)
    return c.failAt(start, "expression stream must leave exactly one value");
  return true;
}

bool readType(Cursor &c, ElementType &out) {
  const size_t at = c.pos();
  uint8_t kind;
  uint32_t bits;
  if (!c.u8(kind) || !c.u32(bits))
    return false;
  bool ok = false;
  if (kind == 0)
    ok = bits == 16 || bits == 32 || bits == 64;
  else if (kind == 1)
    ok = bits == 16;
  else if (kind == 2)
    ok = bits >= 1 && bits <= 64;
  else if (kind == 3)
    ok = bits == 64;
  if (!ok)
    return c.failAt(at, "invalid element type kind/bitwidth");
  out = ElementType{static_cast<ElementTypeKind>(kind), bits};
  return true;
}

bool readExprList(Cursor &c, uint32_t n, size_t nsym, std::vector<ExprStream> &out) {
  out.clear();
  out.reserve(n);
  for (uint32_t i = 0; i < n; ++i) {
    ExprStream e;
    if (!readExpr(c, Where::Plan, nsym, 0, e))
      return false;
    out.push_back(std::move(e));
  }
  return true;
}

bool readTensor(Cursor &c, size_t nsym, TensorDesc &out) {
  uint32_t rank;
  if (!c.count(rank, "tensor_desc rank") || !readExprList(c, rank, nsym, out.extents))
    return false;
  const size_t at = c.pos();
  uint32_t nstrides;
  if (!c.count(nstrides, "tensor_desc stride_count"))
    return false;
  if (nstrides != 0 && nstrides != rank)
    return c.failAt(at, "tensor_desc stride_count must be 0 or the rank");
  if (!readExprList(c, nstrides, nsym, out.strides))
    return false;
  return readExpr(c, Where::Plan, nsym, 0, out.offset) && readType(c, out.elementType);
}

bool readFlag(Cursor &c, uint8_t &out, const char *message) {
  const size_t at = c.pos();
  if (!c.u8(out))
    return false;
  return out <= 1 || c.failAt(at, message);
}

/// v0 sections 3..12 (also the body of a v1 layout).
bool readLayout(Cursor &c, RelocationPlan &plan) {
  const size_t nsym = plan.symbols.size();
  if (!readTensor(c, nsym, plan.src))
    return false;
  const size_t dstAt = c.pos();
  if (!readTensor(c, nsym, plan.dst))
    return false;

  const size_t permAt = c.pos();
  uint32_t nperm;
  if (!c.count(nperm, "perm count"))
    return false;
  plan.perm.resize(nperm);
  for (uint32_t &p : plan.perm)
    if (!c.u32(p))
      return false;

  const size_t axesAt = c.pos();
  uint32_t naxes;
  if (!c.count(naxes, "axes count"))
    return false;
  if (naxes < 1)
    return c.failAt(axesAt, "axis count must be >= 1");
  plan.axes.resize(naxes);
  for (Axis &a : plan.axes)
    if (!c.str(a.name) || !readExpr(c, Where::Plan, nsym, 0, a.extent) ||
        !readExpr(c, Where::Plan, nsym, 0, a.srcStride) || !readExpr(c, Where::Plan, nsym, 0, a.dstStride))
      return false;

  // perm is checked against the axis count, which is only known now.
  if (plan.perm.size() != naxes)
    return c.failAt(permAt, "perm size must equal the axis count");
  std::vector<char> seen(naxes, 0);
  for (uint32_t p : plan.perm) {
    if (p >= naxes || seen[p])
      return c.failAt(permAt, "perm is not a permutation of [0, axis count)");
    seen[p] = 1;
  }
  if (plan.dst.extents.size() != naxes)
    return c.failAt(dstAt, "dst rank must equal the axis count");

  uint32_t npad;
  if (!c.count(npad, "pad_fill count"))
    return false;
  plan.padFill.resize(npad);
  for (PadFill &p : plan.padFill) {
    const size_t at = c.pos();
    if (!c.u32(p.dstAxis))
      return false;
    if (p.dstAxis >= naxes)
      return c.failAt(at, "pad_fill dst_axis out of range");
    if (!readExpr(c, Where::Plan, nsym, 0, p.lo) || !readExpr(c, Where::Plan, nsym, 0, p.hi) ||
        !readType(c, p.fillType) || !c.u64(p.fillBits))
      return false;
  }

  uint32_t ndiv;
  if (!c.count(ndiv, "divisibility count"))
    return false;
  plan.divisibility.resize(ndiv);
  for (Divisibility &d : plan.divisibility)
    if (!readExpr(c, Where::Plan, nsym, 0, d.expr) || !c.i64(d.divisor))
      return false;

  uint32_t nalign;
  if (!c.count(nalign, "alignment count"))
    return false;
  plan.alignment.resize(nalign);
  for (Alignment &a : plan.alignment) {
    const size_t at = c.pos();
    if (!c.u32(a.axis))
      return false;
    if (a.axis >= naxes)
      return c.failAt(at, "alignment axis out of range");
    if (!c.i64(a.bytes))
      return false;
  }

  const size_t contAt = c.pos();
  uint32_t ncont;
  if (!c.count(ncont, "contiguity count"))
    return false;
  if (ncont != 0 && ncont != naxes)
    return c.failAt(contAt, "contiguity count must be 0 or the axis count");
  plan.contiguity.resize(ncont);
  for (uint8_t &f : plan.contiguity)
    if (!readFlag(c, f, "contiguity flag must be 0 or 1"))
      return false;

  uint8_t noCopy, padCheck;
  if (!readFlag(c, noCopy, "no_copy flag must be 0 or 1") ||
      !readFlag(c, padCheck, "runtime_pad_check flag must be 0 or 1"))
    return false;
  plan.noCopy = noCopy;
  plan.runtimePadCheck = padCheck;

  const size_t dimsAt = c.pos();
  uint32_t ndims;
  if (!c.u32(ndims))
    return false;
  const size_t resAt = c.pos();
  uint32_t nres;
  if (!c.u32(nres))
    return false;
  if (ndims != naxes)
    return c.failAt(dimsAt, "inverse num_dims must equal the axis count");
  if (nres != naxes)
    return c.failAt(resAt, "inverse num_results must equal the axis count");
  plan.inverse.resize(nres);
  for (ExprStream &e : plan.inverse)
    if (!readExpr(c, Where::Inverse, nsym, ndims, e))
      return false;
  return true;
}

bool readHeader(Cursor &c, uint32_t version, std::vector<std::string> &symbols) {
  if (c.left() < 4)
    return c.fail("truncated: expected magic");
  if (std::memcmp(c.data(), "RPLN", 4) != 0)
    return c.failAt(0, "bad magic (expected RPLN)");
  c.skip(4);
  const size_t at = c.pos();
  uint32_t v;
  if (!c.u32(v))
    return false;
  if (v != version)
    return c.failAt(at, "unsupported wire format version");
  uint32_t n;
  if (!c.count(n, "symbol table count"))
    return false;
  symbols.resize(n);
  for (std::string &s : symbols)
    if (!c.str(s))
      return false;
  return true;
}

// ----- v1 -------------------------------------------------------------------

bool isF(ElementType t, uint32_t w) { return t.kind == ElementTypeKind::Float && t.bitwidth == w; }
bool isBF(ElementType t) { return t.kind == ElementTypeKind::BFloat && t.bitwidth == 16; }
bool isI8(ElementType t) { return t.kind == ElementTypeKind::Integer && t.bitwidth == 8; }

bool readStageType(Cursor &c, StageType &out) {
  if (!readType(c, out.type))
    return false;
  const size_t at = c.pos();
  uint8_t s;
  if (!c.u8(s))
    return false;
  if (s > 2)
    return c.failAt(at, "invalid stage type signedness");
  out.signedness = static_cast<Signedness>(s);
  return true;
}

bool readParam(Cursor &c, size_t nsym, StageParam &out) {
  const size_t at = c.pos();
  uint8_t kind;
  if (!c.u8(kind))
    return false;
  if (kind > 2)
    return c.failAt(at, "invalid parameter kind");
  out.kind = static_cast<ParamKind>(kind);
  if (out.kind == ParamKind::None)
    return true;
  if (out.kind == ParamKind::Binding) {
    const size_t nameAt = c.pos();
    if (!c.str(out.bindingName))
      return false;
    if (out.bindingName.empty())
      return c.failAt(nameAt, "binding name must not be empty");
  }
  const size_t rankAt = c.pos();
  if (!c.u8(out.rank))
    return false;
  if (out.rank > 1)
    return c.failAt(rankAt, "parameter rank must be 0 or 1");
  if (out.kind == ParamKind::Binding) {
    for (uint8_t i = 0; i < out.rank; ++i) {
      ExprStream e;
      if (!readExpr(c, Where::Plan, nsym, 0, e))
        return false;
      out.bindingExtents.push_back(std::move(e));
    }
    return readType(c, out.elementType);
  }
  if (!readType(c, out.elementType))
    return false;
  const size_t countAt = c.pos();
  uint32_t n;
  if (!c.count(n, "inline parameter count"))
    return false;
  if (n == 0)
    return c.failAt(countAt, "inline parameter must hold a value");
  if (out.rank == 0 && n != 1)
    return c.failAt(countAt, "rank-0 inline parameter must hold exactly one value");
  if (n > c.left() / 8)
    return c.failAt(countAt, "count exceeds remaining bytes: inline parameter");
  out.inlineBits.resize(n);
  for (uint64_t &b : out.inlineBits)
    if (!c.u64(b))
      return false;
  return true;
}

bool readStage(Cursor &c, size_t nsym, size_t resultRank, ValueStage &s) {
  const size_t at = c.pos();
  uint8_t transform, policy;
  if (!c.u8(transform))
    return false;
  if (transform > 2)
    return c.failAt(at, "unknown stage transform");
  s.transform = static_cast<ValueTransformKind>(transform);
  const size_t policyAt = c.pos();
  if (!c.u8(policy))
    return false;
  if (policy > 3)
    return c.failAt(policyAt, "unknown numerical policy");
  s.policy = static_cast<NumericPolicyKind>(policy);
  if (!readStageType(c, s.input) || !readStageType(c, s.output))
    return false;
  const size_t rankAt = c.pos();
  uint32_t rank;
  if (!c.count(rank, "stage shape rank"))
    return false;
  if (rank == 0)
    return c.failAt(rankAt, "stage shape must have rank >= 1");
  if (!readExprList(c, rank, nsym, s.shape))
    return false;
  if (!readParam(c, nsym, s.scale) || !readParam(c, nsym, s.zeroPoint) || !c.i64(s.axis))
    return false;
  uint8_t has;
  if (!readFlag(c, has, "has_channel flag must be 0 or 1"))
    return false;
  s.hasChannel = has;
  if (s.hasChannel) {
    const size_t dimsAt = c.pos();
    uint32_t ndims;
    if (!c.u32(ndims))
      return false;
    if (ndims != resultRank)
      return c.failAt(dimsAt, "channel map num_dims must equal the result rank");
    if (!readExpr(c, Where::Channel, nsym, ndims, s.channel))
      return false;
  }
  return true;
}

bool sameStream(const ExprStream &a, const ExprStream &b) {
  if (a.size() != b.size())
    return false;
  for (size_t i = 0; i < a.size(); ++i)
    if (a[i].op != b[i].op || a[i].value != b[i].value)
      return false;
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

bool isNaN(uint64_t bits, ElementType t) {
  if (isBF(t))
    return ((bits >> 7) & 0xffu) == 0xffu && (bits & 0x7fu);
  if (isF(t, 32))
    return ((bits >> 23) & 0xffu) == 0xffu && (bits & 0x7fffffu);
  if (isF(t, 16))
    return ((bits >> 10) & 0x1fu) == 0x1fu && (bits & 0x3ffu);
  return false;
}

/// Signature check of one stage; returns the message or nullptr.
const char *stageSignature(const ValueStage &s) {
  const bool signless = s.input.signedness == Signedness::Signless && s.output.signedness == Signedness::Signless;
  switch (s.transform) {
  case ValueTransformKind::Cast: {
    const bool narrow = isF(s.input.type, 32) && (isF(s.output.type, 16) || isBF(s.output.type)) &&
                        s.policy == NumericPolicyKind::IeeeRne;
    const bool widen = (isF(s.input.type, 16) || isBF(s.input.type)) && isF(s.output.type, 32) &&
                       s.policy == NumericPolicyKind::Exact;
    if (!(narrow || widen) || !signless)
      return "invalid cast signature (f32 -> f16/bf16 ieee_rne or f16/bf16 -> f32 exact, signless)";
    if (s.scale.kind != ParamKind::None || s.zeroPoint.kind != ParamKind::None || s.axis != -1 || s.hasChannel)
      return "cast stages carry no parameters";
    return nullptr;
  }
  case ValueTransformKind::Quantize:
    if (!isF(s.input.type, 32) || s.input.signedness != Signedness::Signless || !isI8(s.output.type) ||
        s.output.signedness != Signedness::Signed || s.policy != NumericPolicyKind::SymmetricRne)
      return "invalid quantize signature (f32 -> signed int 8, symmetric_rne)";
    return nullptr;
  case ValueTransformKind::Dequantize:
    if (!isI8(s.input.type) || s.input.signedness != Signedness::Signed || !isF(s.output.type, 32) ||
        s.output.signedness != Signedness::Signless || s.policy != NumericPolicyKind::Affine)
      return "invalid dequantize signature (signed int 8 -> f32, affine)";
    return nullptr;
  }
  return nullptr;
}

/// Parameter checks of a quantize/dequantize stage; message or empty.
std::string stageParameters(const ValueStage &s) {
  if (s.scale.kind == ParamKind::None)
    return "quantize/dequantize stages require a scale";
  if (!isF(s.scale.elementType, 32))
    return "scale element type must be f32";
  if (s.zeroPoint.kind != ParamKind::None) {
    if (s.zeroPoint.elementType.kind != ElementTypeKind::Integer)
      return "zero_point element type must be an integer";
    if (s.zeroPoint.kind == ParamKind::Binding && s.zeroPoint.elementType.bitwidth != 32)
      return "zero_point bindings must declare int 32";
  }
  if (s.axis == -1) {
    if (s.scale.rank != 0 || (s.zeroPoint.kind != ParamKind::None && s.zeroPoint.rank != 0) || s.hasChannel)
      return "per-tensor stage requires rank-0 parameters and no channel map";
  } else {
    if (s.axis < 0 || static_cast<uint64_t>(s.axis) >= s.shape.size())
      return "axis out of range for the stage shape";
    if (s.scale.rank != 1)
      return "per-channel stage requires a rank-1 scale";
    if (!s.hasChannel)
      return "per-channel stage requires a channel map";
    const ExprStream &ext = s.shape[static_cast<size_t>(s.axis)];
    if (ext.size() == 1 && ext[0].op == ExprOp::PushConst)
      for (const StageParam *p : {&s.scale, &s.zeroPoint})
        if (p->kind == ParamKind::Inline && p->rank == 1 &&
            static_cast<int64_t>(p->inlineBits.size()) != ext[0].value)
          return "inline parameter length must equal the channel extent";
  }
  if (s.scale.kind == ParamKind::Inline)
    for (uint64_t b : s.scale.inlineBits) {
      const uint32_t u = static_cast<uint32_t>(b);
      float v;
      std::memcpy(&v, &u, 4);
      if (!std::isfinite(v) || !(v > 0.0f))
        return "inline scale must be finite and strictly positive";
    }
  if (s.zeroPoint.kind == ParamKind::Inline)
    for (uint64_t b : s.zeroPoint.inlineBits) {
      const int64_t v = sext(b, s.zeroPoint.elementType.bitwidth);
      if (v < -128 || v > 127)
        return "inline zero point out of [-128, 127]";
      if (s.policy == NumericPolicyKind::SymmetricRne && v != 0)
        return "symmetric_rne admits only the constant zero point 0";
    }
  if (s.policy == NumericPolicyKind::SymmetricRne && s.zeroPoint.kind == ParamKind::Binding)
    return "symmetric_rne rejects a zero-point binding";
  if (s.scale.kind == ParamKind::Binding && s.zeroPoint.kind == ParamKind::Binding &&
      s.scale.bindingName == s.zeroPoint.bindingName)
    return "runtime parameters must use distinct binding names";
  return {};
}

bool validateTypedPlan(Cursor &c, const TypedRelocationPlan &plan, size_t layoutAt, size_t stagesAt,
                       const std::vector<size_t> &stageAt, size_t fillsAt, const std::vector<size_t> &fillAt) {
  using typed::sameType;
  const ElementType src = plan.source.elementType, res = plan.result.elementType;
  if (!sameType(plan.layout.src.elementType, src))
    return c.failAt(layoutAt, "layout src element type must equal the source type");
  if (!sameType(plan.layout.dst.elementType, res))
    return c.failAt(layoutAt, "layout dst element type must equal the result type");
  if (plan.layout.src.extents.size() != plan.source.extents.size())
    return c.failAt(layoutAt, "layout src rank must equal the source rank");
  if (plan.stages.empty())
    return c.failAt(stagesAt, "typed plan needs at least one stage");
  if (!sameType(plan.stages.front().input.type, src))
    return c.failAt(stageAt[0], "stage 0 input type must equal the source type");
  for (size_t k = 1; k < plan.stages.size(); ++k)
    if (!sameType(plan.stages[k].input.type, plan.stages[k - 1].output.type))
      return c.failAt(stageAt[k], "stage input type must equal the previous stage's output type");
  if (!sameType(plan.stages.back().output.type, res))
    return c.failAt(stageAt.back(), "last stage output type must equal the result type");

  std::vector<const StageParam *> declared;
  for (size_t k = 0; k < plan.stages.size(); ++k) {
    const ValueStage &s = plan.stages[k];
    if (const char *m = stageSignature(s))
      return c.failAt(stageAt[k], m);
    if (s.transform == ValueTransformKind::Cast)
      continue;
    const std::string m = stageParameters(s);
    if (!m.empty())
      return c.failAt(stageAt[k], m);
    for (const StageParam *p : {&s.scale, &s.zeroPoint}) {
      if (p->kind != ParamKind::Binding)
        continue;
      for (const StageParam *q : declared) {
        if (q->bindingName != p->bindingName)
          continue;
        bool same = q->rank == p->rank && sameType(q->elementType, p->elementType) &&
                    q->bindingExtents.size() == p->bindingExtents.size();
        for (size_t e = 0; same && e < q->bindingExtents.size(); ++e)
          same = sameStream(q->bindingExtents[e], p->bindingExtents[e]);
        if (!same)
          return c.failAt(stageAt[k], "conflicting parameter declaration for binding '" + p->bindingName + "'");
      }
      declared.push_back(p);
    }
  }

  std::vector<char> padFilled(plan.layout.padFill.size(), 0);
  for (size_t i = 0; i < plan.fills.size(); ++i) {
    const TypedFill &f = plan.fills[i];
    const PadFill *pad = nullptr;
    for (size_t p = 0; p < plan.layout.padFill.size(); ++p)
      if (plan.layout.padFill[p].dstAxis == f.dstAxis) {
        if (padFilled[p])
          return c.failAt(fillAt[i], "duplicate fill for a layout pad");
        padFilled[p] = 1;
        pad = &plan.layout.padFill[p];
      }
    if (!pad)
      return c.failAt(fillAt[i], "fill dst_axis has no layout pad");
    if (f.stage > plan.stages.size())
      return c.failAt(fillAt[i], "fill stage out of range");
    const ElementType entry = f.stage == 0 ? src : plan.stages[f.stage - 1].output.type;
    if (!sameType(f.type, entry))
      return c.failAt(fillAt[i], "fill type must equal the type entering its stage");
    if (!sameType(pad->fillType, res))
      return c.failAt(fillAt[i], "layout pad fill type must equal the result type");
    uint64_t bits = f.bits;
    ElementType t = f.type;
    for (size_t k = f.stage; k < plan.stages.size(); ++k) {
      const auto folded = typed::foldFill(bits, t, plan.stages[k]);
      if (!folded)
        return c.failAt(fillAt[i], "fill cannot fold through a per-channel or runtime-parameter stage");
      bits = *folded;
      t = plan.stages[k].output.type;
    }
    if (bits != pad->fillBits && !(isNaN(bits, res) && isNaN(pad->fillBits, res)))
      return c.failAt(fillAt[i], "fill fold mismatch with the layout's fused fill");
  }
  for (char filled : padFilled)
    if (!filled)
      return c.failAt(fillsAt, "layout pad without a typed fill");
  return true;
}

} // namespace

std::optional<uint32_t> peekWireVersion(const uint8_t *data, size_t size) {
  if (size < 8 || std::memcmp(data, "RPLN", 4) != 0)
    return std::nullopt;
  return static_cast<uint32_t>(data[4]) | static_cast<uint32_t>(data[5]) << 8 |
         static_cast<uint32_t>(data[6]) << 16 | static_cast<uint32_t>(data[7]) << 24;
}

DecodeResult decodePlan(const uint8_t *data, size_t size) {
  Cursor c(data, size);
  RelocationPlan plan;
  if (!readHeader(c, kWireFormatVersion, plan.symbols) || !readLayout(c, plan))
    return c.error();
  if (c.left() != 0) {
    c.fail("trailing bytes after inverse section");
    return c.error();
  }
  return plan;
}

TypedDecodeResult decodeTypedPlan(const uint8_t *data, size_t size) {
  Cursor c(data, size);
  TypedRelocationPlan plan;
  if (!readHeader(c, kTypedWireFormatVersion, plan.symbols))
    return c.error();
  const size_t nsym = plan.symbols.size();
  if (!readTensor(c, nsym, plan.source) || !readTensor(c, nsym, plan.result))
    return c.error();
  const size_t layoutAt = c.pos();
  plan.layout.symbols = plan.symbols;
  if (!readLayout(c, plan.layout))
    return c.error();
  const size_t stagesAt = c.pos();
  uint32_t nstages;
  if (!c.count(nstages, "stage count"))
    return c.error();
  std::vector<size_t> stageAt;
  plan.stages.resize(nstages);
  for (ValueStage &s : plan.stages) {
    stageAt.push_back(c.pos());
    if (!readStage(c, nsym, plan.result.extents.size(), s))
      return c.error();
  }
  const size_t fillsAt = c.pos();
  uint32_t nfills;
  if (!c.count(nfills, "fill count"))
    return c.error();
  std::vector<size_t> fillAt;
  plan.fills.resize(nfills);
  for (TypedFill &f : plan.fills) {
    fillAt.push_back(c.pos());
    if (!c.u32(f.dstAxis) || !c.u32(f.stage) || !readType(c, f.type) || !c.u64(f.bits))
      return c.error();
  }
  if (c.left() != 0) {
    c.fail("trailing bytes after fills section");
    return c.error();
  }
  if (!validateTypedPlan(c, plan, layoutAt, stagesAt, stageAt, fillsAt, fillAt))
    return c.error();
  return plan;
}

} // namespace reloc
