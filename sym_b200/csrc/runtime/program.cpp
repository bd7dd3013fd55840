// The checked typed program (include/reloc/TypedExecute.h). Validation and
// parameter materialization follow libreloc/src/TypedExecute.cpp:293-470.
#include "reloc/TypedExecute.h"
#include "reloc/TypedValue.h"

#include <cmath>
#include <cstring>

namespace reloc {
namespace typed {
namespace {

ExecutionError err(const char *code, std::string msg) { return ExecutionError{code, std::move(msg)}; }
bool isF32(ElementType t) { return t.kind == ElementTypeKind::Float && t.bitwidth == 32; }
bool isF16(ElementType t) { return t.kind == ElementTypeKind::Float && t.bitwidth == 16; }
bool isBF16(ElementType t) { return t.kind == ElementTypeKind::BFloat && t.bitwidth == 16; }
bool isS8(ElementType t) { return t.kind == ElementTypeKind::Integer && t.bitwidth == 8; }

bool scales(const BoundParameter &p, std::vector<float> &out, std::string &why) {
  if (!p.present)
    return (why = "scale is absent"), false;
  if (!isF32(p.elementType))
    return (why = "scale is not f32"), false;
  if (p.bytes.size() != static_cast<size_t>(p.length) * 4)
    return (why = "scale byte size disagrees with its length"), false;
  out.resize(static_cast<size_t>(p.length));
  std::memcpy(out.data(), p.bytes.data(), out.size() * 4);
  for (float v : out)
    if (!std::isfinite(v) || v <= 0.0f)
      return (why = "scale is not finite and strictly positive"), false;
  return true;
}

bool zeroPoints(const BoundParameter &p, std::vector<int32_t> &out, std::string &why) {
  if (!p.present) {
    out.assign(1, 0);
    return true;
  }
  const uint32_t bw = p.elementType.bitwidth;
  if (p.elementType.kind != ElementTypeKind::Integer || bw == 0 || bw > 64 || bw % 8)
    return (why = "zero point is not a byte-multiple integer type"), false;
  const size_t w = bw / 8;
  if (p.bytes.size() != static_cast<size_t>(p.length) * w)
    return (why = "zero point byte size disagrees with its length"), false;
  out.resize(static_cast<size_t>(p.length));
  for (int64_t i = 0; i < p.length; ++i) {
    uint64_t raw = 0;
    std::memcpy(&raw, p.bytes.data() + i * static_cast<int64_t>(w), w);
    const unsigned sh = 64 - bw;
    const int64_t v = static_cast<int64_t>(raw << sh) >> sh;
    if (v < -128 || v > 127)
      return (why = "zero point outside [-128, 127]"), false;
    out[static_cast<size_t>(i)] = static_cast<int32_t>(v);
  }
  return true;
}

uint64_t applyConstant(const StageArithmetic &s, uint64_t bits) {
  switch (s.transform) {
  case ValueTransformKind::Cast:
    if (isF32(s.input))
      return isBF16(s.output) ? narrowBF16(static_cast<uint32_t>(bits)) : narrowF16(static_cast<uint32_t>(bits));
    return isBF16(s.input) ? widenBF16(static_cast<uint16_t>(bits)) : widenF16(static_cast<uint16_t>(bits));
  case ValueTransformKind::Quantize:
    return static_cast<uint8_t>(quantizeOne(static_cast<uint32_t>(bits), s.invScale[0]));
  case ValueTransformKind::Dequantize:
    return dequantizeOne(static_cast<int8_t>(static_cast<uint8_t>(bits)), s.zeroPoint[0], s.scale[0]);
  }
  return bits;
}

} // namespace

std::variant<Program, ExecutionError> prepareProgram(const TypedBoundPlan &plan) {
  Program prog;
  prog.plan = plan;
  const size_t rank = plan.resultExtents.size();
  prog.resultStrides.assign(rank, 1);
  for (size_t j = rank; j-- > 1;)
    prog.resultStrides[j - 1] = prog.resultStrides[j] * plan.resultExtents[j];
  prog.resultElements = 1;
  for (int64_t e : plan.resultExtents)
    prog.resultElements *= e;
  prog.sourceElements = 1;
  for (int64_t e : plan.sourceExtents)
    prog.sourceElements *= e;

  for (size_t k = 0; k < plan.stages.size(); ++k) {
    const BoundStage &b = plan.stages[k];
    StageArithmetic s;
    s.transform = b.transform;
    s.policy = b.policy;
    s.input = b.input.type;
    s.output = b.output.type;
    const std::string where = "stage " + std::to_string(k) + ": ";
    std::string why;
    if (b.transform == ValueTransformKind::Cast) {
      const bool narrow = isF32(s.input) && (isF16(s.output) || isBF16(s.output)) && b.policy == NumericPolicyKind::IeeeRne;
      const bool widen = (isF16(s.input) || isBF16(s.input)) && isF32(s.output) && b.policy == NumericPolicyKind::Exact;
      if (!narrow && !widen)
        return err("unsupported_stage", where + "only cast f32->f16/bf16 ieee_rne and f16/bf16->f32 exact have a "
                                                "reference implementation");
    } else if (b.transform == ValueTransformKind::Quantize) {
      if (!isF32(s.input) || !isS8(s.output) || b.policy != NumericPolicyKind::SymmetricRne)
        return err("unsupported_stage", where + "only quantize f32->s8 symmetric_rne has a reference implementation");
      if (!scales(b.scale, s.scale, why))
        return err("invalid_parameter", where + why);
      std::vector<int32_t> zp;
      if (!zeroPoints(b.zeroPoint, zp, why))
        return err("invalid_parameter", where + why);
      for (int32_t z : zp)
        if (z != 0)
          return err("invalid_parameter", where + "symmetric_rne admits only zero point 0");
      s.invScale.resize(s.scale.size());
      for (size_t i = 0; i < s.scale.size(); ++i)
        s.invScale[i] = 1.0f / s.scale[i]; // fl32(1/scale), formed once, on the host
    } else {
      if (!isS8(s.input) || !isF32(s.output) || b.policy != NumericPolicyKind::Affine)
        return err("unsupported_stage", where + "only dequantize s8->f32 affine has a reference implementation");
      if (!scales(b.scale, s.scale, why))
        return err("invalid_parameter", where + why);
      if (!zeroPoints(b.zeroPoint, s.zeroPoint, why))
        return err("invalid_parameter", where + why);
    }
    s.perChannel = b.hasChannel;
    if (b.hasChannel) {
      if (s.scale.empty())
        return err("invalid_parameter", where + "per-channel stage without scales");
      s.channelLength = static_cast<int64_t>(s.scale.size());
      if (s.zeroPoint.size() > 1 && s.zeroPoint.size() != s.scale.size())
        return err("invalid_parameter", where + "zero point length disagrees with the scale");
      const ExprStream &ch = b.channel;
      if (!ch.empty() && ch.front().op == ExprOp::PushDim && ch.front().value >= 0 &&
          static_cast<size_t>(ch.front().value) < rank) {
        s.channelDim = static_cast<uint32_t>(ch.front().value);
        s.channelIsDim = ch.size() == 1;
        // (dN mod M) with M >= the coordinate's extent is the coordinate itself.
        if (ch.size() == 3 && ch[2].op == ExprOp::Mod &&
            (ch[1].op == ExprOp::PushConst || ch[1].op == ExprOp::PushSym)) {
          int64_t m = 0;
          if (evalChannel({ch[1]}, plan.symbols, {}, m, why) && m > 0 && plan.resultExtents[s.channelDim] <= m)
            s.channelIsDim = true;
        }
      }
      prog.needsCoordinates = true;
    } else if (s.scale.size() > 1 || s.zeroPoint.size() > 1) {
      return err("invalid_parameter", where + "per-tensor stage with more than one parameter");
    }
    prog.stages.push_back(std::move(s));
  }
  return prog;
}

ElementType typeAt(const Program &p, uint32_t boundary) {
  return boundary == 0 ? p.plan.sourceType : p.stages[boundary - 1].output;
}

uint32_t widthAt(const Program &p, uint32_t boundary) { return byteWidth(typeAt(p, boundary)); }

bool padsSettledBy(const Program &p, uint32_t boundary) {
  for (const TypedFill &f : p.plan.fills)
    if (f.stage > boundary)
      return false;
  return true;
}

std::variant<std::optional<uint64_t>, ExecutionError> fillAt(const Program &p, uint32_t boundary) {
  if (boundary > p.stages.size())
    return err("invalid_boundary", "boundary beyond the last stage");
  if (p.plan.fills.empty())
    return std::optional<uint64_t>();
  std::optional<uint64_t> agreed;
  for (const TypedFill &f : p.plan.fills) {
    if (f.stage > boundary)
      return err("pad_not_entered", "a pad enters at stage " + std::to_string(f.stage) + ", after boundary " +
                                        std::to_string(boundary));
    uint64_t bits = f.bits;
    ElementType t = f.type;
    for (uint32_t k = f.stage; k < boundary; ++k) {
      const StageArithmetic &s = p.stages[k];
      if (s.perChannel)
        return err("fill_crosses_channel_stage", "a pad fill would cross per-channel stage " + std::to_string(k));
      if (!sameType(t, s.input))
        return err("fill_type_mismatch", "pad fill type disagrees with stage " + std::to_string(k));
      bits = applyConstant(s, bits);
      t = s.output;
    }
    if (!sameType(t, typeAt(p, boundary)))
      return err("fill_type_mismatch", "pad fill type disagrees with boundary " + std::to_string(boundary));
    if (agreed && *agreed != bits)
      return err("mixed_fills_unsupported", "pads carry different values at boundary " + std::to_string(boundary));
    agreed = bits;
  }
  if (boundary == p.stages.size() && !p.plan.layout.padRegions.empty() &&
      p.plan.layout.padRegions.front().fillBits != *agreed)
    return err("fill_mismatch", "folded fill disagrees with the layout's fused fill");
  return agreed;
}

int64_t bytesAt(const Program &p, uint32_t boundary, bool resultLayout) {
  return (resultLayout ? p.resultElements : p.sourceElements) * static_cast<int64_t>(widthAt(p, boundary));
}

} // namespace typed
} // namespace reloc
