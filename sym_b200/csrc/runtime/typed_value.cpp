// Host scalar arithmetic for constant folding (pad fills). See
// include/reloc/TypedValue.h. Compiled with -ffp-contract=off so each float
// expression below is exactly one binary32 operation.
#include "reloc/TypedValue.h"

#include <cmath>
#include <cstring>

namespace reloc {
namespace typed {
namespace {

bool isFloat(ElementType t, uint32_t w) { return t.kind == ElementTypeKind::Float && t.bitwidth == w; }
bool isBF16(ElementType t) { return t.kind == ElementTypeKind::BFloat && t.bitwidth == 16; }
bool isS8(ElementType t) { return t.kind == ElementTypeKind::Integer && t.bitwidth == 8; }

uint32_t roundShift(uint32_t m, unsigned s) {
  if (s >= 32)
    return 0;
  const uint32_t q = m >> s, rem = m & ((1u << s) - 1u), half = 1u << (s - 1);
  return (rem > half || (rem == half && (q & 1u))) ? q + 1 : q;
}

float f32(uint32_t b) {
  float f;
  std::memcpy(&f, &b, 4);
  return f;
}
uint32_t bits32(float f) {
  uint32_t b;
  std::memcpy(&b, &f, 4);
  return b;
}

int64_t signExtend(uint64_t bits, uint32_t width) {
  if (width >= 64)
    return static_cast<int64_t>(bits);
  const uint64_t mask = (uint64_t{1} << width) - 1;
  uint64_t v = bits & mask;
  if (v >> (width - 1))
    v |= ~mask;
  return static_cast<int64_t>(v);
}

} // namespace

uint32_t byteWidth(ElementType type) {
  return (type.bitwidth == 0 || type.bitwidth % 8) ? 0 : type.bitwidth / 8;
}

bool sameType(ElementType a, ElementType b) { return a.kind == b.kind && a.bitwidth == b.bitwidth; }

uint16_t narrowF16(uint32_t x) {
  const uint32_t sign = (x >> 16) & 0x8000u, a = x & 0x7fffffffu;
  if (a > 0x7f800000u) // NaN: quiet, top payload bits kept
    return static_cast<uint16_t>(sign | 0x7e00u | ((a >> 13) & 0x3ffu));
  if (a == 0x7f800000u)
    return static_cast<uint16_t>(sign | 0x7c00u);
  const int be = static_cast<int>(a >> 23);
  const uint32_t m = be ? ((a & 0x7fffffu) | 0x800000u) : (a & 0x7fffffu);
  if (a < 0x38800000u) { // binary16 subnormal grid (quantum 2^-24)
    const int e = be ? be - 150 : -149;
    return static_cast<uint16_t>(sign | roundShift(m, static_cast<unsigned>(-24 - e)));
  }
  uint32_t r = roundShift(m, 13);
  int eh = be - 112;
  if (r == 0x800u) {
    r = 0x400u;
    ++eh;
  }
  if (eh >= 31)
    return static_cast<uint16_t>(sign | 0x7c00u);
  return static_cast<uint16_t>(sign | (static_cast<uint32_t>(eh) << 10) | (r & 0x3ffu));
}

uint16_t narrowBF16(uint32_t x) {
  const uint32_t a = x & 0x7fffffffu;
  if (a > 0x7f800000u)
    return static_cast<uint16_t>((x >> 16) | 0x40u);
  return static_cast<uint16_t>(((x >> 16) & 0x8000u) | roundShift(a, 16));
}

uint32_t widenF16(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  if (e == 0)
    return m == 0 ? sign : (sign | bits32(std::ldexp(static_cast<float>(m), -24)));
  if (e == 31)
    return sign | 0x7f800000u | (m << 13);
  return sign | ((e + 112u) << 23) | (m << 13);
}

uint32_t widenBF16(uint16_t b) { return static_cast<uint32_t>(b) << 16; }

int8_t quantizeOne(uint32_t x, float inv) {
  float t = f32(x) * inv;
  t = std::fmax(t, -128.0f);
  t = std::fmin(t, 127.0f);
  return static_cast<int8_t>(std::nearbyint(t));
}

uint32_t dequantizeOne(int8_t q, int32_t zp, float scale) {
  const float d = static_cast<float>(static_cast<int32_t>(q) - zp);
  return bits32(d * scale);
}

std::optional<uint64_t> foldFill(uint64_t bits, ElementType type, const ValueStage &stage) {
  if (!sameType(type, stage.input.type))
    return std::nullopt;
  switch (stage.transform) {
  case ValueTransformKind::Cast:
    if (isFloat(stage.input.type, 32) && isFloat(stage.output.type, 16))
      return narrowF16(static_cast<uint32_t>(bits));
    if (isFloat(stage.input.type, 32) && isBF16(stage.output.type))
      return narrowBF16(static_cast<uint32_t>(bits));
    if (isFloat(stage.input.type, 16) && isFloat(stage.output.type, 32))
      return widenF16(static_cast<uint16_t>(bits));
    if (isBF16(stage.input.type) && isFloat(stage.output.type, 32))
      return widenBF16(static_cast<uint16_t>(bits));
    return std::nullopt;
  case ValueTransformKind::Quantize:
  case ValueTransformKind::Dequantize: {
    // Only a per-tensor inline scale gives every pad one value.
    if (stage.axis >= 0 || stage.scale.kind != ParamKind::Inline || stage.scale.rank != 0 ||
        stage.scale.inlineBits.empty())
      return std::nullopt;
    const float scale = f32(static_cast<uint32_t>(stage.scale.inlineBits[0]));
    if (stage.transform == ValueTransformKind::Quantize) {
      // symmetric_rne admits only the zero point 0 (checked by the decoder).
      if (!isFloat(type, 32) || !isS8(stage.output.type))
        return std::nullopt;
      return static_cast<uint8_t>(quantizeOne(static_cast<uint32_t>(bits), 1.0f / scale));
    }
    if (!isS8(type) || !isFloat(stage.output.type, 32))
      return std::nullopt;
    int64_t zp = 0;
    if (stage.zeroPoint.kind == ParamKind::Inline) {
      if (stage.zeroPoint.rank != 0 || stage.zeroPoint.inlineBits.empty())
        return std::nullopt;
      zp = signExtend(stage.zeroPoint.inlineBits[0], stage.zeroPoint.elementType.bitwidth);
    } else if (stage.zeroPoint.kind != ParamKind::None) {
      return std::nullopt;
    }
    return dequantizeOne(static_cast<int8_t>(static_cast<uint8_t>(bits)), static_cast<int32_t>(zp), scale);
  }
  }
  return std::nullopt;
}

} // namespace typed
} // namespace reloc
