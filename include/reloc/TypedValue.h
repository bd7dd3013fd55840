// sym_b200 -- host-side scalar reference arithmetic used by the decoder to
// verify fused pad fills, and by the runtime to fold fills to a boundary.
//
// Mirrors libreloc/include/reloc/TypedValue.h (foldFill, byteWidth) with the
// contract of libreloc docs/reloc-typed-semantics.md §3. Only constants are
// folded here: the decoder needs one value per pad. Element data is never
// converted on the host -- that is the device's job.
#ifndef SYM_B200_RELOC_TYPEDVALUE_H
#define SYM_B200_RELOC_TYPEDVALUE_H

#include "reloc/Plan.h"

#include <cstdint>
#include <optional>

namespace reloc {
namespace typed {

/// Byte width of a wire element type, 0 when not a positive multiple of 8.
uint32_t byteWidth(ElementType type);
bool sameType(ElementType lhs, ElementType rhs);

/// Fold one constant through one stage (casts always; quantize/dequantize
/// only with inline per-tensor parameters). nullopt when not foldable.
std::optional<uint64_t> foldFill(uint64_t bits, ElementType type, const ValueStage &stage);

/// Scalar contract (docs/reloc-typed-semantics.md §3.1-§3.6).
uint16_t narrowF16(uint32_t f32Bits);
uint16_t narrowBF16(uint32_t f32Bits);
uint32_t widenF16(uint16_t h);
uint32_t widenBF16(uint16_t b);
int8_t quantizeOne(uint32_t f32Bits, float invScale);
uint32_t dequantizeOne(int8_t q, int32_t zeroPoint, float scale);

} // namespace typed
} // namespace reloc

#endif
