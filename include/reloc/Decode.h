// sym_b200 -- strict wire decoder (v0 layout plans, v1 typed plans).
//
// Same entry points and the same diagnostics (byte offset + message) as the
// reference decoder, libreloc/include/reloc/Decode.h:35-52, so callers that
// branch on a DecodeError keep working. Every count is checked against the
// remaining bytes before anything is allocated.
#ifndef SYM_B200_RELOC_DECODE_H
#define SYM_B200_RELOC_DECODE_H

#include "reloc/Plan.h"

#include <cstddef>
#include <cstdint>
#include <optional>
#include <string>
#include <variant>

namespace reloc {

inline constexpr uint32_t kWireFormatVersion = 0;
inline constexpr uint32_t kTypedWireFormatVersion = 1;

struct DecodeError {
  size_t offset = 0;
  std::string message;
};

using DecodeResult = std::variant<RelocationPlan, DecodeError>;
using TypedDecodeResult = std::variant<TypedRelocationPlan, DecodeError>;

/// Decode a wire v0 plan; any other version fails at byte offset 4.
DecodeResult decodePlan(const uint8_t *data, size_t size);

/// Decode a wire v1 typed plan with every decoder-enforced invariant of the
/// format (stage signatures, parameter domains, fill folding).
TypedDecodeResult decodeTypedPlan(const uint8_t *data, size_t size);

/// Version field of a blob with a valid header, else nullopt.
std::optional<uint32_t> peekWireVersion(const uint8_t *data, size_t size);

} // namespace reloc

#endif
