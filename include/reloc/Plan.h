// sym_b200 -- B200-native executor for libreloc relocation plans.
//
// The decoded plan model. It mirrors the sections of the wire format
// (libreloc docs/reloc-plan-format.md, v0 layout plans and v1 typed plans)
// field for field, because callers written against the reference's
// libreloc/include/reloc/Plan.h:20-191 hand these structs around and the wire
// format fixes their content. Expressions stay as postfix token streams; the
// binder evaluates them with a small stack machine.
#ifndef SYM_B200_RELOC_PLAN_H
#define SYM_B200_RELOC_PLAN_H

#include <cstdint>
#include <string>
#include <vector>

namespace reloc {

/// Wire opcodes of a symbolic expression (values are the wire bytes).
enum class ExprOp : uint8_t {
  PushSym = 0x00,
  PushConst = 0x01,
  Add = 0x02,
  Sub = 0x03,
  Mul = 0x04,
  FloorDiv = 0x05,
  Mod = 0x06,
  PushDim = 0x07,
};

/// One postfix token; `value` is the symbol index, the constant or the
/// coordinate index (0 for operators).
struct ExprToken {
  ExprOp op;
  int64_t value;
};
using ExprStream = std::vector<ExprToken>;

enum class ElementTypeKind : uint8_t { Float = 0, BFloat = 1, Integer = 2, Index = 3 };

struct ElementType {
  ElementTypeKind kind;
  uint32_t bitwidth;
};

/// Symbolic tensor descriptor; empty `strides` means row-major.
struct TensorDesc {
  std::vector<ExprStream> extents;
  std::vector<ExprStream> strides;
  ExprStream offset;
  ElementType elementType;
};

/// One plan axis, in destination order.
struct Axis {
  std::string name;
  ExprStream extent;
  ExprStream srcStride;
  ExprStream dstStride;
};

/// Leading/trailing pad widths on one destination axis with the fill value
/// (bit pattern zero-extended to 64 bits).
struct PadFill {
  uint32_t dstAxis;
  ExprStream lo;
  ExprStream hi;
  ElementType fillType;
  uint64_t fillBits;
};

struct Divisibility {
  ExprStream expr;
  int64_t divisor;
};

struct Alignment {
  uint32_t axis;
  int64_t bytes;
};

/// Wire v0: a layout-only relocation plan.
struct RelocationPlan {
  std::vector<std::string> symbols;
  TensorDesc src;
  TensorDesc dst;
  std::vector<uint32_t> perm;
  std::vector<Axis> axes;
  std::vector<PadFill> padFill;
  std::vector<Divisibility> divisibility;
  std::vector<Alignment> alignment;
  std::vector<uint8_t> contiguity;
  bool noCopy = false;
  bool runtimePadCheck = false;
  std::vector<ExprStream> inverse;
};

// ----- wire v1: typed plans -------------------------------------------------

enum class ValueTransformKind : uint8_t { Cast = 0, Quantize = 1, Dequantize = 2 };
enum class NumericPolicyKind : uint8_t { IeeeRne = 0, Exact = 1, SymmetricRne = 2, Affine = 3 };
enum class Signedness : uint8_t { Signless = 0, Signed = 1, Unsigned = 2 };

struct StageType {
  ElementType type;
  Signedness signedness = Signedness::Signless;
};

enum class ParamKind : uint8_t { None = 0, Inline = 1, Binding = 2 };

/// A quantization parameter as declared: absent, inline bit patterns, or a
/// runtime binding identified by name.
struct StageParam {
  ParamKind kind = ParamKind::None;
  uint8_t rank = 0;
  ElementType elementType{};
  std::vector<uint64_t> inlineBits;
  std::string bindingName;
  std::vector<ExprStream> bindingExtents;
};

/// One value stage: transform, policy, types, operand shape, parameters and
/// the channel map (an expression over logical result coordinates).
struct ValueStage {
  ValueTransformKind transform = ValueTransformKind::Cast;
  NumericPolicyKind policy = NumericPolicyKind::IeeeRne;
  StageType input;
  StageType output;
  std::vector<ExprStream> shape;
  StageParam scale;
  StageParam zeroPoint;
  int64_t axis = -1;
  bool hasChannel = false;
  ExprStream channel;
};

/// An original pad fill and the stage boundary it entered at.
struct TypedFill {
  uint32_t dstAxis = 0;
  uint32_t stage = 0;
  ElementType type{};
  uint64_t bits = 0;
};

struct TypedRelocationPlan {
  std::vector<std::string> symbols;
  TensorDesc source;
  TensorDesc result;
  RelocationPlan layout;
  std::vector<ValueStage> stages;
  std::vector<TypedFill> fills;
};

} // namespace reloc

#endif
