// sym_b200 -- symbol binding: a decoded plan plus {symbol -> value} (and, for
// typed plans, runtime parameter values) becomes a concrete bound plan.
//
// Entry points and result types follow the reference binder,
// libreloc/include/reloc/Bind.h:71-207 (bind :111, bindTyped :205): the same
// guards, error messages and axis coalescing, so bound layouts, footprints
// (`cuts`) and diagnostics are identical. Rebinding a symbol never touches
// device code: kernels take runtime extents and strides.
#ifndef SYM_B200_RELOC_BIND_H
#define SYM_B200_RELOC_BIND_H

#include "reloc/Plan.h"

#include <cstdint>
#include <map>
#include <optional>
#include <string>
#include <variant>
#include <vector>

namespace reloc {

using SymbolValues = std::vector<int64_t>;
using SymbolMap = std::map<std::string, int64_t>;

/// Evaluate a plan-context stream (PUSH_DIM is an error here).
bool evalExpr(const ExprStream &stream, const SymbolValues &symbols, int64_t &out, std::string &error);
/// Evaluate a channel-context stream; PUSH_DIM reads `dims`.
bool evalChannel(const ExprStream &stream, const SymbolValues &symbols, const std::vector<int64_t> &dims,
                 int64_t &out, std::string &error);

/// Layout execution strategy of the reference's host executors. Recorded for
/// API compatibility; the B200 executor chooses its own device route.
enum class Strategy { Auto, ViewNoCopy, SingleThreadSimd, MultiThreadTiled, ChunkedPipeline };

/// A pad region in coalesced destination order.
struct PadRegion {
  size_t axis;
  int64_t lo;
  int64_t hi;
  uint64_t fillBits = 0;
};

/// The concrete layout: coalesced axes in destination order with element
/// strides on both sides.
struct BoundPlan {
  std::vector<int64_t> extents;
  std::vector<int64_t> srcStrides;
  std::vector<int64_t> dstStrides;
  std::vector<uint32_t> perm;
  std::vector<PadRegion> padRegions;
  uint32_t elementSize = 0;
  int64_t totalBytes = 0;
  bool noCopy = false;
  bool typed = false; // layout of a typed plan: widths differ between ends
  Strategy strategy = Strategy::Auto;
  int64_t L = 1; // innermost contiguous run, elements
  std::vector<Alignment> requiredAlignments;
};

struct BindError {
  std::string message;
};

using BindResult = std::variant<BoundPlan, BindError>;

BindResult bind(const RelocationPlan &plan, const SymbolMap &symbols, Strategy override = Strategy::Auto);

// ----- typed binding --------------------------------------------------------

/// A runtime parameter value: element type, extents ({} rank 0, {n} rank 1)
/// and little-endian element bytes (copied by bindTyped).
struct ParameterValue {
  ElementType elementType{};
  std::vector<int64_t> extents;
  std::vector<uint8_t> bytes;
};
using ParameterMap = std::map<std::string, ParameterValue>;

struct BoundParameter {
  bool present = false;
  ElementType elementType{};
  int64_t length = 0;
  std::vector<uint8_t> bytes;
  std::string bindingName;
};

struct BoundStage {
  ValueTransformKind transform = ValueTransformKind::Cast;
  NumericPolicyKind policy = NumericPolicyKind::IeeeRne;
  StageType input;
  StageType output;
  std::vector<int64_t> shape;
  int64_t axis = -1;
  bool hasChannel = false;
  ExprStream channel;
  BoundParameter scale;
  BoundParameter zeroPoint;
};

/// Bytes at one stage boundary (0 = source side, k = output of stage k).
struct StageFootprint {
  uint32_t boundary = 0;
  ElementType elementType{};
  int64_t elements = 0;
  int64_t bytes = 0;
};

struct TypedBoundPlan {
  BoundPlan layout;
  std::vector<int64_t> sourceExtents;
  std::vector<int64_t> resultExtents;
  ElementType sourceType{};
  ElementType resultType{};
  SymbolValues symbols;
  std::vector<BoundStage> stages;
  std::vector<TypedFill> fills;
  std::vector<StageFootprint> cuts;
  int64_t sourceBytes = 0;
  int64_t destinationBytes = 0;
  int64_t parameterBytes = 0;
  std::vector<std::string> requirements;
};

using TypedBindResult = std::variant<TypedBoundPlan, BindError>;

TypedBindResult bindTyped(const TypedRelocationPlan &plan, const SymbolMap &symbols,
                          const ParameterMap &parameters);

} // namespace reloc

#endif
